"""The tuner (``kernelforge/tuning/tuner.py:1-370``).

    problem -> candidates -> filters -> launch+verify -> benchmark -> rank -> persist

Two guarantees carry over unchanged. A candidate that fails the correctness
gate is never ranked, however fast (skipping work is fast). And every
candidate is verified before any is timed, so no first-launch cost lands in a
measurement. With native kernels there is no JIT compile: "compile" is the
first launch, and a config the library cannot run surfaces as
``OutOfResources`` -> ``compile_error``. After each verification the device
status word is read, so a kernel whose bounded wait gave up is recorded as a
``runtime_error`` instead of poisoning the rest of the sweep.
"""

from __future__ import annotations

import time
from collections.abc import Callable
from dataclasses import dataclass, field

import torch

from kernelo_b200.benchmark import metrics
from kernelo_b200.benchmark.runner import DEFAULT_ITERATIONS, DEFAULT_WARMUP, TimingResult, benchmark
from kernelo_b200.db import Measurement, ResultsDB
from kernelo_b200.kernels.base import Operator
from kernelo_b200.runtime.env import Environment, capture_environment, device_caps, require_cuda
from kernelo_b200.testing import VerificationResult, exact_fp32_matmul, verify
from kernelo_b200.tuning.cache import ConfigCache
from kernelo_b200.tuning.config import KernelConfig, Problem

STATUS_OK = "ok"
STATUS_COMPILE_ERROR = "compile_error"
STATUS_RUNTIME_ERROR = "runtime_error"
STATUS_INCORRECT = "incorrect"
STATUS_OOM = "out_of_memory"

_MAX_ERROR_CHARS = 400


def _classify(exc: BaseException) -> tuple[str, str]:
    """Status and short message for an exception raised by a candidate."""
    name = type(exc).__name__
    text = " ".join(str(exc).split())[:_MAX_ERROR_CHARS]
    if "OutOfMemory" in name:
        return STATUS_OOM, text
    if "OutOfResources" in name or "Compil" in name or "Resource" in name:
        return STATUS_COMPILE_ERROR, f"{name}: {text}"
    return STATUS_RUNTIME_ERROR, f"{name}: {text}"


@dataclass(frozen=True)
class CandidateOutcome:
    config: KernelConfig
    status: str
    verification: VerificationResult | None = None
    timing: TimingResult | None = None
    error: str = ""

    @property
    def ok(self) -> bool:
        return self.status == STATUS_OK

    @property
    def median_ms(self) -> float:
        if self.timing is None:
            raise ValueError(f"candidate {self.config!r} has no timing ({self.status})")
        return self.timing.median_ms


@dataclass
class TuningResult:
    problem: Problem
    environment: Environment
    generated: int
    feasible: int
    outcomes: tuple[CandidateOutcome, ...]
    baselines: dict[str, TimingResult]
    flops: int
    bytes_moved: int
    elapsed_s: float
    memory_bound: bool = False
    rejections: tuple[tuple[KernelConfig, str], ...] = field(default=(), repr=False)

    @property
    def tested(self) -> int:
        return len(self.outcomes)

    @property
    def correct(self) -> int:
        return sum(o.ok for o in self.outcomes)

    def ranked(self) -> list[CandidateOutcome]:
        """Correct candidates, fastest median first."""
        return sorted((o for o in self.outcomes if o.ok and o.timing is not None), key=lambda o: o.median_ms)

    @property
    def best(self) -> CandidateOutcome | None:
        ranked = self.ranked()
        return ranked[0] if ranked else None

    @property
    def best_config(self) -> KernelConfig | None:
        best = self.best
        return None if best is None else best.config

    def tflops(self, ms: float) -> float:
        return metrics.tflops(self.flops, ms)

    def gbps(self, ms: float) -> float:
        return metrics.gbps(self.bytes_moved, ms)

    def speedup_over(self, label: str) -> float | None:
        best = self.best
        if best is None or label not in self.baselines:
            return None
        return metrics.speedup(self.baselines[label].median_ms, best.median_ms)

    def status_counts(self) -> dict[str, int]:
        counts: dict[str, int] = {}
        for o in self.outcomes:
            counts[o.status] = counts.get(o.status, 0) + 1
        return counts


def _outcome_from_row(config: KernelConfig, row: dict) -> CandidateOutcome:
    """A stored measurement as a candidate outcome (times are kept in us)."""
    timing = None
    if row["median_us"] is not None:
        ms = {k: (row[f"{k}_us"] or 0.0) / 1e3 for k in ("median", "mean", "std", "min", "max", "p95", "p99")}
        timing = TimingResult(ms["median"], ms["mean"], ms["std"], ms["min"], ms["max"], ms["p95"], ms["p99"],
                              int(row["warmup"] or 0), int(row["iterations"] or 0), row["timer"] or "",
                              bool(row["flushed_l2"]))
    verification = None
    if row["correct"] is not None:
        verification = VerificationResult(bool(row["correct"]), row["rel_error"] or 0.0, 0.0, 0, 0, 0.0,
                                          "" if row["correct"] else row["error"])
    return CandidateOutcome(config=config, status=row["status"], verification=verification, timing=timing,
                            error=row["error"] or "")


def _device_status_check(device: torch.device) -> None:
    if device.type != "cuda":
        return
    from kernelo_b200.runtime import native

    native.raise_on_device_status(device.index)


class Tuner:
    """Runs the tuning pipeline for any :class:`Operator`."""

    def __init__(
        self,
        *,
        warmup: int = DEFAULT_WARMUP,
        iterations: int = DEFAULT_ITERATIONS,
        flush_l2: bool = True,
        max_candidates: int | None = None,
        measure_baselines: bool = True,
        seed: int = 0,
        db: ResultsDB | None = None,
        cache: ConfigCache | None = None,
        log: Callable[[str], None] | None = None,
        candidate_filter: Callable[[int, KernelConfig], bool] | None = None,
        resume: bool = False,
    ) -> None:
        self.warmup = warmup
        self.iterations = iterations
        self.flush_l2 = flush_l2
        self.max_candidates = max_candidates
        self.measure_baselines = measure_baselines
        self.seed = seed
        self.db = db
        self.cache = cache
        self._log = log
        #: (index, config) -> keep? Used to shard one candidate list over workers.
        self.candidate_filter = candidate_filter
        #: Reuse the outcome of every candidate the database already holds for
        #: this problem and device, so an interrupted sweep continues where it
        #: stopped (needs ``db``).
        self.resume = resume
        if resume and db is None:
            raise ValueError("resume needs a results database")

    def log(self, message: str) -> None:
        if self._log is not None:
            self._log(message)

    def tune(
        self, operator: Operator, problem: Problem, *, device: torch.device | str | None = None
    ) -> TuningResult:
        started = time.perf_counter()
        target = torch.device(device) if device is not None else require_cuda()
        env = capture_environment(target)
        caps = device_caps(target)
        cset = operator.search_space().generate(problem, caps, max_candidates=self.max_candidates)
        candidates = list(cset.candidates)
        if self.candidate_filter is not None:
            candidates = [c for i, c in enumerate(candidates) if self.candidate_filter(i, c)]
        inputs = operator.make_inputs(problem, target, seed=self.seed)

        reused: dict[KernelConfig, CandidateOutcome] = {}
        if self.resume:
            for c in candidates:
                row = self.db.latest_result(problem, c, device_key=env.device_key)
                if row is not None:
                    reused[c] = _outcome_from_row(c, row)
            if reused:
                self.log(f"Resuming: {len(reused)} of {len(candidates)} candidates already measured")
        fresh = [c for c in candidates if c not in reused]

        with exact_fp32_matmul():
            reference = operator.reference(*inputs)
            self.log(f"Verifying candidates... ({len(fresh)} to check)")
            verified = [self._verify_candidate(operator, c, inputs, reference, problem) for c in fresh]
            self.log(f"{sum(o.ok for o in verified)} / {len(fresh)} configurations passed correctness")
            self.log("Benchmarking...")
            measured = {o.config: self._time_candidate(operator, o, inputs, target) for o in verified}
            timed = [reused[c] if c in reused else measured[c] for c in candidates]
            baselines = (
                self._measure_baselines(operator, problem, inputs, reference, target)
                if self.measure_baselines
                else {}
            )

        result = TuningResult(
            problem=problem,
            environment=env,
            generated=cset.generated,
            feasible=cset.feasible,
            outcomes=tuple(timed),
            baselines=baselines,
            flops=operator.flops(problem),
            bytes_moved=operator.bytes_moved(problem),
            elapsed_s=time.perf_counter() - started,
            memory_bound=operator.is_memory_bound(),
            rejections=cset.rejected,
        )
        self._persist(result, env, skip=set(reused))
        return result

    # stages -------------------------------------------------------------------
    def _verify_candidate(self, operator, config, inputs, reference, problem) -> CandidateOutcome:
        try:
            output = operator.run(config, *inputs)
            _device_status_check(output.device)
        except Exception as exc:  # one failing candidate must not end the sweep
            status, message = _classify(exc)
            return CandidateOutcome(config=config, status=status, error=message)
        check = verify(reference, output, dtype=problem.dtype)
        return CandidateOutcome(
            config=config,
            status=STATUS_OK if check.passed else STATUS_INCORRECT,
            verification=check,
            error="" if check.passed else check.reason,
        )

    def _time_candidate(self, operator, outcome, inputs, device) -> CandidateOutcome:
        if not outcome.ok:
            return outcome
        try:
            timing = benchmark(
                lambda: operator.run(outcome.config, *inputs),
                warmup=self.warmup,
                iterations=self.iterations,
                device=device,
                flush_l2=self.flush_l2,
            )
            _device_status_check(device)
        except Exception as exc:
            status, message = _classify(exc)
            return CandidateOutcome(config=outcome.config, status=status,
                                    verification=outcome.verification, error=message)
        return CandidateOutcome(config=outcome.config, status=STATUS_OK,
                                verification=outcome.verification, timing=timing)

    def _measure_baselines(self, operator, problem, inputs, reference, device) -> dict[str, TimingResult]:
        """Every comparison label, gated and timed exactly like the candidates."""
        out: dict[str, TimingResult] = {}
        for label, fn in operator.baselines(problem, inputs).items():
            try:
                check = verify(reference, fn(), dtype=problem.dtype)
                if not check.passed:
                    self.log(f"  baseline {label} disagrees with the reference: {check.reason}")
                    continue
                out[label] = benchmark(fn, warmup=self.warmup, iterations=self.iterations,
                                       device=device, flush_l2=self.flush_l2)
            except Exception as exc:
                self.log(f"  baseline {label} unavailable: {_classify(exc)[1]}")
        return out

    def _persist(self, result: TuningResult, env: Environment, *, skip: set[KernelConfig] = frozenset()) -> None:
        best = result.best
        if self.cache is not None and best is not None:
            self.cache.put(
                result.problem,
                env.device_key,
                best.config,
                median_us=best.timing.median_us if best.timing else None,
                timestamp=env.timestamp,
                candidates_tested=result.tested,
            )
        if self.db is None:
            return
        from kernelo_b200 import __version__

        run_id = self.db.start_run(env, notes="tune", version=__version__)
        rows = []
        for o in result.outcomes:
            if o.config in skip:  # reused from an earlier run: its row is already there
                continue
            ms = o.timing.median_ms if o.timing else None
            rows.append(
                Measurement(
                    label="kernelforge",
                    status=o.status,
                    config=o.config,
                    verification=o.verification,
                    timing=o.timing,
                    tflops=result.tflops(ms) if ms else None,
                    gbps=result.gbps(ms) if ms else None,
                    error=o.error,
                )
            )
        for label, timing in result.baselines.items():
            rows.append(
                Measurement(
                    label=label,
                    status=STATUS_OK,
                    timing=timing,
                    tflops=result.tflops(timing.median_ms),
                    gbps=result.gbps(timing.median_ms),
                )
            )
        self.db.record_many(run_id, result.problem, rows)
