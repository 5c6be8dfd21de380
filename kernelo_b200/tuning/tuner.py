"""The tuning pipeline: candidates -> gate -> timing -> ranking -> persistence.

The reference's ``Tuner.tune`` (``kernelforge/tuning/tuner.py:184-239``) fixes
the contract this keeps: a candidate that fails the correctness gate is never
ranked however fast it is; every candidate is gated before any is timed, so
no first-launch cost lands in a measurement; one failing candidate never ends
the sweep; failures are recorded with the statuses ``compile_error``,
``runtime_error``, ``incorrect`` and ``out_of_memory``; the winner goes to the
config cache and every outcome to the results database.

The structure is this project's own. A :class:`_Sweep` holds one tuning
run's state and walks it through explicit stages -- :meth:`~_Sweep.plan`
(generate, filter, split off what a resumed run already measured),
:meth:`~_Sweep.gate`, :meth:`~_Sweep.time`, :meth:`~_Sweep.compare` -- and
:class:`Tuner` is the configuration plus persistence around it. With native
kernels there is no JIT step: "compile" is the first launch, and a config
the library refuses raises ``OutOfResources``, which classifies as
``compile_error``. After every launch the device status word is read, so a
kernel whose bounded wait gave up is a ``runtime_error`` of that candidate
instead of a poisoned sweep.
"""

from __future__ import annotations

import time
from collections import Counter
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

#: Exception-class-name fragments and the status each maps to, first match
#: wins. Names, not types: the native layer's ``OutOfResources`` and torch's
#: ``OutOfMemoryError`` are matched the way the reference matches Triton's.
_STATUS_BY_NAME: tuple[tuple[tuple[str, ...], str], ...] = (
    (("OutOfMemory",), STATUS_OOM),
    (("OutOfResources", "Compil", "Resource"), STATUS_COMPILE_ERROR),
)


def _classify(exc: BaseException) -> tuple[str, str]:
    """Status and a one-line message for an exception raised by a candidate."""
    kind = type(exc).__name__
    text = " ".join(str(exc).split())[:_MAX_ERROR_CHARS]
    status = next((s for fragments, s in _STATUS_BY_NAME if any(f in kind for f in fragments)),
                  STATUS_RUNTIME_ERROR)
    return status, text if status == STATUS_OOM else f"{kind}: {text}"


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
        if self.timing is not None:
            return self.timing.median_ms
        raise ValueError(f"candidate {self.config!r} has no timing ({self.status})")


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
        return sum(1 for o in self.outcomes if o.ok)

    def ranked(self) -> list[CandidateOutcome]:
        """Correct, timed candidates, fastest median first (stable for ties)."""
        timed = [o for o in self.outcomes if o.ok and o.timing is not None]
        return sorted(timed, key=lambda o: o.timing.median_ms)

    @property
    def best(self) -> CandidateOutcome | None:
        return next(iter(self.ranked()), None)

    @property
    def best_config(self) -> KernelConfig | None:
        return self.best.config if self.best is not None else None

    def tflops(self, ms: float) -> float:
        return metrics.tflops(self.flops, ms)

    def gbps(self, ms: float) -> float:
        return metrics.gbps(self.bytes_moved, ms)

    def speedup_over(self, label: str) -> float | None:
        best, other = self.best, self.baselines.get(label)
        if best is None or other is None:
            return None
        return metrics.speedup(other.median_ms, best.median_ms)

    def status_counts(self) -> dict[str, int]:
        return dict(Counter(o.status for o in self.outcomes))


def _outcome_from_row(config: KernelConfig, row: dict) -> CandidateOutcome:
    """A stored ``results`` row (times in microseconds) as a candidate outcome."""
    timing = None
    if row["median_us"] is not None:
        stats = [(row[f"{name}_us"] or 0.0) / 1e3 for name in ("median", "mean", "std", "min", "max", "p95", "p99")]
        timing = TimingResult(*stats, int(row["warmup"] or 0), int(row["iterations"] or 0), row["timer"] or "",
                              bool(row["flushed_l2"]))
    verification = None
    if row["correct"] is not None:
        passed = bool(row["correct"])
        verification = VerificationResult(passed, row["rel_error"] or 0.0, 0.0, 0, 0, 0.0,
                                          "" if passed else row["error"])
    return CandidateOutcome(config, row["status"], verification, timing, row["error"] or "")


def _check_device_status(device: torch.device) -> None:
    """Raise if a kernel's bounded wait gave up since the last check."""
    if device.type == "cuda":
        from kernelo_b200.runtime import native

        native.raise_on_device_status(device.index)


def _time_gated(tuner: Tuner, operator: Operator, outcome: CandidateOutcome, inputs, device: torch.device
                ) -> CandidateOutcome:
    """Time a gated candidate with the tuner's settings (failures pass through)."""
    if not outcome.ok:
        return outcome
    try:
        timing = benchmark(lambda: operator.run(outcome.config, *inputs), warmup=tuner.warmup,
                           iterations=tuner.iterations, device=device, flush_l2=tuner.flush_l2)
        _check_device_status(device)
    except Exception as exc:  # noqa: BLE001 - a failure is this candidate's outcome
        status, message = _classify(exc)
        return CandidateOutcome(outcome.config, status, outcome.verification, error=message)
    return CandidateOutcome(outcome.config, STATUS_OK, outcome.verification, timing)


class _Sweep:
    """One tuning run's state, walked through the stages in order."""

    def __init__(self, tuner: Tuner, operator: Operator, problem: Problem, device: torch.device) -> None:
        self.tuner, self.operator, self.problem, self.device = tuner, operator, problem, device
        self.env = capture_environment(device)
        self.started = time.perf_counter()
        self.reused: dict[KernelConfig, CandidateOutcome] = {}

    def plan(self) -> None:
        """The candidate list (generated, filtered, budgeted, dealt to this
        worker) and, when resuming, the outcomes already on record."""
        tuner = self.tuner
        self.space = self.operator.search_space().generate(self.problem, device_caps(self.device),
                                                           max_candidates=tuner.max_candidates)
        keep = tuner.candidate_filter or (lambda index, config: True)
        self.candidates = [c for i, c in enumerate(self.space.candidates) if keep(i, c)]
        if tuner.resume:
            for config in self.candidates:
                row = tuner.db.latest_result(self.problem, config, device_key=self.env.device_key)
                if row is not None:
                    self.reused[config] = _outcome_from_row(config, row)
            if self.reused:
                tuner.log(f"Resuming: {len(self.reused)} of {len(self.candidates)} candidates already measured")
        self.inputs = self.operator.make_inputs(self.problem, self.device, seed=tuner.seed)

    def _run_checked(self, config: KernelConfig) -> torch.Tensor:
        output = self.operator.run(config, *self.inputs)
        _check_device_status(output.device)
        return output

    def gate(self) -> list[CandidateOutcome]:
        """Launch and verify every new candidate before anything is timed."""
        fresh = [c for c in self.candidates if c not in self.reused]
        self.tuner.log(f"Verifying candidates... ({len(fresh)} to check)")
        self.reference = self.operator.reference(*self.inputs)
        gated = []
        for config in fresh:
            try:
                output = self._run_checked(config)
            except Exception as exc:  # noqa: BLE001 - one failing candidate must not end the sweep
                status, message = _classify(exc)
                gated.append(CandidateOutcome(config, status, error=message))
                continue
            check = verify(self.reference, output, dtype=self.problem.dtype)
            gated.append(CandidateOutcome(config, STATUS_OK if check.passed else STATUS_INCORRECT, check,
                                          error="" if check.passed else check.reason))
        self.tuner.log(f"{sum(o.ok for o in gated)} / {len(fresh)} configurations passed correctness")
        return gated

    def time(self, gated: list[CandidateOutcome]) -> tuple[CandidateOutcome, ...]:
        self.tuner.log("Benchmarking...")
        measured = {o.config: _time_gated(self.tuner, self.operator, o, self.inputs, self.device) for o in gated}
        return tuple(self.reused.get(c) or measured[c] for c in self.candidates)

    def compare(self) -> dict[str, TimingResult]:
        """Every comparison label, gated and timed like the candidates; a label
        that disagrees with the reference or fails is logged and left out."""
        tuner, found = self.tuner, {}
        for label, call in self.operator.baselines(self.problem, self.inputs).items():
            try:
                check = verify(self.reference, call(), dtype=self.problem.dtype)
                if check.passed:
                    found[label] = benchmark(call, warmup=tuner.warmup, iterations=tuner.iterations,
                                             device=self.device, flush_l2=tuner.flush_l2)
                else:
                    tuner.log(f"  baseline {label} disagrees with the reference: {check.reason}")
            except Exception as exc:  # noqa: BLE001
                tuner.log(f"  baseline {label} unavailable: {_classify(exc)[1]}")
        return found

    def result(self, outcomes: tuple[CandidateOutcome, ...], baselines: dict[str, TimingResult]) -> TuningResult:
        op, problem = self.operator, self.problem
        return TuningResult(problem, self.env, self.space.generated, self.space.feasible, outcomes, baselines,
                            op.flops(problem), op.bytes_moved(problem), time.perf_counter() - self.started,
                            op.is_memory_bound(), self.space.rejected)


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
        if resume and db is None:
            raise ValueError("resume needs a results database")
        self.warmup, self.iterations, self.flush_l2 = warmup, iterations, flush_l2
        self.max_candidates = max_candidates
        self.measure_baselines = measure_baselines
        self.seed = seed
        self.db, self.cache = db, cache
        self._log = log
        #: (index, config) -> keep? Deals one candidate list over several workers.
        self.candidate_filter = candidate_filter
        #: Reuse every outcome the database already holds for this problem on
        #: this device, so an interrupted sweep continues where it stopped.
        self.resume = resume

    def log(self, message: str) -> None:
        if self._log is not None:
            self._log(message)

    def tune(
        self, operator: Operator, problem: Problem, *, device: torch.device | str | None = None
    ) -> TuningResult:
        target = torch.device(device) if device is not None else require_cuda()
        sweep = _Sweep(self, operator, problem, target)
        sweep.plan()
        with exact_fp32_matmul():
            gated = sweep.gate()
            outcomes = sweep.time(gated)
            baselines = sweep.compare() if self.measure_baselines else {}
        result = sweep.result(outcomes, baselines)
        self._persist(result, sweep.env, skip=set(sweep.reused))
        return result

    def _time_candidate(self, operator, outcome, inputs, device) -> CandidateOutcome:
        """Time one gated candidate on ``inputs`` (used to re-time finalists)."""
        return _time_gated(self, operator, outcome, inputs, torch.device(device))

    def _persist(self, result: TuningResult, env: Environment, *, skip: set[KernelConfig] = frozenset()) -> None:
        """Winner to the cache; every new outcome and baseline to the database
        (outcomes reused from an earlier run already have their rows)."""
        best = result.best
        if self.cache is not None and best is not None:
            self.cache.put(result.problem, env.device_key, best.config,
                           median_us=best.timing.median_us if best.timing else None, timestamp=env.timestamp,
                           candidates_tested=result.tested)
        if self.db is None:
            return
        from kernelo_b200 import __version__

        def rates(ms: float | None) -> dict:
            return {"tflops": result.tflops(ms), "gbps": result.gbps(ms)} if ms else {"tflops": None, "gbps": None}

        rows = [Measurement("kernelforge", o.status, o.config, o.verification, o.timing,
                            error=o.error, **rates(o.timing.median_ms if o.timing else None))
                for o in result.outcomes if o.config not in skip]
        rows += [Measurement(label, STATUS_OK, timing=t, **rates(t.median_ms)) for label, t in result.baselines.items()]
        run_id = self.db.start_run(env, notes="tune", version=__version__)
        self.db.record_many(run_id, result.problem, rows)
