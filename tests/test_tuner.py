"""The tuner, end to end on the CPU (tuning/tuner.py).

A fake operator fails in each way a native config can fail -- the library
rejects it (``OutOfResources``), a bounded device wait gives up
(``KernelTimeoutError``), a launch error, a wrong answer -- next to correct fast
and slow configs. Failures are made on the host; no GPU is involved. The
central guarantee: nothing incorrect is ever ranked.
"""

from __future__ import annotations

from collections.abc import Iterator

import pytest
import torch

from kernelo_b200.db import ResultsDB
from kernelo_b200.kernels.base import Operator
from kernelo_b200.runtime import native
from kernelo_b200.tuning.cache import ConfigCache
from kernelo_b200.tuning.config import KernelConfig, Problem
from kernelo_b200.tuning.search import SearchSpace
from kernelo_b200.tuning.tuner import (
    STATUS_COMPILE_ERROR,
    STATUS_INCORRECT,
    STATUS_OK,
    STATUS_RUNTIME_ERROR,
    Tuner,
)

FAST, LAUNCH_FAILS, WRONG, SLOW, INFEASIBLE, OUT_OF_RESOURCES, TIMES_OUT = range(7)


class _Space(SearchSpace):
    operation = "cpu_double"

    def grid(self, problem: Problem) -> Iterator[KernelConfig]:
        for mode in range(7):
            yield KernelConfig(self.operation, MODE=mode)

    def reject_reason(self, config, problem, caps):
        return "infeasible by construction" if config["MODE"] == INFEASIBLE else None


class _FakeOperator(Operator):
    name = "cpu_double"

    def search_space(self):
        return _Space()

    def make_inputs(self, problem, device, *, seed=0):
        gen = torch.Generator().manual_seed(seed)
        return (torch.randn(problem["n"], generator=gen).to(device),)

    def reference(self, x):
        return x * 2

    def run(self, config, x):
        mode = config["MODE"]
        if mode == LAUNCH_FAILS:
            native.check(native.KF_ERR_LAUNCH, "simulated launch failure")
        if mode == OUT_OF_RESOURCES:
            native.check(native.KF_ERR_INVALID_CONFIG, "simulated infeasible config")
        if mode == TIMES_OUT:
            native.check(native.KF_ERR_TIMEOUT, "simulated bounded-wait timeout")
        if mode == WRONG:
            return x * 3
        if mode == SLOW:
            y = x.clone()
            for _ in range(40):
                y = y * 1.0
            return y * 2
        return x * 2

    def default_config(self, problem):
        return KernelConfig(self.name, MODE=FAST)

    def flops(self, problem):
        return problem["n"]

    def bytes_moved(self, problem):
        return 2 * problem["n"] * problem.itemsize

    def baselines(self, problem, inputs):
        (x,) = inputs
        return {"torch_eager": lambda: x * 2}


PROBLEM = Problem.create("cpu_double", "fp32", n=200_000)


@pytest.fixture(scope="module")
def tuned():
    return Tuner(warmup=2, iterations=5, flush_l2=False).tune(_FakeOperator(), PROBLEM, device="cpu")


def test_stage_counts(tuned):
    assert (tuned.generated, tuned.feasible, tuned.tested, tuned.correct) == (7, 6, 6, 2)
    assert sum(tuned.status_counts().values()) == tuned.tested


def test_every_failure_is_classified(tuned):
    by = {o.config["MODE"]: o for o in tuned.outcomes}
    assert by[FAST].status == by[SLOW].status == STATUS_OK
    assert by[LAUNCH_FAILS].status == STATUS_RUNTIME_ERROR and "simulated launch" in by[LAUNCH_FAILS].error
    assert by[OUT_OF_RESOURCES].status == STATUS_COMPILE_ERROR
    assert by[TIMES_OUT].status == STATUS_RUNTIME_ERROR and "timeout" in by[TIMES_OUT].error
    assert by[WRONG].status == STATUS_INCORRECT
    assert INFEASIBLE not in by


def test_only_correct_candidates_are_ranked(tuned):
    assert {o.config["MODE"] for o in tuned.ranked()} == {FAST, SLOW}
    assert tuned.best.config["MODE"] == FAST
    for o in tuned.outcomes:
        if not o.ok:
            assert o.timing is None
            with pytest.raises(ValueError, match="no timing"):
                _ = o.median_ms


def test_rejections_baselines_and_metrics(tuned):
    assert [(c["MODE"], r) for c, r in tuned.rejections] == [(INFEASIBLE, "infeasible by construction")]
    assert tuned.baselines["torch_eager"].iterations == 5
    assert tuned.speedup_over("torch_eager") > 0 and tuned.speedup_over("nope") is None
    ms = tuned.best.median_ms
    assert tuned.tflops(ms) == pytest.approx(PROBLEM["n"] / (ms * 1e-3) / 1e12)
    assert tuned.environment.torch_version == torch.__version__


def test_persistence(tmp_path):
    db = ResultsDB(tmp_path / "r.db")
    cache = ConfigCache(tmp_path / "c.json")
    result = Tuner(warmup=1, iterations=2, flush_l2=False, db=db, cache=cache).tune(
        _FakeOperator(), PROBLEM, device="cpu")
    assert db.counts()["runs"] == 1
    assert db.counts()["results"] == result.tested + len(result.baselines)
    statuses = {r["status"] for r in db.rows(operation="cpu_double")}
    assert {STATUS_OK, STATUS_INCORRECT, STATUS_RUNTIME_ERROR, STATUS_COMPILE_ERROR} <= statuses
    assert cache.get(PROBLEM, result.environment.device_key) == result.best_config
    assert ConfigCache(tmp_path / "c.json").entries()[0].candidates_tested == result.tested
    db.close()


def test_resumed_sweep_reuses_stored_outcomes(tmp_path):
    """A second tune with resume=True measures nothing already in the database
    (same problem, same device) and ranks the stored outcomes the same way."""
    db = ResultsDB(tmp_path / "r.db")
    first = Tuner(warmup=1, iterations=2, flush_l2=False, measure_baselines=False, db=db).tune(
        _FakeOperator(), PROBLEM, device="cpu")
    rows_after_first = db.counts()["results"]
    calls = []

    class _Counting(_FakeOperator):
        def run(self, config, x):
            calls.append(config)
            return super().run(config, x)

    lines: list[str] = []
    second = Tuner(warmup=1, iterations=2, flush_l2=False, measure_baselines=False, db=db, resume=True,
                   log=lines.append).tune(_Counting(), PROBLEM, device="cpu")
    assert calls == [], "a resumed sweep re-ran stored candidates"
    assert any(line.startswith("Resuming:") for line in lines)
    assert [o.status for o in second.outcomes] == [o.status for o in first.outcomes]
    assert second.best_config == first.best_config
    assert abs(second.best.median_ms - first.best.median_ms) < 1e-9
    assert db.counts()["results"] == rows_after_first  # nothing recorded twice
    with pytest.raises(ValueError, match="resume needs"):
        Tuner(resume=True)
    db.close()


def test_budget_filter_and_log():
    lines = []
    result = Tuner(warmup=1, iterations=2, max_candidates=2, measure_baselines=False, log=lines.append).tune(
        _FakeOperator(), PROBLEM, device="cpu")
    assert result.tested == 2
    assert "Verifying candidates" in "\n".join(lines) and "Benchmarking" in "\n".join(lines)
    odd = Tuner(warmup=1, iterations=2, measure_baselines=False,
                candidate_filter=lambda i, c: i % 2 == 1).tune(_FakeOperator(), PROBLEM, device="cpu")
    assert odd.tested == 3


def test_no_feasible_candidates_means_no_best():
    class _Empty(_Space):
        def reject_reason(self, config, problem, caps):
            return "nothing fits"

    class _EmptyOp(_FakeOperator):
        def search_space(self):
            return _Empty()

    result = Tuner(warmup=1, iterations=2, measure_baselines=False).tune(_EmptyOp(), PROBLEM, device="cpu")
    assert result.tested == 0 and result.best is None and result.ranked() == []
