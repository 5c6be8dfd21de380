"""Host-side components kept from the reference API: descriptors, the gate,
the timer's statistics, the results DB and the config cache. CPU only.

Each group mirrors the behaviour the reference pins in its own tests
(tests/test_config.py, test_verification.py, test_benchmark_runner.py,
test_db_and_cache.py) against this implementation.
"""

from __future__ import annotations

import json
import sqlite3

import numpy as np
import pytest
import torch

from kernelo_b200.benchmark.runner import TIMER_RESOLUTION_MS, benchmark, summarize
from kernelo_b200.db import SCHEMA_VERSION, Measurement, ResultsDB
from kernelo_b200.dtypes import dtype_name, itemsize, native_code, parse_dtype
from kernelo_b200.runtime.env import capture_environment
from kernelo_b200.testing import (
    ERROR_THRESHOLDS,
    VerificationResult,
    assert_verified,
    exact_fp32_matmul,
    threshold_for,
    verify,
)
from kernelo_b200.tuning.cache import CACHE_VERSION, ConfigCache
from kernelo_b200.tuning.config import KernelConfig, Problem

PROBLEM = Problem.create("matmul", "fp16", M=2048, N=4096, K=4096)
CONFIG = KernelConfig("matmul", KERNEL=1, BLOCK_M=128, BLOCK_N=256, BLOCK_K=64, GROUP_M=8, num_stages=4)


# ---------------------------------------------------------------- descriptors
def test_config_identity_ignores_keyword_order():
    a = KernelConfig("matmul", BLOCK_M=128, BLOCK_N=64)
    b = KernelConfig("matmul", BLOCK_N=64, BLOCK_M=128)
    assert a == b and hash(a) == hash(b) and len({a, b}) == 1


def test_config_meta_launch_split_and_json_round_trip():
    c = KernelConfig("rmsnorm", BLOCK_SIZE=4096, ROWS_PER_PROGRAM=2, num_warps=8, num_stages=2)
    assert c.launch == {"num_stages": 2, "num_warps": 8}
    assert c.meta == {"BLOCK_SIZE": 4096, "ROWS_PER_PROGRAM": 2}
    assert KernelConfig.from_json("rmsnorm", c.to_json()) == c


def test_config_digest_separates_operations_and_values():
    a = KernelConfig("matmul", BLOCK_N=128)
    assert a.digest == KernelConfig("matmul", BLOCK_N=128).digest
    assert a.digest != KernelConfig("matmul", BLOCK_N=64).digest
    assert a.digest != KernelConfig("fused_linear", BLOCK_N=128).digest


@pytest.mark.parametrize("bad", [64.0, True, "64"])
def test_config_rejects_non_int_values(bad):
    with pytest.raises(TypeError):
        KernelConfig("matmul", BLOCK_M=bad)


def test_config_render_order_and_replace():
    c = KernelConfig("matmul", BLOCK_M=128, BLOCK_N=64, num_stages=4)
    assert [l.split(":")[0] for l in c.render(("num_stages", "BLOCK_N")).splitlines()] == [
        "num_stages", "BLOCK_N", "BLOCK_M"]
    assert c.replace(BLOCK_N=256)["BLOCK_N"] == 256 and c["BLOCK_N"] == 64


def test_problem_keys_and_validation():
    p = Problem.create("matmul", "bf16", M=1, N=11008, K=4096)
    assert p.shape_key == "1x11008x4096" and p.cache_key == "matmul/bf16/1x11008x4096"
    assert p["K"] == 4096 and p.itemsize == 2
    assert p == Problem.create("matmul", torch.bfloat16, M=1, N=11008, K=4096)
    for bad in (0, -3):
        with pytest.raises(ValueError, match="positive"):
            Problem.create("matmul", "fp16", M=bad, N=1, K=1)


@pytest.mark.parametrize("name,dtype,size,code", [("fp16", torch.float16, 2, 0), ("bf16", torch.bfloat16, 2, 1),
                                                  ("fp32", torch.float32, 4, 2)])
def test_dtype_names_round_trip(name, dtype, size, code):
    assert parse_dtype(name) is dtype and parse_dtype(name.upper()) is dtype
    assert dtype_name(dtype) == name and itemsize(dtype) == size and native_code(dtype) == code


def test_unknown_dtypes_are_rejected():
    with pytest.raises(ValueError):
        parse_dtype("int8")
    with pytest.raises(ValueError):
        native_code(torch.int32)


# ---------------------------------------------------------------- the gate
def test_gate_identical_and_rounded_outputs():
    x = torch.randn(64, 64)
    r = verify(x, x.clone())
    assert r.passed and r.error == 0 and r.mismatched == 0 and r.total == 4096
    assert verify(x, x.half(), dtype=torch.float16).passed
    assert not verify(x, x.half().float()).passed  # fp32 threshold is the strict one


def test_gate_catches_unwritten_regions_nan_and_shape():
    ref = torch.randn(128, 128)
    broken = ref.clone()
    broken[:, -1] = 0.0
    r = verify(ref, broken)
    assert not r.passed and r.mismatched > 0
    broken[0, 0] = float("nan")
    r = verify(ref, broken)
    assert not r.passed and "non-finite" in r.reason and r.error == float("inf")
    assert "shape mismatch" in verify(torch.zeros(8, 8), torch.zeros(8, 9)).reason


def test_gate_zero_reference_empty_and_scale_invariance():
    z = torch.zeros(16, 16)
    assert verify(z, z.clone()).passed and not verify(z, z + 0.5).passed
    assert verify(torch.empty(0), torch.empty(0)).passed
    ref = torch.randn(128, 128)
    out = ref + 1e-4 * torch.randn(128, 128)
    assert verify(ref, out).error == pytest.approx(verify(ref * 1000, out * 1000).error, rel=1e-3)


def test_gate_thresholds_and_overrides():
    for dtype in ERROR_THRESHOLDS:
        assert threshold_for(dtype) > 0
    with pytest.raises(ValueError, match="no correctness threshold"):
        threshold_for(torch.int32)
    ref = torch.randn(32, 32)
    assert not verify(ref, ref + 0.1).passed and verify(ref, ref + 0.1, threshold=10.0).passed
    with pytest.raises(AssertionError, match="BLOCK_N=64"):
        assert_verified(torch.zeros(4), torch.ones(4), context="BLOCK_N=64")


def test_exact_fp32_matmul_restores_settings_even_on_error():
    before = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        with pytest.raises(RuntimeError), exact_fp32_matmul():
            assert torch.backends.cuda.matmul.allow_tf32 is False
            raise RuntimeError("boom")
        assert torch.backends.cuda.matmul.allow_tf32 is True
    finally:
        torch.backends.cuda.matmul.allow_tf32 = before


# ---------------------------------------------------------------- timer
def test_summary_statistics():
    s = [1.0, 2.0, 3.0, 4.0, 100.0]
    r = summarize(s, warmup=5, iterations=5, timer="cuda_event", flushed_l2=True)
    assert (r.median_ms, r.min_ms, r.max_ms) == (3.0, 1.0, 100.0)
    assert r.mean_ms == pytest.approx(22.0)
    assert r.p95_ms == pytest.approx(float(np.percentile(s, 95)))
    assert r.std_ms == pytest.approx(float(np.std(s, ddof=1)))
    spiked = summarize([2.0] * 199 + [400.0], warmup=0, iterations=200, timer="cuda_event", flushed_l2=True)
    assert spiked.median_ms == 2.0 and spiked.mean_ms > 3.0
    with pytest.raises(ValueError, match="empty"):
        summarize([], warmup=0, iterations=0, timer="cuda_event", flushed_l2=False)


def test_timer_resolution_flag_and_samples():
    tiny = summarize([TIMER_RESOLUTION_MS / 2], warmup=0, iterations=1, timer="cuda_event", flushed_l2=True)
    assert tiny.at_timer_resolution
    cpu = summarize([TIMER_RESOLUTION_MS / 2], warmup=0, iterations=1, timer="perf_counter", flushed_l2=False)
    assert not cpu.at_timer_resolution
    kw = dict(warmup=0, iterations=3, timer="perf_counter", flushed_l2=False)
    assert summarize([1.0, 2.0, 3.0], **kw).samples_ms == ()
    assert summarize([1.0, 2.0, 3.0], keep_samples=True, **kw).samples_ms == (1.0, 2.0, 3.0)


def test_cpu_benchmark_counts_iterations_and_is_labelled():
    calls = []
    r = benchmark(lambda: calls.append(1), warmup=3, iterations=7, device="cpu")
    assert len(calls) == 10 and r.iterations == 7 and r.timer == "perf_counter" and not r.flushed_l2
    assert "samples_ms" not in r.as_dict()
    for warmup, iters in ((-1, 10), (0, 0)):
        with pytest.raises(ValueError):
            benchmark(lambda: None, warmup=warmup, iterations=iters, device="cpu")


# ---------------------------------------------------------------- results DB
def _timing(ms: float):
    return summarize([ms], warmup=25, iterations=1, timer="cuda_event", flushed_l2=True)


def _ok_check():
    return VerificationResult(True, 1e-4, 1e-3, 0, 100, 5e-3)


@pytest.fixture
def db(tmp_path):
    with ResultsDB(tmp_path / "r.db") as handle:
        yield handle


def test_db_schema_version_recorded_and_enforced(tmp_path):
    path = tmp_path / "r.db"
    ResultsDB(path).close()
    con = sqlite3.connect(path)
    assert int(con.execute("PRAGMA user_version").fetchone()[0]) == SCHEMA_VERSION
    con.execute(f"PRAGMA user_version = {SCHEMA_VERSION + 1}")
    con.commit()
    con.close()
    with pytest.raises(RuntimeError, match="schema version"):
        ResultsDB(path)


def test_db_dedup_and_round_trip(db):
    assert db.problem_id(PROBLEM) == db.problem_id(PROBLEM)
    assert db.config_id(CONFIG) == db.config_id(CONFIG)
    assert db.config_id(KernelConfig("matmul", BLOCK_M=64)) != db.config_id(KernelConfig("fused_linear", BLOCK_M=64))
    env = capture_environment()
    run = db.start_run(env, notes="t", version="0.1.0")
    db.record(run, PROBLEM, Measurement("kernelforge", "ok", CONFIG, _ok_check(), _timing(0.5), tflops=137.4))
    db.record(run, PROBLEM, Measurement("kernelforge", "compile_error", CONFIG, error="OutOfResources: smem"))
    db.record(run, PROBLEM, Measurement("torch_eager", "ok", timing=_timing(1.0)))
    rows = db.rows()
    assert rows[0]["median_us"] == pytest.approx(500.0) and rows[0]["correct"] == 1
    assert json.loads(rows[0]["params_json"])["BLOCK_N"] == 256
    assert rows[1]["median_us"] is None and "OutOfResources" in rows[1]["error"]
    assert rows[2]["params_json"] is None
    assert rows[0]["torch_version"] == env.torch_version
    assert db.has_result(PROBLEM, CONFIG) and not db.has_result(PROBLEM, CONFIG.replace(BLOCK_N=64))


def test_db_best_per_label_ignores_incorrect_rows(db):
    run = db.start_run(capture_environment())
    for ms, label, ok in ((0.9, "kernelforge", True), (0.4, "kernelforge", False), (0.7, "kernelforge", True),
                          (1.5, "torch_eager", True)):
        check = _ok_check() if ok else VerificationResult(False, 1.0, 1.0, 10, 10, 5e-3, "wrong")
        db.record(run, PROBLEM, Measurement(label, "ok" if ok else "incorrect",
                                            CONFIG if label == "kernelforge" else None, check, _timing(ms)))
    best = {r["label"]: r["median_us"] for r in db.best_per_label()}
    assert best["kernelforge"] == pytest.approx(700.0) and best["torch_eager"] == pytest.approx(1500.0)
    assert db.counts()["results"] == 4 and db.operations() == ["matmul"]


# ---------------------------------------------------------------- config cache
def test_cache_round_trip_keys_and_atomic_write(tmp_path):
    path = tmp_path / "configs.json"
    cache = ConfigCache(path)
    assert cache.get(PROBLEM, "NVIDIA_B200_sm100") is None
    cache.put(PROBLEM, "NVIDIA_B200_sm100", CONFIG, median_us=421.0, timestamp="t")
    assert ConfigCache(path).get(PROBLEM, "NVIDIA_B200_sm100") == CONFIG
    assert cache.get(PROBLEM, "NVIDIA_H100_sm90") is None
    assert cache.get(Problem.create("matmul", "bf16", M=2048, N=4096, K=4096), "NVIDIA_B200_sm100") is None
    assert sorted(p.name for p in tmp_path.iterdir()) == ["configs.json"]
    cache.put(PROBLEM, "NVIDIA_B200_sm100", CONFIG.replace(BLOCK_N=128), median_us=400.0)
    assert len(cache) == 1 and "400.0 us" in cache.entries()[0].describe()
    assert cache.clear() == 1 and not path.exists()


def test_cache_writers_merge_instead_of_overwriting(tmp_path):
    """Two processes' caches on one file (a tuner per GPU): each put merges into
    the file as it is on disk, so neither loses the other's entry."""
    path = tmp_path / "configs.json"
    first, second = ConfigCache(path), ConfigCache(path)
    other = Problem.create("matmul", "bf16", M=2048, N=4096, K=4096)
    first.put(PROBLEM, "NVIDIA_B200_sm100", CONFIG, median_us=1.0)
    second.put(other, "NVIDIA_B200_sm100", CONFIG.replace(BLOCK_N=64), median_us=2.0)
    merged = ConfigCache(path)
    assert merged.get(PROBLEM, "NVIDIA_B200_sm100") == CONFIG
    assert merged.get(other, "NVIDIA_B200_sm100") == CONFIG.replace(BLOCK_N=64)
    doc = json.loads(path.read_text())
    assert doc["version"] == CACHE_VERSION and set(doc["entries"]["NVIDIA_B200_sm100"]["matmul"]) == {"fp16", "bf16"}


def test_cache_refuses_corrupt_or_foreign_versions(tmp_path):
    path = tmp_path / "c.json"
    path.write_text("{not json")
    with pytest.raises(RuntimeError, match="not valid JSON"):
        ConfigCache(path)
    path.write_text(json.dumps({"version": CACHE_VERSION + 1, "entries": {}}))
    with pytest.raises(RuntimeError, match="cache clear"):
        ConfigCache(path)
