"""The command line interface (``kernelforge/cli/main.py``), the report tables
and the Nsight Compute command builder. CPU tests drive the parser, ``env``,
``tune --explain``, ``cache`` and ``report``; GPU tests run ``tune``,
``compare``, ``benchmark``, ``profile`` and the transformer comparison on small
shapes with a temporary database and cache."""

from __future__ import annotations

import json

import pytest
import torch

from kernelo_b200 import cli
from kernelo_b200.profiling import nsight


def run_cli(argv, capsys):
    code = cli.main(argv)
    out = capsys.readouterr()
    return code, out.out, out.err


# ------------------------------------------------------------------ CPU
def test_parser_knows_every_operation_and_rejects_others():
    parser = cli.build_parser()
    for op in ("matmul", "fused_linear", "fused_linear_erf", "gemv", "rmsnorm", "softmax"):
        assert parser.parse_args(["tune", op]).operation == op
    with pytest.raises(SystemExit):
        parser.parse_args(["tune", "vector_add"])
    assert parser.parse_args(["compare", "transformer"]).operation == "transformer"


def test_build_problem_defaults_and_flags():
    parser = cli.build_parser()
    p = cli.build_problem("gemv", parser.parse_args(["tune", "gemv"]))
    assert p.dims_dict == {"M": 1, "N": 11008, "K": 4096}
    p = cli.build_problem("softmax", parser.parse_args(["tune", "softmax", "--rows", "8", "--cols", "1000"]))
    assert p.dims_dict == {"rows": 8, "cols": 1000}


def test_env_runs_without_a_gpu(capsys):
    code, out, _ = run_cli(["env"], capsys)
    assert code == 0 and "Device limits" in out and "148" in out


def test_tune_explain_prints_the_sm100_candidate_breakdown(capsys):
    code, out, _ = run_cli(["tune", "fused_linear_erf", "-m", "4096", "-n", "11008", "-k", "4096",
                            "--dtype", "bf16", "--explain"], capsys)
    assert code == 0
    assert "grid points" in out and "feasible" in out and "rejections by rule" in out
    code, out, _ = run_cli(["tune", "softmax", "--rows", "32768", "--cols", "1000", "--explain",
                            "--max-candidates", "5"], capsys)
    assert code == 0 and "of 5" in out


def test_cache_list_and_clear(tmp_path, capsys):
    from kernelo_b200.tuning.cache import ConfigCache
    from kernelo_b200.tuning.config import KernelConfig, Problem

    path = tmp_path / "cache.json"
    cache = ConfigCache(path)
    problem = Problem.create("gemv", "fp16", M=4, N=11008, K=4096)
    cache.put(problem, "NVIDIA_B200_sm100", KernelConfig("gemv", KERNEL=4, BLOCK_M=8, num_stages=2),
              median_us=17.3)
    code, out, _ = run_cli(["cache", "list", "--cache", str(path)], capsys)
    assert code == 0 and "1 entry" in out and "gemv" in out
    code, out, _ = run_cli(["cache", "clear", "--cache", str(path)], capsys)
    assert code == 0 and "removed 1" in out
    assert len(ConfigCache(path)) == 0


def _fake_rows(db):
    from kernelo_b200.benchmark.runner import TimingResult
    from kernelo_b200.db import Measurement
    from kernelo_b200.runtime.env import Environment
    from kernelo_b200.testing import VerificationResult
    from kernelo_b200.tuning.config import KernelConfig, Problem

    env = Environment("2026-01-01T00:00:00+00:00", "host", "linux", "3.12", "2.11", "0.1.0", "12.8", "580",
                      "NVIDIA B200", "10.0", 183 << 30, 148, "NVIDIA_B200_sm100")
    run = db.start_run(env, notes="test")
    problem = Problem.create("softmax", "fp16", rows=32768, cols=4096)
    ok = VerificationResult(True, 1e-4, 1e-4, 0, 10, 5e-3)
    for label, ms, gbps in (("torch_eager", 0.2, 2684.0), ("kernelforge", 0.083, 6467.0)):
        timing = TimingResult(ms, ms, 0.0, ms, ms, ms, ms, 5, 20, "cuda_event", True)
        cfg = KernelConfig("softmax", ROW_KERNEL=1, num_warps=2) if label == "kernelforge" else None
        db.record(run, problem, Measurement(label=label, status="ok", config=cfg, verification=ok,
                                            timing=timing, gbps=gbps))


def test_report_writes_tables_from_the_database(tmp_path, capsys):
    from kernelo_b200.db import ResultsDB

    db_path = tmp_path / "r.db"
    with ResultsDB(db_path) as db:
        _fake_rows(db)
    code, out, _ = run_cli(["report", "--db", str(db_path), "--out", str(tmp_path / "rep")], capsys)
    assert code == 0 and "2 measurements" in out
    summary = (tmp_path / "rep" / "summary.md").read_text()
    assert "## softmax" in summary and "NVIDIA B200" in summary
    assert "6467.0" in summary and "2.41x" in summary  # 200 us / 83 us
    assert (tmp_path / "rep" / "softmax.csv").read_text().count("\n") == 3
    code, _, err = run_cli(["report", "--db", str(tmp_path / "missing.db")], capsys)
    assert code == 2 and "no results database" in err


def test_nsight_command_never_locks_clocks_and_profiles_one_launch():
    cmd = nsight.build_command(["python", "-c", "pass"], sections=("throughput", "memory"))
    assert cmd[:3] == ["ncu", "--clock-control", "none"]
    assert cmd[cmd.index("--launch-count") + 1] == "1"
    assert "SpeedOfLight" in cmd and "MemoryWorkloadAnalysis" in cmd
    with pytest.raises(ValueError, match="unknown sections"):
        nsight.build_command(["x"], sections=("everything",))
    args = cli.build_parser().parse_args(["profile", "softmax", "--backend", "nsight", "--rows", "64",
                                          "--cols", "1000", "--no-cache"])
    child = cli.nsight_child_argv(args)
    assert child[:2] == ["profile", "softmax"] and "--rows" in child and "1000" in child
    assert child[-2:] == ["--backend", "launch-once"] and "--no-db" in child


def test_nsight_raw_page_parser():
    text = ('==PROF== Connected\n"ID","Kernel Name","Grid Size","gpu__time_duration.sum","dram__bytes_read.sum"\n'
            '"","","","us","MB"\n"0","rows_kernel","(32768, 1, 1)","85.2","268.5"\n')
    parsed = nsight.parse_raw_csv(text)
    assert parsed == {"rows_kernel": {"Grid Size": "(32768, 1, 1)", "gpu__time_duration.sum": "85.2 us",
                                      "dram__bytes_read.sum": "268.5 MB"}}
    assert nsight.parse_raw_csv("not csv") == {}


# ------------------------------------------------------------------ GPU
@pytest.mark.gpu
def test_tune_records_and_caches(tmp_path, capsys, device):
    db, cache = tmp_path / "t.db", tmp_path / "c.json"
    code, out, _ = run_cli(["tune", "rmsnorm", "--rows", "1024", "--cols", "4096", "--dtype", "bf16",
                            "--warmup", "2", "--iterations", "5", "--max-candidates", "4",
                            "--db", str(db), "--cache", str(cache)], capsys)
    assert code == 0, out
    assert "Best configuration" in out and "GB/s" in out
    assert json.loads(cache.read_text())
    code, out, _ = run_cli(["report", "--db", str(db), "--out", str(tmp_path / "rep")], capsys)
    assert code == 0 and "## rmsnorm" in (tmp_path / "rep" / "summary.md").read_text()


@pytest.mark.gpu
def test_compare_benchmark_and_profile(tmp_path, capsys, device):
    code, out, _ = run_cli(["compare", "softmax", "--rows", "2048", "--cols", "1000", "--warmup", "2",
                            "--iterations", "5", "--no-cache"], capsys)
    assert code == 0 and "kernelforge" in out and "torch_eager" in out
    code, out, _ = run_cli(["benchmark", "gemv", "--suite", "smoke", "--warmup", "2", "--iterations", "5",
                            "--db", str(tmp_path / "b.db"), "--no-cache"], capsys)
    assert code == 0 and "INCORRECT" not in out and "kernelforge" in out
    code, out, _ = run_cli(["profile", "fused_linear", "-m", "256", "-n", "512", "-k", "256", "--warmup", "2",
                            "--iterations", "3", "--no-cache", "--no-db"], capsys)
    assert code == 0 and "kernel launches per call" in out
    code, _, _ = run_cli(["profile", "softmax", "--rows", "64", "--cols", "1000", "--backend", "launch-once",
                          "--no-cache", "--no-db"], capsys)
    assert code == 0


@pytest.mark.gpu
def test_compare_transformer_prints_the_amdahl_breakdown(capsys, device):
    code, out, _ = run_cli(["compare", "transformer", "--hidden", "256", "--heads", "8", "--intermediate", "512",
                            "--seq", "64", "--warmup", "2", "--iterations", "5", "--no-cache"], capsys)
    assert code == 0
    assert "predicted" in out and "measured" in out and "swapped share" in out
    torch.cuda.synchronize()
