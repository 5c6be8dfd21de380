"""The sharded decode GEMV benchmark's host side (no GPU): its byte counts,
the JSON line it prints, and its refusal to run outside a multi-process
launch. The measurement itself needs two or more GPUs."""

from __future__ import annotations

import pytest

from kernelo_b200.benchmark import sharded


def test_byte_counts_follow_the_shard():
    # 11008 x 4096 fp16 over 2 GPUs: 5504 weight rows per rank
    assert sharded.shard_bytes(16, 4096, 5504) == (5504 * 4096 + 16 * 4096 + 16 * 5504) * 2
    assert sharded.nvlink_bytes(16, 5504, 2) == 16 * 5504 * 2
    assert sharded.nvlink_bytes(16, 1376, 8) == 16 * 1376 * 2 * 7
    assert sharded.nvlink_bytes(1, 5504, 1) == 0


def test_summary_line_is_hbm_bound_against_the_given_peak():
    times = {"full_us": 17.0, "shard_us": 9.0, "step_us": 12.0, "eager_step_us": 40.0, "nccl_us": 60.0}
    line = sharded.summary(16, 11008, 4096, 2, 5504, times, 6500.0, "measured")
    roof = line["roofline"]
    assert roof["bound"] == "hbm" and roof["unit"] == "GB/s" and roof["peak"] == 6500.0
    achieved = sharded.shard_bytes(16, 4096, 5504) / 9e-6 / 1e9
    assert roof["achieved"] == pytest.approx(achieved, abs=0.1)
    assert roof["frac"] == pytest.approx(achieved / 6500.0, abs=1e-4)
    assert line["speedup_vs_one_gpu"] == pytest.approx(17.0 / 12.0, abs=1e-3)
    assert line["higher_is_better"] is False and line["n_gpus"] == 2 and line["step_us"] == 12.0


def test_refuses_a_single_process_and_rows_outside_the_tile_range(monkeypatch):
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    with pytest.raises(SystemExit):
        sharded.main(["--rows", "1"])
    monkeypatch.setenv("WORLD_SIZE", "2")
    with pytest.raises(SystemExit):
        sharded.main(["--rows", "33"])


def test_peak_falls_back_without_the_measured_file(monkeypatch, tmp_path):
    monkeypatch.setattr(sharded, "PEAKS_FILE", tmp_path / "absent.json")
    assert sharded.hbm_peak() == (sharded.HBM_FALLBACK_GBS, "fallback")
    path = tmp_path / "peaks.json"
    path.write_text('{"hbm_gbs": 6493.7}')
    monkeypatch.setattr(sharded, "PEAKS_FILE", path)
    assert sharded.hbm_peak() == (6493.7, "measured")
