"""bench.py's output contract, on the CPU: the reference arm's JSON line, the
warm-up rule, the fused compute + collective roofline and the clock summary."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))

import bench  # noqa: E402


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["steps"] == 2
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert set(line["cpu_baseline"]) >= {"value", "unit", "cores", "kind", "sample"}
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_fewer_than_three_warmup_steps_is_refused():
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "2"], capture_output=True, text=True, timeout=300, cwd=REPO)
    assert out.returncode != 0 and "at least 3" in (out.stderr + out.stdout)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_allgather_roofline_names_the_binding_resource(world):
    m, n, k = bench.M, bench.N, bench.K
    from kernelo_b200.distributed import shard_chunk

    chunk = shard_chunk(n, world)
    flop = 2 * m * chunk * k
    link = m * chunk * 2 * (world - 1)
    r = bench.allgather_roofline(flop, link, 0.2, 1651.8, "measured burst bf16", 770.0)
    t_tensor, t_link = flop / 1651.8e12, link / (770.0 * 1e9)
    assert r["bound"] == ("nvlink" if t_link > t_tensor else "tensor")
    assert r["frac"] == pytest.approx(max(t_tensor, t_link) * 1e3 / 0.2, abs=1e-4)
    assert r["nvlink_bytes_per_rank"] == link and r["traffic"] is None and r["nvlink_peak"] == 770.0
    assert (world == 2) == (r["bound"] == "tensor")  # 4096 x 11008 x 4096: the link binds from 4 GPUs on


def test_clock_summary_names_throttle_reasons():
    s = bench.ClockSampler(0)
    s.rows = [(1500.0, 1965.0, 900.0, 0x4), (1480.0, 1965.0, 950.0, 0x4 | 0x40), (300.0, 1965.0, 80.0, 0x1)]
    summary = s.summary()
    assert summary["sm_mhz"] == 1490.0 and summary["sm_max_mhz"] == 1965.0 and summary["samples"] == 2
    assert summary["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]
    assert bench.ClockSampler(0).summary()["samples"] == 0


def test_tensor_peak_follows_the_run():
    """Burst for a short region or one with no power cap; sustained only for a
    seconds-long region under sw_power_cap."""
    pk = {"bf16_tflops": 1651.8, "bf16_tflops_sustained": 1372.7}
    assert bench.tensor_peak_for_run(pk, "measured", {"reasons": []}, 5.0)[0] == 1651.8
    assert bench.tensor_peak_for_run(pk, "measured", {"reasons": ["sw_power_cap"]}, 0.0055)[0] == 1651.8
    peak, kind = bench.tensor_peak_for_run(pk, "measured", {"reasons": ["sw_power_cap"]}, 2.5)
    assert peak == 1372.7 and "sustained" in kind
    assert bench.tensor_peak_for_run({"bf16_tflops": 1590.0}, "fallback", {"reasons": ["sw_power_cap"]}, 9.0)[0] \
        == 1590.0
