"""Decode GEMV column-sharded over the GPUs of one node: time per call.

Run one process per GPU::

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \\
        --master-addr 127.0.0.1 -m kernelo_b200.benchmark.sharded --rows 1 4 16

For each M, rank 0 prints one JSON line with the max over ranks of:

* ``full_us`` -- one GPU's GEMV over the whole [N, K] weight (the single-GPU
  baseline, :func:`kernelo_b200.kernels.gemv.gemv`);
* ``shard_us`` -- this rank's shard kernel with its peer stores (the tile
  GEMV writing every peer's copy of Y), without the barrier;
* ``step_us`` -- the whole sharded step (shard kernel + the bounded peer
  barrier) captured in a CUDA graph and replayed, the way a decode loop runs
  it: the barrier keeps its epoch on the device, so every replay
  synchronises the ranks again;
* ``eager_step_us`` -- the same step launched from Python each call (host
  launch cost included);
* ``nccl_us`` -- the NCCL alternative, eager: the local GEMV, then
  ``all_gather_into_tensor`` and the permute.

Kernel-only figures replay the launches as one CUDA graph over enough
weight sets to exceed twice the L2 per rank, so no launch finds its weight
cached. The roofline of the shard kernel is HBM: its algorithmic bytes
(N/g·K + M·K + M·N/g)·2 over the measured copy bandwidth. The bytes each
rank sends over NVLink, M·(N/g)·2·(g−1), are a few hundred KB at most.

The reference has no multi-GPU code and no dedicated GEMV (single-GPU decode
is its ``matmul`` at M in {1, 4, 16}, kernelforge/kernels/matmul.py:132-155).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import time
from pathlib import Path

import torch
import torch.distributed as dist

HBM_FALLBACK_GBS = 6650.0
PEAKS_FILE = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"


def hbm_peak() -> tuple[float, str]:
    """The measured copy bandwidth (GB/s) of this pool's B200s, else the fallback."""
    if PEAKS_FILE.exists():
        try:
            return float(json.loads(PEAKS_FILE.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return HBM_FALLBACK_GBS, "fallback"


def shard_bytes(m: int, k: int, chunk: int, elt: int = 2) -> int:
    """Algorithmic HBM bytes of one rank's shard kernel: its weight rows, x, its Y slice."""
    return (chunk * k + m * k + m * chunk) * elt


def nvlink_bytes(m: int, chunk: int, world: int, elt: int = 2) -> int:
    """Bytes one rank stores into its peers' copies of Y per call."""
    return m * chunk * elt * (world - 1)


def summary(m: int, n: int, k: int, world: int, chunk: int, times_us: dict, peak_gbs: float,
            peak_kind: str) -> dict:
    """The JSON line for one M (times already maxed over ranks)."""
    shard_b = shard_bytes(m, k, chunk)
    achieved = shard_b / (times_us["shard_us"] * 1e-6) / 1e9
    line = {
        "metric": "sharded decode GEMV time per call", "unit": "us", "higher_is_better": False,
        "n_gpus": world, "M": m, "N": n, "K": k, "dtype": "fp16", "chunk_per_rank": chunk,
        **{key: round(v, 2) for key, v in times_us.items()},
        "roofline": {"bound": "hbm", "kernel": "gemv_mma_kernel (peer stores)",
                     "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
                     "frac": round(achieved / peak_gbs, 4), "peak_kind": peak_kind,
                     "bytes_per_rank": shard_b, "nvlink_bytes_per_rank": nvlink_bytes(m, chunk, world)},
    }
    line["speedup_vs_one_gpu"] = round(times_us["full_us"] / times_us["step_us"], 3)
    return line


def _max_over_ranks(value: float, device: torch.device) -> float:
    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sync_ranks() -> None:
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()


def _graph_us(fn, calls_per_replay: int, replays: int = 7) -> float:
    """Median µs per call of ``fn`` (which issues ``calls_per_replay`` calls),
    captured once and replayed, the ranks aligned before each replay."""
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    samples = []
    for _ in range(replays):
        _sync_ranks()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        end.record()
        end.synchronize()
        samples.append(start.elapsed_time(end) * 1e3 / calls_per_replay)
    _sync_ranks()
    del graph
    samples.sort()
    return samples[len(samples) // 2]


def _eager_us(fn, iters: int = 200, warmup: int = 20) -> float:
    for _ in range(warmup):
        fn()
    _sync_ranks()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) * 1e3 / iters


def run(rows: list[int], n: int, k: int) -> list[dict]:
    """Measure every M in ``rows`` on this process group (collective)."""
    from kernelo_b200.benchmark.runner import graph_time_per_launch, rotation_sets
    from kernelo_b200.distributed import ShardedGemv, shard_chunk
    from kernelo_b200.kernels.gemv import gemv
    from kernelo_b200.runtime import native

    if not dist.is_initialized() or dist.get_world_size() < 2:
        raise RuntimeError("the sharded GEMV benchmark runs one process per GPU on 2 or more GPUs")
    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    chunk = shard_chunk(n, world)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    sets = rotation_sets(chunk * k * 2, dev)
    # each rank builds its shards directly (no full weight per rank): seeded
    # N(0, 1/K) weight rows, the baseline's GEMV distribution
    fused = [ShardedGemv(None, out_features=n, gather="fused",
                         shard_weight=torch.randn(chunk, k, device=dev, generator=gen).mul_(k ** -0.5).half())
             for _ in range(sets)]
    nccl = [ShardedGemv(None, out_features=n, gather="nccl", shard_weight=layer.w) for layer in fused]
    full_sets = rotation_sets(n * k * 2, dev)
    full_w = [torch.randn(n, k, device=dev, generator=gen).mul_(k ** -0.5).half() for _ in range(full_sets)]
    peak, kind = hbm_peak()
    lines = []
    for m in rows:
        x = torch.randn(m, k, device=dev, generator=gen).half()
        full = graph_time_per_launch([lambda w=w: gemv(x, w) for w in full_w] * 2) * 1e3
        for layer in fused:  # peer buffers for this M (collective), parity back to 0
            layer(x)
            layer(x)
        _sync_ranks()
        peer_calls = []
        for layer in fused:
            sym = layer._symm[m]
            mine = sym.bufs[0][:, rank * chunk:(rank + 1) * chunk]
            peers = [sym.peer_ptrs[0][j] + rank * chunk * 2 for j in range(world) if j != rank]
            peer_calls.append(lambda layer=layer, mine=mine, peers=peers: native.linear_bias_act_allgather(
                x, layer.w.t(), mine, peers, bias=None, epilogue=native.KF_EPI_NONE))
        shard = graph_time_per_launch(peer_calls * 2) * 1e3
        _sync_ranks()

        def steps():
            for _ in range(2):  # an even count keeps every layer's buffer parity
                for layer in fused:
                    layer(x)

        step = _graph_us(steps, 2 * len(fused))
        i = [0]

        def eager_step():
            fused[i[0] % len(fused)](x)
            i[0] += 1

        def nccl_step():
            nccl[i[0] % len(nccl)](x)
            i[0] += 1

        eager = _eager_us(eager_step)
        nccl_t = _eager_us(nccl_step)
        same = bool(torch.equal(fused[0](x), nccl[0](x)))
        _sync_ranks()
        # every rank's verdict: any rank that differs, or any status word set
        same = _max_over_ranks(0.0 if same else 1.0, dev) == 0.0
        status = int(_max_over_ranks(float(native.device_status(dev.index)), dev))
        times = {name: _max_over_ranks(v, dev) for name, v in
                 (("full_us", full), ("shard_us", shard), ("step_us", step), ("eager_step_us", eager),
                  ("nccl_us", nccl_t))}
        line = summary(m, n, k, world, chunk, times, peak, kind)
        line["equal_to_nccl"] = same
        line["status"] = status
        lines.append(line)
    for layer in fused + nccl:
        layer.close()
    return lines


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--rows", type=int, nargs="+", default=[1, 4, 16], help="rows of x (M <= 32)")
    p.add_argument("-n", type=int, default=11008)
    p.add_argument("-k", type=int, default=4096)
    args = p.parse_args(argv)
    if any(m < 1 or m > 32 for m in args.rows):
        p.error("--rows takes M in 1..32 (the tile GEMV's range)")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world < 2:
        p.error("launch with torch.distributed.run on 2 or more GPUs (one process per GPU)")
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")  # no NVLink multicast binding anywhere
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    t0 = time.time()
    try:
        lines = run(args.rows, args.n, args.k)
    finally:
        dist.destroy_process_group()
    if int(os.environ.get("RANK", "0")) == 0:
        for line in lines:
            line["seconds"] = round(time.time() - t0, 1)
            print(json.dumps(line), flush=True)
    return 0 if all(line["equal_to_nccl"] and line["status"] == 0 for line in lines) else 1


if __name__ == "__main__":
    raise SystemExit(main())
