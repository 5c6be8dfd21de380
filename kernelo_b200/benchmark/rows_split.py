"""Softmax and RMSNorm with their rows split over the GPUs of one node.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \\
        --master-addr 127.0.0.1 -m kernelo_b200.benchmark.rows_split

Rows are independent, so the split needs no collective: rank r normalises
rows ``row_range(R, N, r)`` of the baseline tensors (softmax over
[32768, C], C in {1000, 4096, 4097, 32000}; RMSNorm over [16384, C], C in
{4096, 8192}; fp16), each rank generating its own rows from a seed. The total
work is fixed as N grows (strong scaling). For each case rank 0 prints one
JSON line with the slowest rank's device time per launch (a CUDA graph of
back-to-back launches over rotating input sets larger than twice the L2, as
in ``bench.py``'s memory-bound lines), the aggregate GB/s over all ranks
(algorithmic bytes of the whole tensor ÷ that time) and the per-GPU fraction
of the measured copy bandwidth.

The reference is single-GPU; its row kernels are ``kernelforge/kernels/
softmax.py:31-58`` and ``rmsnorm.py:41-72``.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

SOFTMAX_COLS = (1000, 4096, 4097, 32000)
RMSNORM_COLS = (4096, 8192)


def run() -> list[dict]:
    from kernelo_b200.benchmark.metrics import rmsnorm_bytes, softmax_bytes
    from kernelo_b200.benchmark.runner import graph_time_per_launch, rotation_sets
    from kernelo_b200.benchmark.sharded import hbm_peak
    from kernelo_b200.distributed import row_range
    from kernelo_b200.kernels.rmsnorm import rmsnorm
    from kernelo_b200.kernels.softmax import softmax

    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    peak, kind = hbm_peak()
    cases = [("softmax", 32768, c) for c in SOFTMAX_COLS] + [("rmsnorm", 16384, c) for c in RMSNORM_COLS]
    lines = []
    for op, rows, cols in cases:
        start, stop = row_range(rows, world, rank)
        mine = stop - start
        total = softmax_bytes(rows, cols, 2) if op == "softmax" else rmsnorm_bytes(rows, cols, 2)
        local = softmax_bytes(mine, cols, 2) if op == "softmax" else rmsnorm_bytes(mine, cols, 2)
        sets = rotation_sets(local, dev)
        scale = 4.0 if op == "softmax" else 1.0
        xs = [(torch.randn(mine, cols, device=dev, generator=gen) * scale).half() for _ in range(sets)]
        gamma = (torch.randn(cols, device=dev, generator=gen) * 0.1 + 1).half()
        if op == "softmax":
            calls = [lambda x=x: softmax(x) for x in xs] * 2
        else:
            calls = [lambda x=x: rmsnorm(x, gamma, eps=1e-6) for x in xs] * 2
        ms = graph_time_per_launch(calls)
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        gbs = total / (ms * 1e-3) / 1e9
        lines.append({
            "metric": f"{op} rows split {rows}x{cols} fp16", "unit": "GB/s", "value": round(gbs, 1),
            "higher_is_better": True, "n_gpus": world, "scaling": "strong", "us_per_launch": round(ms * 1e3, 2),
            "rows_per_rank": mine, "per_gpu_frac": round(gbs / world / peak, 3), "peak_gbs": peak,
            "peak_kind": f"{kind} HBM copy", "collective": "none (rows are independent)",
        })
        del xs, calls
    return lines


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.parse_args(argv)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        lines = run()
        if dist.get_rank() == 0:
            for line in lines:
                print(json.dumps(line), flush=True)
    finally:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
