"""The full tuner sweep on sm_100a, with a summary per problem.

    python -m kernelo_b200.benchmark.sweep [--db PATH] [--cache PATH] [--out DIR]
    python -m torch.distributed.run --nproc-per-node N -m kernelo_b200.benchmark.sweep ...

Every shape of the ``sweep_sm100`` workload suite -- the primes 4099^3 and
1021 x 2053 x 509 (whose rows no TMA tensor map can describe), the one-off-a-tile
129^3 and 257^3, the single-row 1 x 11008 x 4096 and the plain-GEMM baseline
2048 x 4096 x 4096 -- in fp16, bf16 and fp32, through the tuner: candidates
generated and filtered for the device, each gated against the reference
before any is timed, the survivors timed with CUDA events, every outcome
written to the results database and each winner to the config cache. Inputs
are N(0, 1) from a fixed seed. This is the reference's own pipeline
(``kernelforge/tuning/tuner.py:184-239``) over this library's sm_100a grid.

Under torchrun each problem's candidates are dealt round-robin to one worker
per GPU; rank 0 re-times the finalists on its own GPU, ranks, and alone writes
the database and the cache (``kernelo_b200.distributed.distributed_tune``).

The summary (JSON and a markdown table, on rank 0) gives per problem the
funnel counts, failures by status, the winner against the library default,
the winner's gate error, and whether the cache now holds the winner.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

from kernelo_b200.benchmark import workloads

DTYPES = ("fp16", "bf16", "fp32")


def summarize_result(result, operator, cache) -> dict:
    """One problem's line of the sweep summary."""
    problem = result.problem
    default = operator.default_config(problem)
    by_config = {o.config: o for o in result.outcomes}
    best = result.best
    default_outcome = by_config.get(default)
    row = {
        "problem": problem.shape_key, "dtype": problem.dtype_name,
        "generated": result.generated, "feasible": result.feasible, "tested": result.tested,
        "correct": result.correct, "statuses": result.status_counts(),
        "winner": None, "winner_us": None, "default_us": None, "speedup_over_default": None,
        "winner_gate_error": None, "winner_gated": False, "cached": False,
        "torch_eager_us": None,
    }
    if "torch_eager" in result.baselines:
        row["torch_eager_us"] = round(result.baselines["torch_eager"].median_us, 2)
    if best is None:
        return row
    row.update(winner=best.config.as_dict(), winner_us=round(best.timing.median_us, 2),
               winner_gate_error=best.verification.error if best.verification else None,
               winner_gated=bool(best.verification and best.verification.passed))
    if default_outcome is not None and default_outcome.timing is not None:
        row["default_us"] = round(default_outcome.timing.median_us, 2)
        row["speedup_over_default"] = round(default_outcome.timing.median_us / best.timing.median_us, 3)
    if cache is not None:
        row["cached"] = cache.get(problem, result.environment.device_key) == best.config
    return row


def render_markdown(rows: list[dict], environment: dict) -> str:
    lines = [
        "# Tuner sweep on sm_100a",
        "",
        f"Device: {environment.get('gpu_name')} ({environment.get('device_key')}), driver "
        f"{environment.get('driver_version')}, torch {environment.get('torch_version')}, "
        f"{environment.get('workers')} worker(s); {environment.get('timestamp')}.",
        "",
        "| problem | dtype | grid | feasible | tested | correct | failures | winner | winner us | "
        "default us | vs default | torch us | gate err | cached |",
        "|---|---|---|---|---|---|---|---|---|---|---|---|---|---|",
    ]
    for r in rows:
        failures = ", ".join(f"{k} {v}" for k, v in sorted(r["statuses"].items()) if k != "ok") or "-"
        w = r["winner"] or {}
        winner = "-" if not w else " ".join(f"{k}={v}" for k, v in w.items() if k not in ("GROUP_M", "SWAP_AB",
                                                                                            "CLUSTER_N"))
        err = "-" if r["winner_gate_error"] is None else f"{r['winner_gate_error']:.1e}"
        lines.append(f"| {r['problem']} | {r['dtype']} | {r['generated']} | {r['feasible']} | {r['tested']} | "
                     f"{r['correct']} | {failures} | {winner} | {r['winner_us']} | {r['default_us']} | "
                     f"{r['speedup_over_default']} | {r['torch_eager_us']} | {err} | {r['cached']} |")
    ok = all(r["winner_gated"] and r["cached"] for r in rows)
    lines += ["", f"Every winner passed the gate and is cached: {'yes' if ok else 'NO'}."]
    return "\n".join(lines) + "\n"


def run(args) -> int:
    from kernelo_b200.db import ResultsDB
    from kernelo_b200.distributed import distributed_tune, world_info
    from kernelo_b200.kernels import get_operator
    from kernelo_b200.runtime.env import capture_environment
    from kernelo_b200.tuning.cache import ConfigCache
    from kernelo_b200.tuning.tuner import Tuner

    world, rank = world_info()
    device = torch.device("cuda", torch.cuda.current_device())
    db = ResultsDB(args.db) if rank == 0 else None
    cache = ConfigCache(args.cache) if rank == 0 else None
    log = print if rank == 0 else None
    tuner = Tuner(warmup=args.warmup, iterations=args.iterations, max_candidates=args.max_candidates,
                  db=db, cache=cache, log=log, resume=args.resume and rank == 0)
    operator = get_operator("matmul")
    rows = []
    for dtype in args.dtypes:
        for problem in workloads.problems("matmul", "sweep_sm100", dtype):
            if rank == 0:
                print(f"\n== {problem.describe()}", flush=True)
            result = (distributed_tune(tuner, operator, problem, device=device) if world > 1
                      else tuner.tune(operator, problem, device=device))
            if rank == 0:
                rows.append(summarize_result(result, operator, cache))
                print(json.dumps(rows[-1]), flush=True)
    if rank == 0:
        env = capture_environment(device).as_dict()
        env["workers"] = world
        out = Path(args.out)
        out.mkdir(parents=True, exist_ok=True)
        (out / "sweep_sm100.json").write_text(json.dumps({"environment": env, "problems": rows}, indent=1))
        (out / "sweep_sm100.md").write_text(render_markdown(rows, env))
        db.close()
        failed = [r["problem"] + " " + r["dtype"] for r in rows if not (r["winner_gated"] and r["cached"])]
        print(f"\n{len(rows)} problems; winners gated and cached: {len(rows) - len(failed)}", flush=True)
        return 1 if failed else 0
    return 0


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--db", default="results/sweep_sm100.db")
    p.add_argument("--cache", default="results/sweep_sm100_configs.json")
    p.add_argument("--out", default="results")
    p.add_argument("--dtypes", nargs="+", default=list(DTYPES), choices=DTYPES)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--iterations", type=int, default=50)
    p.add_argument("--max-candidates", type=int, default=None)
    p.add_argument("--resume", action="store_true")
    args = p.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        return run(args)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
