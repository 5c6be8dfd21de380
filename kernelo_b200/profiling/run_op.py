"""Run one operator a few times at a given shape: the target of an ncu capture.

    python -m kernelo_b200.profiling.run_op softmax rows=32768 cols=4096 --dtype fp16 --iters 3
    python -m kernelo_b200.profiling.run_op gemv M=1 N=11008 K=4096 --config '{"KERNEL": 3}'

Inputs come from the operator's own seeded ``make_inputs`` (the baseline
distributions); the config is the library default unless ``--config`` gives
KernelConfig parameters as JSON. Prints the kernel-launch count it made so the
``-s``/``-c`` of an ncu command can be chosen, and exits non-zero when the
result fails the correctness gate against the operator's PyTorch reference.
"""

from __future__ import annotations

import argparse
import json
import sys

import torch


def main(argv: list[str] | None = None) -> int:
    from kernelo_b200.kernels import get_operator
    from kernelo_b200.testing import verify
    from kernelo_b200.tuning.config import KernelConfig, Problem

    parser = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    parser.add_argument("op", help="operator name (softmax, rmsnorm, gemv, matmul, fused_linear_erf, ...)")
    parser.add_argument("dims", nargs="+", help="NAME=VALUE dimensions in the operator's order")
    parser.add_argument("--dtype", default="fp16")
    parser.add_argument("--iters", type=int, default=3)
    parser.add_argument("--config", default=None, help="KernelConfig parameters as a JSON object")
    args = parser.parse_args(argv)

    dims = {}
    for item in args.dims:
        name, _, value = item.partition("=")
        dims[name] = int(value)
    op = get_operator(args.op)
    problem = Problem.create(args.op, args.dtype, **dims)
    device = torch.device("cuda", 0)
    inputs = op.make_inputs(problem, device)
    config = KernelConfig(args.op, **json.loads(args.config)) if args.config else op.default_config(problem)
    out = None
    for _ in range(args.iters):
        out = op.run(config, *inputs)
    torch.cuda.synchronize()
    result = verify(op.reference(*inputs).float(), out.float(), dtype=problem.dtype)
    print(f"{args.op} {problem.shape_key} {config}: {args.iters} calls; {result}")
    return 0 if result.passed else 1


if __name__ == "__main__":
    sys.exit(main())
