"""Generate the golden fixtures in this directory from the reference itself.

Run once, on a machine holding the KernelForge source tree (it is never run by
the tests, which only read the ``.npz`` files):

    python tests/golden/make_golden.py --reference /path/to/KernelO

For each case this script
  1. builds the inputs with the reference's own ``Operator.make_inputs`` on the
     CPU (so the input distributions are pinned too);
  2. records the reference's own gate reference (``Operator.reference`` /
     ``linear_gelu_reference`` / ``rmsnorm_reference`` / ``torch.softmax``),
     computed by torch on the CPU in the operand dtype, as ``ref_torch``;
  3. for fp16/fp32, runs the reference's Triton kernel itself under
     ``TRITON_INTERPRET=1`` and records it as ``ref_kernel`` (bf16 is skipped:
     the interpreter mis-handles bf16, an interpreter artefact).
Inputs and outputs are stored as float32 holding the exact operand values.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _np(t):
    return t.detach().to("cpu").float().numpy()


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="root of the KernelForge source tree")
    args = parser.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"  # must precede the first triton import
    sys.path.insert(0, str(Path(args.reference).resolve()))

    import torch
    import torch.nn.functional as F

    from kernelforge.kernels import fused_linear as ref_fl
    from kernelforge.kernels import matmul as ref_mm
    from kernelforge.kernels import rmsnorm as ref_rms
    from kernelforge.kernels import softmax as ref_sm
    from kernelforge.testing import exact_fp32_matmul
    from kernelforge.tuning.config import Problem

    cpu = torch.device("cpu")
    manifest = []

    def save(name: str, meta: dict, inputs: list, ref_torch, ref_kernel=None) -> None:
        arrays = {f"in{i}": _np(t) for i, t in enumerate(inputs)}
        arrays["ref_torch"] = _np(ref_torch)
        if ref_kernel is not None:
            arrays["ref_kernel"] = _np(ref_kernel)
        arrays["meta"] = np.array(json.dumps(meta))
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
        manifest.append({"name": name, **meta, "has_kernel_output": ref_kernel is not None})
        print(name, "kernel" if ref_kernel is not None else "")

    def interp(fn):
        try:
            return fn()
        except Exception as exc:  # interpreter gaps are recorded, not fatal
            print("  interpreter failed:", type(exc).__name__, str(exc)[:120])
            return None

    dtypes = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}

    # ---- matmul (kernels/matmul.py)
    for (m, n, k) in ((127, 129, 65), (33, 70, 100), (1, 128, 128), (64, 64, 8)):
        for dn, dt in dtypes.items():
            p = Problem.create("matmul", dn, M=m, N=n, K=k)
            op = ref_mm.MatmulOperator()
            a, b = op.make_inputs(p, cpu, seed=0)
            ref = op.reference(a, b)
            kern = None if dn == "bf16" else interp(lambda: ref_mm.matmul(a, b, config=ref_mm.DEFAULT_CONFIG))
            save(f"matmul_{dn}_{m}x{n}x{k}", {"op": "matmul", "dtype": dn, "M": m, "N": n, "K": k},
                 [a, b], ref, kern)

    # ---- fused linear, tanh GELU (kernels/fused_linear.py)
    for (m, n, k) in ((127, 129, 65), (64, 256, 128), (1, 128, 256)):
        for dn, dt in dtypes.items():
            p = Problem.create("fused_linear", dn, M=m, N=n, K=k)
            op = ref_fl.FusedLinearOperator()
            x, w, b = op.make_inputs(p, cpu, seed=0)
            with exact_fp32_matmul():
                ref = op.reference(x, w, b)
            kern = None if dn == "bf16" else interp(
                lambda: ref_fl.fused_linear_gelu(x, w, b, config=ref_fl.DEFAULT_CONFIG))
            save(f"fused_linear_{dn}_{m}x{n}x{k}",
                 {"op": "fused_linear", "dtype": dn, "M": m, "N": n, "K": k, "approximate": "tanh"},
                 [x, w, b], ref, kern)

    # GELU across its range through an identity weight (tests/test_fused_linear.py:96-122)
    values = torch.cat([torch.linspace(-60.0, 60.0, 512),
                        torch.tensor([-1e4, -100.0, -1e-7, 0.0, 1e-7, 100.0, 1e4])]).float()
    n = values.numel()
    x = values.reshape(1, n).contiguous()
    w = torch.eye(n)
    b = torch.zeros(n)
    kern = interp(lambda: ref_fl.fused_linear_gelu(x, w, b, config=ref_fl.DEFAULT_CONFIG))
    save("fused_linear_gelu_range_fp32", {"op": "fused_linear", "dtype": "fp32", "M": 1, "N": n, "K": n,
                                          "approximate": "tanh", "pin": "gelu_range"},
         [x, w, b], F.gelu(x, approximate="tanh"), kern)
    # bias before activation (tests/test_fused_linear.py:125-139)
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(8, 32, generator=gen)
    w = torch.zeros(32, 64)
    b = torch.linspace(-4.0, 4.0, 64)
    kern = interp(lambda: ref_fl.fused_linear_gelu(x, w, b, config=ref_fl.DEFAULT_CONFIG))
    save("fused_linear_bias_order_fp32", {"op": "fused_linear", "dtype": "fp32", "M": 8, "N": 64, "K": 32,
                                          "approximate": "tanh", "pin": "bias_order"},
         [x, w, b], F.gelu(b, approximate="tanh").expand(8, 64), kern)

    # ---- softmax (kernels/softmax.py)
    for (r, c) in ((3, 127), (17, 257), (4, 1000), (2, 4097)):
        for dn, dt in dtypes.items():
            p = Problem.create("softmax", dn, rows=r, cols=c)
            op = ref_sm.SoftmaxOperator()
            (x,) = op.make_inputs(p, cpu, seed=0)
            ref = op.reference(x)
            kern = None if dn == "bf16" else interp(lambda: ref_sm.softmax(x, config=ref_sm.default_config(c)))
            save(f"softmax_{dn}_{r}x{c}", {"op": "softmax", "dtype": dn, "rows": r, "cols": c}, [x], ref, kern)
    x = torch.full((4, 512), 60.0, dtype=torch.float16)
    x[:, 0] = 80.0
    kern = interp(lambda: ref_sm.softmax(x, config=ref_sm.default_config(512)))
    save("softmax_overflow_logits_fp16", {"op": "softmax", "dtype": "fp16", "rows": 4, "cols": 512,
                                          "pin": "overflow_logits"}, [x], torch.softmax(x.float(), -1), kern)
    x = torch.full((2, 128), -3.5)
    kern = interp(lambda: ref_sm.softmax(x, config=ref_sm.default_config(128)))
    save("softmax_constant_row_fp32", {"op": "softmax", "dtype": "fp32", "rows": 2, "cols": 128,
                                       "pin": "constant_row"}, [x], torch.softmax(x, -1), kern)

    # ---- RMSNorm (kernels/rmsnorm.py), reference eps 1e-5 and the baseline's 1e-6
    for (r, c) in ((3, 127), (17, 257), (4, 4097), (2, 1024)):
        for dn, dt in dtypes.items():
            for eps in (1e-5, 1e-6):
                p = Problem.create("rmsnorm", dn, rows=r, cols=c)
                op = ref_rms.RMSNormOperator()
                x, g = op.make_inputs(p, cpu, seed=0)
                ref = ref_rms.rmsnorm_reference(x, g, eps=eps)
                kern = None if dn == "bf16" else interp(
                    lambda: ref_rms.rmsnorm(x, g, eps=eps, config=ref_rms.default_config(c)))
                save(f"rmsnorm_{dn}_{r}x{c}_eps{eps:g}",
                     {"op": "rmsnorm", "dtype": dn, "rows": r, "cols": c, "eps": eps}, [x, g], ref, kern)
    x = torch.zeros(4, 256, dtype=torch.float16)
    g = torch.ones(256, dtype=torch.float16)
    kern = interp(lambda: ref_rms.rmsnorm(x, g, config=ref_rms.default_config(256)))
    save("rmsnorm_zero_row_fp16", {"op": "rmsnorm", "dtype": "fp16", "rows": 4, "cols": 256, "eps": 1e-5,
                                   "pin": "zero_row"}, [x, g], ref_rms.rmsnorm_reference(x, g), kern)

    (HERE / "MANIFEST.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print(len(manifest), "fixtures")
    return 0


if __name__ == "__main__":
    sys.exit(main())
