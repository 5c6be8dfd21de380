"""fp32 GEMM on tensor cores as 3xTF32 (csrc/tf32_split.cu + the tcgen05 kernel
on kind::tf32), held to the reference's fp32 gate of 1e-5
(kernelforge/testing.py:31-35) against the CPU fp32 oracle.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from kernelo_b200.kernels.fused_linear import fused_linear_gelu
from kernelo_b200.kernels.matmul import matmul
from kernelo_b200.runtime import native
from kernelo_b200.tuning.config import KernelConfig
from oracle import cpu_reference as ref
from tests.parity import gate, host, sample_rows

pytestmark = pytest.mark.gpu


def operands(m, k, n, device, seed=0):
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(m, k, generator=gen).to(device), torch.randn(k, n, generator=gen).to(device))


def tf32_cfg(op="matmul", **kw):
    # a TF32 stage holds both split parts: 8 bytes per (row, k)
    base = dict(KERNEL=1, BLOCK_M=128, BLOCK_N=128, BLOCK_K=32, GROUP_M=8, num_stages=3, STREAM_K=2, SWAP_AB=2)
    base.update(kw)
    return KernelConfig(op, **base)


def split_workspace_bytes(a, b, c) -> int:
    """Workspace the library plans for this call: the TF32 split copies make it
    at least 8 bytes per operand element (0 or the stream-K state otherwise)."""
    lib = native.load()
    cfg = native.GemmLaunch().struct()
    return lib.kf_gemm_workspace_bytes_for(a.device.index or 0, native.native_code(a.dtype), a.data_ptr(),
                                           a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
                                           c.data_ptr(), c.stride(0), c.stride(1), a.shape[0], b.shape[1],
                                           a.shape[1], ctypes.byref(cfg))


def ran_on_tensor_cores(a, b, out) -> bool:
    """The default path planned the split (workspace for both TF32 copies) and
    its result is not the CUDA-core kernel's bit for bit."""
    planned = split_workspace_bytes(a, b, out) >= 8 * (a.numel() + b.numel())
    simt = matmul(a, b, config=KernelConfig("matmul", KERNEL=2, BLOCK_M=128, BLOCK_N=128, BLOCK_K=8))
    return planned and not torch.equal(simt, out)


@pytest.mark.parametrize("shape", [(512, 1024, 256), (640, 520, 1000), (1021, 2053, 509), (2048, 4096, 4096)],
                         ids=lambda s: "x".join(map(str, s)))
def test_default_fp32_runs_3xtf32_at_the_fp32_gate(shape, device):
    m, k, n = shape[0], shape[2], shape[1]
    a, b = operands(m, k, n, device, seed=m + n)
    out = matmul(a, b)
    assert ran_on_tensor_cores(a, b, out)
    rows = sample_rows(m, 64)
    result = gate(ref.matmul_ref(host(a[rows]), host(b)), out[rows], torch.float32, context=f"{shape}")
    assert result.error < 1e-5


@pytest.mark.parametrize("cfg", [
    dict(BLOCK_K=32), dict(BLOCK_N=64, BLOCK_K=64, num_stages=2), dict(BLOCK_N=64, STREAM_K=1),
    dict(BLOCK_M=256, BLOCK_N=128, BLOCK_K=32, num_stages=4, CLUSTER_M=2, STREAM_K=3),
    dict(BLOCK_N=16, num_stages=6), dict(SWAP_AB=1, BLOCK_N=64),
], ids=lambda c: "-".join(f"{k}{v}" for k, v in c.items()))
@pytest.mark.parametrize("shape", [(300, 200, 100), (640, 520, 1000), (70, 4099, 33)],
                         ids=lambda s: "x".join(map(str, s)))
def test_explicit_tf32_tiles(cfg, shape, device):
    """Every tile shape, schedule and swap of the kernel on TF32 operands, at
    ragged M/N and K not a multiple of the 32-element atom."""
    m, n, k = shape
    a, b = operands(m, k, n, device, seed=k)
    out = matmul(a, b, config=tf32_cfg(**cfg))
    gate(ref.matmul_ref(host(a), host(b)), out, torch.float32, context=f"{shape} {cfg}")


def test_tf32_layouts_and_views(device):
    """The split reads any strides: a transposed A, B as an nn.Linear [N, K]
    weight's transpose (K-contiguous), column slices off the 16-byte grid."""
    gen = torch.Generator().manual_seed(3)
    a_t = torch.randn(384, 200, generator=gen).to(device).t()  # A [200, 384], M-contiguous
    w = torch.randn(330, 384, generator=gen).to(device)  # B = w.t(): [384, 330], K-contiguous
    gate(ref.matmul_ref(host(a_t), host(w.t())), matmul(a_t, w.t()), torch.float32)
    base = torch.randn(260, 515, generator=gen).to(device)
    a = base[:, 3:500]  # K = 497, odd base, row pitch 515
    b = torch.randn(497, 301, generator=gen).to(device)
    gate(ref.matmul_ref(host(a), host(b)), matmul(a, b), torch.float32)
    out = torch.empty(260, 400, device=device)[:, 7:308]  # C off the 16-byte grid
    from kernelo_b200.runtime.native import gemm

    gemm(a, b, out)
    gate(ref.matmul_ref(host(a), host(b)), out, torch.float32)


@pytest.mark.parametrize("approximate", ["none", "tanh"])
def test_fp32_fused_linear_on_tf32(approximate, device):
    gen = torch.Generator().manual_seed(7)
    x = torch.randn(400, 512, generator=gen).to(device)  # 1.4e8 multiply-adds: past the 2^27 threshold
    w = (torch.randn(700, 512, generator=gen) * 512 ** -0.5).to(device)
    b = (torch.randn(700, generator=gen) * 0.3).to(device)
    out = fused_linear_gelu(x, w.t(), b, approximate=approximate)
    assert split_workspace_bytes(x, w.t(), out) >= 8 * (x.numel() + w.numel())
    expect = ref.linear_gelu_ref(host(x), host(w.t()), host(b), approximate=approximate)
    gate(expect, out, torch.float32)


def test_tf32_tiles_refuse_blocks_wider_than_their_register_sums(device):
    a, b = operands(256, 256, 512, device)
    with pytest.raises(native.OutOfResources, match="BLOCK_N must be at most 128"):
        matmul(a, b, config=tf32_cfg(BLOCK_N=256))


def test_tf32_accuracy_holds_over_long_k(device):
    """Accumulator chunks summed in fp32 registers keep the error flat in K
    (one TMEM chain of K = 16384 measured 3.8e-5, over the gate)."""
    a, b = operands(256, 16384, 256, device, seed=5)
    result = gate(ref.matmul_ref(host(a), host(b)), matmul(a, b), torch.float32)
    assert result.error < 2e-6


def test_small_fp32_keeps_ieee_fma(device):
    """Below 2^27 multiply-adds fp32 stays on the CUDA-core kernel: no split
    planned, and the result is that kernel's bit for bit."""
    a, b = operands(257, 257, 257, device)
    out = matmul(a, b)
    assert split_workspace_bytes(a, b, out) < 8 * (a.numel() + b.numel())
    simt = matmul(a, b, config=KernelConfig("matmul", KERNEL=2, BLOCK_M=64, BLOCK_N=64, BLOCK_K=16))
    assert torch.equal(simt, out)
