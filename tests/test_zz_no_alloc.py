"""kf_gemv_noalloc against kf_gemv and the CPU oracle, through the C ABI.

kf_gemv_noalloc serves callers that cannot allocate device memory -- a plugin
inside a host application that owns all device allocations and offers no
workspace, or a latency-critical path that cannot pay for cudaMalloc/cudaFree
-- by keeping the GEMV's stream-K scratch in a fixed device array inside the
library ([N, K] 16-bit weights take the tile kernel, which needs none). Two
calls in a row (the second finds the array as the first left it) must agree
with the workspace-taking entry point and with the float64 oracle within the
reference's gate for the dtype.

This file is named to be collected last; it passes on its own in a fresh
process as well as after the rest of the suite.
"""

from __future__ import annotations

import pytest
import torch

from kernelo_b200.runtime import native
from kernelo_b200.testing import assert_verified
from oracle import cpu_reference as ref

pytestmark = pytest.mark.gpu

_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def _w_strides(w, layout):
    """(sw_n, sw_k) of W stored [N, K] ("nk") or [K, N] ("kn")."""
    return (w.stride(0), w.stride(1)) if layout == "nk" else (w.stride(1), w.stride(0))


def _call_noalloc(x, w, y, layout="nk"):
    lib = native.load()
    m, k = x.shape
    n = y.shape[1]
    sw_n, sw_k = _w_strides(w, layout)
    return lib.kf_gemv_noalloc(_CODE[x.dtype], x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), sw_n,
                               sw_k, y.data_ptr(), y.stride(0), y.stride(1), m, n, k,
                               native.current_stream_handle(y.device))


def _call_with_workspace(x, w, y, layout="nk"):
    lib = native.load()
    m, k = x.shape
    n = y.shape[1]
    dev = y.device
    sw_n, sw_k = _w_strides(w, layout)
    need = lib.kf_gemv_workspace_bytes(dev.index, _CODE[x.dtype], x.stride(0), x.stride(1), sw_n, sw_k, m, n,
                                       k, None)
    assert need >= 0
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device=dev)
    status = lib.kf_gemv(_CODE[x.dtype], x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), sw_n, sw_k,
                         y.data_ptr(), y.stride(0), y.stride(1), m, n, k, None, ws.data_ptr(), need,
                         native.current_stream_handle(dev))
    native.check(status, "kf_gemv")
    torch.cuda.synchronize(dev)
    return ws


def _check_twice(x, w, layout, n, device):
    """Two no-alloc calls in a row against kf_gemv and the float64 oracle."""
    m = x.shape[0]
    expected = torch.empty(m, n, device=device, dtype=x.dtype)
    _call_with_workspace(x, w, expected, layout)
    w_nk = w if layout == "nk" else w.t()
    oracle = torch.from_numpy(ref.gemv_ref(x.cpu().double().numpy(), w_nk.cpu().double().numpy()))
    for attempt in range(2):
        y = torch.full((m, n), float("nan"), device=device, dtype=x.dtype)
        native.check(_call_noalloc(x, w, y, layout), "kf_gemv_noalloc")
        torch.cuda.synchronize(device)
        assert_verified(expected.float(), y.float(), dtype=x.dtype, context=f"vs kf_gemv, call {attempt}")
        assert_verified(oracle, y.cpu().double(), dtype=x.dtype, context=f"vs oracle, call {attempt}")
    assert native.device_status(device.index) == 0


@pytest.mark.parametrize("m", [1, 4, 16])
@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_noalloc_gemv_matches_the_workspace_entry_point_twice(m, layout, device):
    """[N, K] weights take the tile kernel (no scratch); [K, N] weights the
    stream-K kernel on the library's scratch array."""
    gen = torch.Generator().manual_seed(11 + m)
    x = torch.randn(m, 4096, generator=gen).half().to(device)
    w = (torch.randn(11008, 4096, generator=gen) * 4096 ** -0.5).half().to(device)
    if layout == "kn":
        w = w.t().contiguous()
    _check_twice(x, w, layout, 11008, device)


@pytest.mark.parametrize(
    "dtype,m,k,layout",
    [
        (torch.bfloat16, 16, 4096, "kn"),  # stream-K tcgen05 GEMV, bf16
        (torch.float32, 1, 1024, "nk"),  # warp-per-row kernel
        (torch.float32, 8, 1024, "kn"),  # CUDA-core GEMM (no fp32 MMA)
        (torch.float16, 4, 1028, "nk"),  # K % 8 != 0: rows off the 16-byte grid
    ],
)
def test_noalloc_takes_every_input_kf_gemv_takes(dtype, m, k, layout, device):
    gen = torch.Generator().manual_seed(31 + m + k)
    n = 2304
    x = torch.randn(m, k, generator=gen).to(dtype).to(device)
    w = (torch.randn(n, k, generator=gen) * k ** -0.5).to(dtype).to(device)
    if layout == "kn":
        w = w.t().contiguous()
    _check_twice(x, w, layout, n, device)


def test_noalloc_rejects_more_rows_than_its_scratch_holds(device):
    x = torch.randn(17, 256, device=device, dtype=torch.float16)
    w = torch.randn(512, 256, device=device, dtype=torch.float16)
    y = torch.empty(17, 512, device=device, dtype=torch.float16)
    status = _call_noalloc(x, w, y)
    assert status == native.KF_ERR_WORKSPACE
    assert "at most 16 rows" in native.last_error()


def test_noalloc_rejects_a_call_whose_scratch_exceeds_the_array(device):
    """x with unit stride along M gives the swapped GEMV 64-column tiles, whose
    stream-K partials need more than the fixed array: refused, nothing written."""
    lib = native.load()
    m, k, n = 16, 4096, 11008
    x = torch.randn(k, m, device=device, dtype=torch.float16).t()  # strides (1, m)
    w = torch.randn(k, n, device=device, dtype=torch.float16)  # [K, N]
    need = lib.kf_gemv_workspace_bytes(device.index, 0, x.stride(0), x.stride(1), 1, n, m, n, k, None)
    assert need > lib_scratch_bytes()
    y = torch.full((m, n), float("nan"), device=device, dtype=torch.float16)
    status = _call_noalloc(x, w, y, "kn")
    assert status == native.KF_ERR_WORKSPACE
    assert "above the fixed" in native.last_error()
    torch.cuda.synchronize(device)
    assert torch.isnan(y).all()


def lib_scratch_bytes() -> int:
    return 4 * 1024 * 1024  # KF_NOALLOC_SCRATCH_BYTES in include/kernelo_b200.h
