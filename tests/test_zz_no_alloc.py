"""kf_gemv_noalloc against kf_gemv, through the C ABI.

kf_gemv_noalloc serves callers that cannot allocate device memory -- a plugin
inside a host application that owns all device allocations and offers no
workspace, or a latency-critical path that cannot pay for cudaMalloc/cudaFree
-- by keeping the GEMV's stream-K scratch in a fixed device array inside the
library ([N, K] 16-bit weights take the tile kernel, which needs none). Two calls in a row (the second finds the array as the first left it)
must agree with the workspace-taking entry point within the fp16 gate.

This file is named to be collected last; it passes on its own in a fresh
process as well as after the rest of the suite.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from kernelo_b200.runtime import native
from kernelo_b200.testing import assert_verified

pytestmark = pytest.mark.gpu


def _w_strides(w, layout):
    """(sw_n, sw_k) of W stored [N, K] ("nk") or [K, N] ("kn")."""
    return (w.stride(0), w.stride(1)) if layout == "nk" else (w.stride(1), w.stride(0))


def _call_noalloc(x, w, y, layout="nk"):
    lib = native.load()
    m, k = x.shape
    n = y.shape[1]
    sw_n, sw_k = _w_strides(w, layout)
    return lib.kf_gemv_noalloc(0, x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), sw_n, sw_k,
                               y.data_ptr(), y.stride(0), y.stride(1), m, n, k,
                               native.current_stream_handle(y.device))


def _call_with_workspace(x, w, y, layout="nk"):
    lib = native.load()
    m, k = x.shape
    n = y.shape[1]
    dev = y.device
    sw_n, sw_k = _w_strides(w, layout)
    need = lib.kf_gemv_workspace_bytes(dev.index, 0, x.stride(0), x.stride(1), sw_n, sw_k, m, n, k, None)
    assert need >= 0
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device=dev)
    status = lib.kf_gemv(0, x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), sw_n, sw_k,
                         y.data_ptr(), y.stride(0), y.stride(1), m, n, k, None, ws.data_ptr(), need,
                         native.current_stream_handle(dev))
    native.check(status, "kf_gemv")
    torch.cuda.synchronize(dev)
    return ws


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
    expected = torch.empty(m, 11008, device=device, dtype=torch.float16)
    _call_with_workspace(x, w, expected, layout)
    for attempt in range(2):
        y = torch.full((m, 11008), float("nan"), device=device, dtype=torch.float16)
        native.check(_call_noalloc(x, w, y, layout), "kf_gemv_noalloc")
        torch.cuda.synchronize(device)
        assert_verified(expected.float(), y.float(), dtype=torch.float16, context=f"call {attempt}")
    assert native.device_status(device.index) == 0


def test_noalloc_rejects_more_rows_than_its_scratch_holds(device):
    x = torch.randn(17, 256, device=device, dtype=torch.float16)
    w = torch.randn(512, 256, device=device, dtype=torch.float16)
    y = torch.empty(17, 512, device=device, dtype=torch.float16)
    status = _call_noalloc(x, w, y)
    assert status == native.KF_ERR_WORKSPACE
    assert "at most 16 rows" in native.last_error()
