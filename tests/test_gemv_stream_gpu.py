"""The streamed 16-row tile GEMV (csrc/gemv_stream.cu) on the B200, against the CPU oracle.

The kernel keeps a shared-memory ring of TMA weight tiles per SM and walks
its tiles in groups, chunk-major; these tests cover the baseline decode
shapes, ragged N (a last tile past the weight, zero-filled) and ragged K (a
last chunk and a last TMA box past K), one and several groups per CTA and a
short last group, both chunk sizes and ring depths down to two stages, the
fused-linear epilogues, run-to-run determinism, the library's choice of
kernel, and programmatic dependent launch: chains of GEMVs, each reading the
previous one's output, give the same bits with overlap as in stream order,
eagerly and replayed from a CUDA graph.
"""

from __future__ import annotations

import pytest
import torch

from kernelo_b200.kernels import gemm_common as gc
from kernelo_b200.kernels.fused_linear import fused_linear_gelu
from kernelo_b200.kernels.gemv import default_config, gemv
from kernelo_b200.runtime import native
from kernelo_b200.tuning.config import KernelConfig
from oracle import cpu_reference as ref
from tests.parity import gate, host

pytestmark = pytest.mark.gpu


def stream_cfg(op="gemv", **kw):
    return KernelConfig(op, KERNEL=gc.KERNEL_TILE_STREAM, **kw)


def operands(m, n, k, dtype, device, seed):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=gen).to(dtype).to(device)
    w = (torch.randn(n, k, generator=gen) * k ** -0.5).to(dtype).to(device)
    return x, w


@pytest.mark.parametrize("m", [1, 4, 16])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_baseline_decode_shape(m, dtype, device):
    """11008 x 4096 weight, M in {1, 4, 16}; repeated
    calls give the same bits (fixed warp order in the tile sums)."""
    x, w = operands(m, 11008, 4096, dtype, device, seed=m)
    out = gemv(x, w, config=stream_cfg())
    gate(ref.gemv_ref(host(x), host(w)), out, dtype, context=f"M={m} 11008x4096")
    assert torch.equal(out, gemv(x, w, config=stream_cfg()))


@pytest.mark.parametrize("m,n,k", [(1, 1000, 1032), (3, 16581, 1032), (9, 4093, 4104), (16, 33, 8),
                                   (2, 17, 520), (13, 3000, 2048), (16, 2, 16), (7, 100, 4096),
                                   (16, 4096, 11008), (5, 2368, 512)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_ragged_shapes(m, n, k, dtype, device):
    """N off the 16-row grid (the TMA box reads zeros past the weight), K off
    the chunk and box grid (zeros past K, x masked), x rows beyond M masked,
    fewer tiles than SMs (one tile per CTA) and long K."""
    x, w = operands(m, n, k, dtype, device, seed=n + k)
    y = torch.full((m, n), float("nan"), dtype=dtype, device=device)
    gemv(x, w, config=stream_cfg(), out=y)
    gate(ref.gemv_ref(host(x), host(w)), y, dtype, context=f"{m}x{n}x{k}")


@pytest.mark.parametrize("chunk,stages", [(1024, 0), (1024, 2), (1024, 3), (512, 0), (512, 2), (512, 7)])
@pytest.mark.parametrize("ctas", [0, 1, 5, 37])
def test_ring_and_grid_variants(chunk, stages, ctas, device):
    """Both chunk sizes, ring depths down to two stages, and small grids, so a
    CTA walks many groups of tiles (6 per group at M > 8) with a short last
    group and wraps the ring many times."""
    x, w = operands(16, 1000, 2056, torch.float16, device, seed=chunk + stages + ctas)
    cfg = stream_cfg(BLOCK_K=chunk, num_stages=stages, NUM_CTAS=ctas)
    out = gemv(x, w, config=cfg)
    gate(ref.gemv_ref(host(x), host(w)), out, torch.float16, context=f"chunk {chunk} stages {stages} ctas {ctas}")


@pytest.mark.parametrize("m", [1, 8])
def test_eight_tile_groups_at_up_to_eight_rows(m, device):
    """Up to 8 rows of x a group holds 8 tiles; 3 CTAs over 63 tiles leave
    groups of 8 and a last one of 5."""
    x, w = operands(m, 63 * 16 - 3, 1024, torch.bfloat16, device, seed=m)
    out = gemv(x, w, config=stream_cfg(NUM_CTAS=3))
    gate(ref.gemv_ref(host(x), host(w)), out, torch.bfloat16, context=f"M={m} 3 CTAs")


@pytest.mark.parametrize("approximate", ["none", "tanh"])
@pytest.mark.parametrize("m,n,k", [(16, 11008, 4096), (1, 5000, 1024), (11, 777, 2056)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fused_linear_epilogue(approximate, m, n, k, dtype, device):
    """The decode-shape fused linear (bias, then exact or tanh GELU, one
    rounding) through kf_linear_bias_act on the streamed kernel."""
    x, w = operands(m, n, k, dtype, device, seed=n)
    gen = torch.Generator().manual_seed(k)
    b = (torch.randn(n, generator=gen) * 0.316).to(dtype).to(device)
    y = fused_linear_gelu(x, w.t(), b, approximate=approximate, config=stream_cfg("fused_linear"))
    expected = ref.linear_gelu_ref(host(x), host(w.t()), host(b), approximate)
    gate(expected, y, dtype, context=f"{approximate} {m}x{n}x{k}")


@pytest.mark.parametrize("cfg", [None, stream_cfg()], ids=["library", "stream"])
@pytest.mark.parametrize("m", [1, 4, 16])
def test_overlap_chain_matches_stream_order(cfg, m, device):
    """Each GEMV reads the previous one's output. With overlap every launch
    may start before its predecessor finishes (programmatic dependent launch)
    and must still read the finished x: the chain's bits equal those of the
    same kernel in ordinary stream order (the library's choice with overlap
    at this shape, 128 tiles, is the streamed kernel), eagerly and from a
    CUDA graph."""
    gen = torch.Generator().manual_seed(100 + m)
    ws = [(torch.randn(2048, 2048, generator=gen) * 2048 ** -0.5).half().to(device) for _ in range(6)]
    x0 = torch.randn(m, 2048, generator=gen).half().to(device)

    def chain(config, overlap):
        h = x0
        for w in ws * 4:
            h = gemv(h, w, config=config, overlap=overlap)
        return h

    ordered = chain(stream_cfg(), False)
    overlapped = chain(cfg, True)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        replayed = chain(cfg, True)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.isfinite(ordered).all()
    assert torch.equal(ordered, overlapped)
    assert torch.equal(ordered, replayed)
    del graph


def test_library_choice(device):
    """The library takes the streamed kernel beyond 8 rows of x when K is long
    or the tiles are many; with overlap also beyond 8 rows at any N, for long
    K and for few tiles; the register-fed kernel otherwise (the Python mirror
    agrees with what runs)."""
    assert default_config(16, 4096, 11008, torch.float16)["KERNEL"] == gc.KERNEL_TILE_STREAM
    assert default_config(16, 44032, 4096, torch.bfloat16)["KERNEL"] == gc.KERNEL_TILE_STREAM
    assert default_config(16, 11008, 4096, torch.float16)["KERNEL"] == gc.KERNEL_TILE_ROWS
    assert default_config(8, 4096, 11008, torch.float16)["KERNEL"] == gc.KERNEL_TILE_ROWS
    assert gc.tile_stream_preferred(16, 11008, 4096, overlap=True)
    assert not gc.tile_stream_preferred(16, 11008, 4096)  # the register-fed kernel's best shape
    assert gc.tile_stream_preferred(1, 4096, 11008, overlap=True)  # long K
    assert gc.tile_stream_preferred(1, 2048, 2048, overlap=True)  # 128 tiles, under 4 per SM
    assert not gc.tile_stream_preferred(1, 11008, 4096, overlap=True)
    assert not gc.tile_stream_preferred(17, 11008, 4096, overlap=True)
    x, w = operands(16, 4096, 11008, torch.float16, device, seed=5)
    gate(ref.gemv_ref(host(x), host(w)), gemv(x, w), torch.float16, context="library choice, long K")
    x, w = operands(4, 4096, 11008, torch.float16, device, seed=6)
    gate(ref.gemv_ref(host(x), host(w)), gemv(x, w, overlap=True), torch.float16, context="library choice, overlap")


def test_rejects_what_it_cannot_run(device):
    """More than 16 rows, fp32, K off the 16-byte grid, a chunk or ring depth
    it was not built for: clean errors, nothing launched."""
    x, w = operands(17, 256, 512, torch.float16, device, seed=1)
    with pytest.raises(native.OutOfResources, match="1..16 rows"):
        gemv(x, w, config=stream_cfg())
    x, w = operands(4, 256, 512, torch.float32, device, seed=1)
    with pytest.raises(native.OutOfResources, match="fp16 or bf16"):
        gemv(x, w, config=stream_cfg())
    x, w = operands(4, 256, 515, torch.float16, device, seed=1)
    with pytest.raises(native.OutOfResources, match="multiple of 8"):
        gemv(x, w, config=stream_cfg())
    x, w = operands(4, 256, 512, torch.float16, device, seed=1)
    with pytest.raises(native.OutOfResources, match="chunk"):
        gemv(x, w, config=stream_cfg(BLOCK_K=256))
    with pytest.raises(native.OutOfResources, match="stages"):
        gemv(x, w, config=stream_cfg(num_stages=1))
