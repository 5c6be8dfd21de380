"""The decoder block that calls the hot path (``kernelo_b200.integration``).

Both backends share one module and one set of weights, so whatever differs
between their outputs comes from the swapped kernels (the two RMSNorms and the
fused up-projection + bias + GELU). Geometry and backend validation, and the
PyTorch backend's wiring, are checked on the CPU; the native backend needs a
GPU. The reference runs the same experiment (its tests/test_transformer.py).
"""

from __future__ import annotations

import pytest
import torch

from kernelo_b200.integration.transformer import (
    BACKEND_KERNELFORGE,
    BACKEND_TORCH,
    AmdahlBreakdown,
    BlockConfig,
    TransformerBlock,
)
from kernelo_b200.testing import assert_verified

TINY = BlockConfig(hidden=256, heads=8, intermediate=512)


def _block(config=TINY, *, device="cuda", dtype=torch.float16, std=None, **kw) -> TransformerBlock:
    torch.manual_seed(0)
    block = TransformerBlock(config, device=device, dtype=dtype, **kw)
    if std is not None:
        with torch.no_grad():
            for p in block.parameters():
                p.normal_(0.0, std)
    return block


def _outputs_agree(block: TransformerBlock, x: torch.Tensor, label: str) -> None:
    with torch.inference_mode():
        outputs = {}
        for name in (BACKEND_TORCH, BACKEND_KERNELFORGE):
            block.backend = name
            outputs[name] = block(x)
    assert_verified(outputs[BACKEND_TORCH], outputs[BACKEND_KERNELFORGE], dtype=x.dtype, context=label)


# ------------------------------------------------------------------ CPU
def test_geometry_is_validated_and_derived():
    with pytest.raises(ValueError, match="not divisible"):
        BlockConfig(hidden=96, heads=7, intermediate=128)
    default = BlockConfig()
    assert (default.hidden, default.heads, default.intermediate, default.head_dim) == (4096, 32, 11008, 128)


def test_backend_names_are_checked_on_construction_and_assignment():
    block = _block(device="cpu", dtype=torch.float32)
    with pytest.raises(ValueError, match="backend must be one of"):
        block.backend = "eager"
    with pytest.raises(ValueError, match="backend must be one of"):
        TransformerBlock(TINY, device="cpu", dtype=torch.float32, backend="cublas")


def test_torch_backend_shapes_and_residuals_on_the_cpu():
    """With every weight zero the attention and MLP branches add nothing: the
    block is the identity, which checks both residual connections."""
    block = _block(device="cpu", dtype=torch.float32)
    x = torch.randn(3, 5, TINY.hidden)
    with torch.inference_mode():
        y = block(x)
        assert y.shape == x.shape and torch.isfinite(y).all()
        for p in block.parameters():
            p.zero_()
        assert torch.equal(block(x), x)


def test_amdahl_arithmetic():
    """The swapped operators held 60 % of the torch block and got 3x faster:
    Amdahl predicts 1 / (0.4 + 0.2) = 1.667x."""
    br = AmdahlBreakdown(block_ms={BACKEND_TORCH: 10.0, BACKEND_KERNELFORGE: 7.0},
                         swapped_ms={BACKEND_TORCH: 6.0, BACKEND_KERNELFORGE: 2.0})
    assert br.swapped_share == pytest.approx(0.6) and br.operator_speedup == pytest.approx(3.0)
    assert br.predicted_block_speedup == pytest.approx(1 / 0.6)
    assert br.measured_block_speedup == pytest.approx(10 / 7)
    assert "Amdahl" in br.render()


# ------------------------------------------------------------------ GPU
@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_one_set_of_weights_two_backends(dtype, device):
    block = _block(device=device, dtype=dtype, std=0.02)
    _outputs_agree(block, torch.randn(2, 96, TINY.hidden, device=device, dtype=dtype), f"block {dtype}")


@pytest.mark.gpu
@pytest.mark.parametrize("seq", [1, 9, 160])
def test_decode_and_ragged_prefill_lengths(seq, device):
    """One token takes the decode-shape kernels, odd lengths the masked edges."""
    block = _block(device=device)
    _outputs_agree(block, torch.randn(1, seq, TINY.hidden, device=device, dtype=torch.float16), f"seq={seq}")


@pytest.mark.gpu
def test_llama_shapes_one_token(device):
    block = _block(BlockConfig(), device=device, std=0.02)
    _outputs_agree(block, torch.randn(1, 1, 4096, device=device, dtype=torch.float16), "4096/11008, one token")


@pytest.mark.gpu
def test_malformed_inputs_are_refused(device):
    block = _block(device=device)
    with pytest.raises(ValueError, match=r"\(batch, seq, hidden\)"):
        block(torch.zeros(8, TINY.hidden, device=device, dtype=torch.float16))
    with pytest.raises(ValueError, match="expected hidden"):
        block(torch.zeros(1, 3, 2 * TINY.hidden, device=device, dtype=torch.float16))


@pytest.mark.gpu
def test_native_configs_resolve_once_per_shape(device):
    block = _block(device=device, backend=BACKEND_KERNELFORGE)
    x = torch.randn(2, 32, TINY.hidden, device=device, dtype=torch.float16)
    with torch.inference_mode():
        block(x)
        first = block.resolved_configs
        block(x)
    assert block.resolved_configs == first
    assert sorted({key[0] for key in first}) == ["fused_linear", "rmsnorm"]
    assert {key[1] for key in first} == {64}  # 2 x 32 tokens


@pytest.mark.gpu
def test_block_timing_and_breakdown(device):
    from kernelo_b200.integration import amdahl_breakdown, benchmark_block

    timings = benchmark_block(TINY, seq=64, device=device, warmup=2, iterations=4)
    assert set(timings) == {BACKEND_TORCH, BACKEND_KERNELFORGE}
    assert all(t.timer == "cuda_event" and t.median_ms > 0 for t in timings.values())
    br = amdahl_breakdown(TINY, seq=64, device=device, warmup=2, iterations=4)
    assert 0 < br.swapped_share < 1 and br.measured_block_speedup > 0
