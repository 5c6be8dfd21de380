"""Transformer-block integration (``tests/test_transformer.py`` of the
reference): both backends run on one module and one set of weights, so any
difference in output comes from the swapped kernels (RMSNorm, fused linear +
GELU). Config validation runs on the CPU; the forward passes need a GPU."""

from __future__ import annotations

import pytest
import torch

from kernelo_b200.integration.transformer import (
    BACKEND_KERNELFORGE,
    BACKEND_TORCH,
    BlockConfig,
    TransformerBlock,
)

SMALL = BlockConfig(hidden=256, heads=8, intermediate=512)


def test_block_config_rejects_an_indivisible_head_count():
    with pytest.raises(ValueError, match="not divisible"):
        BlockConfig(hidden=100, heads=8, intermediate=256)


def test_head_dim_follows_from_the_geometry():
    assert BlockConfig().head_dim == 128
    assert (BlockConfig().hidden, BlockConfig().intermediate) == (4096, 11008)


def test_unknown_backend_is_rejected():
    with pytest.raises(ValueError, match="backend must be one of"):
        TransformerBlock(SMALL, device="cpu", dtype=torch.float32, backend="cutlass")


def test_torch_backend_runs_on_the_cpu():
    """The reference backend is plain PyTorch: the block's shapes and residual
    wiring can be checked without a GPU."""
    torch.manual_seed(0)
    block = TransformerBlock(SMALL, device="cpu", dtype=torch.float32)
    x = torch.randn(2, 16, SMALL.hidden)
    with torch.inference_mode():
        y = block(x)
    assert y.shape == x.shape and torch.isfinite(y).all()


def _parity(block, x, context):
    from kernelo_b200.testing import assert_verified

    with torch.inference_mode():
        block.backend = BACKEND_TORCH
        expected = block(x)
        block.backend = BACKEND_KERNELFORGE
        actual = block(x)
    assert_verified(expected, actual, dtype=x.dtype, context=context)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_backends_agree_on_one_set_of_weights(dtype, device):
    torch.manual_seed(0)
    block = TransformerBlock(SMALL, device=device, dtype=dtype)
    for parameter in block.parameters():
        torch.nn.init.normal_(parameter, std=0.02)
    _parity(block, torch.randn(2, 128, SMALL.hidden, device=device, dtype=dtype), f"block parity {dtype}")


@pytest.mark.gpu
@pytest.mark.parametrize("seq", [1, 7, 128])
def test_parity_holds_for_awkward_sequence_lengths(seq, device):
    """Decode (one token) and ragged prefill reach different kernel paths."""
    torch.manual_seed(0)
    block = TransformerBlock(SMALL, device=device, dtype=torch.float16)
    _parity(block, torch.randn(1, seq, SMALL.hidden, device=device, dtype=torch.float16), f"seq={seq}")


@pytest.mark.gpu
def test_parity_at_llama_geometry_one_token(device):
    """The real shapes (4096 hidden, 11008 intermediate) on a decode step."""
    torch.manual_seed(0)
    block = TransformerBlock(BlockConfig(), device=device, dtype=torch.float16)
    for parameter in block.parameters():
        torch.nn.init.normal_(parameter, std=0.02)
    _parity(block, torch.randn(1, 1, 4096, device=device, dtype=torch.float16), "llama decode")


@pytest.mark.gpu
def test_input_shape_is_validated(device):
    block = TransformerBlock(SMALL, device=device, dtype=torch.float16)
    with pytest.raises(ValueError, match=r"\(batch, seq, hidden\)"):
        block(torch.zeros(4, SMALL.hidden, device=device, dtype=torch.float16))
    with pytest.raises(ValueError, match="expected hidden"):
        block(torch.zeros(1, 4, SMALL.hidden * 2, device=device, dtype=torch.float16))


@pytest.mark.gpu
def test_configurations_are_resolved_once_per_shape(device):
    block = TransformerBlock(SMALL, device=device, dtype=torch.float16, backend=BACKEND_KERNELFORGE)
    x = torch.randn(1, 64, SMALL.hidden, device=device, dtype=torch.float16)
    with torch.inference_mode():
        block(x)
        resolved = dict(block._selected)
        block(x)
    assert block._selected == resolved
    assert {operation for operation, _, _ in block._selected} == {"rmsnorm", "fused_linear"}


@pytest.mark.gpu
def test_benchmark_block_and_amdahl_breakdown(device):
    from kernelo_b200.integration import amdahl_breakdown, benchmark_block

    results = benchmark_block(SMALL, batch=1, seq=128, device=device, warmup=3, iterations=5)
    assert set(results) == {BACKEND_TORCH, BACKEND_KERNELFORGE}
    for timing in results.values():
        assert timing.median_ms > 0 and timing.timer == "cuda_event"
    br = amdahl_breakdown(SMALL, batch=1, seq=128, device=device, warmup=2, iterations=5)
    assert 0 < br.swapped_share < 1
    assert br.predicted_block_speedup > 0 and br.measured_block_speedup > 0
    assert "Amdahl" in br.render()
