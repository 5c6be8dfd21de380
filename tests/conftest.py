"""Shared fixtures.

``gpu``-marked tests run on a B200 and are skipped without a CUDA device; the
rest (oracle pins, host logic, the C-ABI library's exports, gloo multi-process
tests) run on any CPU.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device available")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def device() -> torch.device:
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device available")
    return torch.device("cuda", torch.cuda.current_device())


def load_golden(name: str) -> dict:
    """One fixture: ``inputs`` (float32 arrays), ``ref_torch``, optional ``ref_kernel``, ``meta``."""
    data = np.load(GOLDEN / f"{name}.npz")
    inputs = []
    i = 0
    while f"in{i}" in data:
        inputs.append(data[f"in{i}"])
        i += 1
    return {
        "inputs": inputs,
        "ref_torch": data["ref_torch"],
        "ref_kernel": data["ref_kernel"] if "ref_kernel" in data else None,
        "meta": json.loads(str(data["meta"])),
    }


def golden_names() -> list[str]:
    manifest = json.loads((GOLDEN / "MANIFEST.json").read_text())
    return [entry["name"] for entry in manifest]


@pytest.fixture
def b200_caps():
    from kernelo_b200.runtime.env import DeviceCaps

    return DeviceCaps(
        name="NVIDIA B200",
        compute_capability="10.0",
        total_memory_bytes=183_359 * 1024**2,
        sm_count=148,
        max_shared_memory_per_block=232_448,
        shared_memory_per_sm=233_472,
        registers_per_sm=65_536,
        max_threads_per_sm=2048,
        warp_size=32,
        l2_cache_bytes=126 * 1024 * 1024,
    )


@pytest.fixture
def a100_caps():
    from kernelo_b200.runtime.env import DeviceCaps

    return DeviceCaps(
        name="NVIDIA A100-SXM4-80GB",
        compute_capability="8.0",
        total_memory_bytes=80 * 1024**3,
        sm_count=108,
        max_shared_memory_per_block=166_912,
        shared_memory_per_sm=167_936,
        registers_per_sm=65_536,
        max_threads_per_sm=2048,
        warp_size=32,
        l2_cache_bytes=40 * 1024 * 1024,
        tmem_columns_per_sm=0,
    )
