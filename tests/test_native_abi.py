"""The C-ABI library: builds, loads and exports what the header declares.

No kernel is launched here (no GPU); the device-free entry points
(version, error text, config feasibility) are exercised.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from kernelo_b200.runtime import native

HEADER = Path(__file__).resolve().parent.parent / "include" / "kernelo_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^KF_API\s+[\w\s\*]+?\b(kf_\w+)\s*\(", text, flags=re.M)


def test_header_declares_every_binding_and_nothing_else():
    assert sorted(declared_symbols()) == sorted(native.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = native.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} missing from {native.library_path()}"


def test_library_exports_nothing_undeclared():
    """-fvisibility=hidden: only the kf_* entry points are dynamic symbols."""
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", native.library_path()],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    kf = {s for s in exported if s.startswith("kf_")}
    assert kf == set(native.EXPORTED_SYMBOLS)


def test_abi_version_and_version_string():
    lib = native.load()
    assert lib.kf_abi_version() == 1
    assert "sm_100a" in native.version()


def test_library_is_built_for_sm100a_only():
    from kernelo_b200.csrc import build

    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert not build.is_stale(), "library out of date with its sources"


@pytest.mark.parametrize(
    "cfg,ok",
    [
        (dict(kernel=1, block_m=128, block_n=256, block_k=64, stages=4), True),
        (dict(kernel=1, block_m=128, block_n=16, block_k=128, stages=6), True),
        (dict(kernel=1, block_m=128, block_n=256, block_k=64, stages=6), False),  # smem
        (dict(kernel=1, block_m=256, block_n=256, block_k=64, stages=6, cluster_m=2), True),  # SM pair
        (dict(kernel=1, block_m=256, block_n=256, block_k=64, stages=8, cluster_m=2), False),  # smem
        (dict(kernel=1, block_m=256, block_n=48, block_k=64, stages=2, cluster_m=2), False),  # halves
        (dict(kernel=1, block_m=64, block_n=64, block_k=64, stages=2), False),    # not built
        (dict(kernel=1, block_m=128, block_n=24, block_k=64, stages=2), False),   # N % 16
        (dict(kernel=1, block_m=128, block_n=64, block_k=32, stages=2), False),   # half atom
        (dict(kernel=1, block_m=128, block_n=64, block_k=64, stages=2, cluster_m=2), False),
    ],
)
def test_query_gemm_config_without_a_gpu(cfg, ok):
    status, smem, tmem, message = native.query_gemm_config(torch.bfloat16, native.GemmLaunch(**cfg))
    assert (status == native.KF_OK) == ok, message
    if ok:
        from kernelo_b200.kernels import gemm_common as gc

        assert smem == gc.tc_smem_bytes(cfg["block_n"], cfg["block_k"], cfg["stages"],
                                        cta_group=gc.cta_group(cfg["block_m"]))
        assert tmem == gc.tc_tmem_columns(cfg["block_n"])
    else:
        assert message


def test_status_codes_map_to_the_tuners_exception_classes():
    from kernelo_b200.tuning.tuner import STATUS_COMPILE_ERROR, STATUS_RUNTIME_ERROR, _classify

    for code, cls, status in (
        (native.KF_ERR_INVALID_CONFIG, native.OutOfResources, STATUS_COMPILE_ERROR),
        (native.KF_ERR_UNALIGNED, native.OutOfResources, STATUS_COMPILE_ERROR),
        (native.KF_ERR_TIMEOUT, native.KernelTimeoutError, STATUS_RUNTIME_ERROR),
        (native.KF_ERR_LAUNCH, native.KernelLaunchError, STATUS_RUNTIME_ERROR),
    ):
        with pytest.raises(cls) as info:
            native.check(code, "probe")
        assert _classify(info.value)[0] == status
    with pytest.raises(ValueError):
        native.check(native.KF_ERR_INVALID_ARGUMENT, "probe")


def test_ctypes_structs_match_the_header_layout():
    assert ctypes.sizeof(native.KfGemmConfig) == 16 * 4
    assert ctypes.sizeof(native.KfRowsConfig) == 8 * 4


def test_product_code_never_imports_the_oracle():
    root = Path(__file__).resolve().parent.parent / "kernelo_b200"
    for path in root.rglob("*.py"):
        text = path.read_text()
        assert "import oracle" not in text and "from oracle" not in text, path
