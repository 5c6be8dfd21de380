"""Device capabilities and run provenance (``kernelforge/runtime/env.py:21-222``).

:class:`DeviceCaps` is the value object the search-space filters read, so they
can be unit-tested against a GPU that is not attached. Beyond the reference's
fields it carries the Blackwell resources the sm_100a filters need: TMEM
columns per SM and the portable thread-block-cluster size. Without a device,
:func:`device_caps` returns B200 values labelled ``measured=False``.
"""

from __future__ import annotations

import platform
import shutil
import socket
import subprocess
import sys
from dataclasses import asdict, dataclass
from datetime import datetime, timezone

import torch


@dataclass(frozen=True)
class DeviceCaps:
    name: str
    compute_capability: str
    total_memory_bytes: int
    sm_count: int
    max_shared_memory_per_block: int
    shared_memory_per_sm: int
    registers_per_sm: int
    max_threads_per_sm: int
    warp_size: int
    l2_cache_bytes: int
    #: False when the values were assumed rather than read from a device.
    measured: bool = True
    #: Tensor-memory columns per SM (128 lanes x 512 columns x 32 bit on sm_100).
    tmem_columns_per_sm: int = 512
    #: Largest portable thread-block cluster.
    max_cluster_size: int = 8

    @property
    def arch(self) -> str:
        return "sm" + self.compute_capability.replace(".", "")

    @property
    def key(self) -> str:
        """Board name plus architecture: two boards of one arch do not share tunings."""
        cleaned = "".join(ch if ch.isalnum() else "_" for ch in self.name).strip("_")
        while "__" in cleaned:
            cleaned = cleaned.replace("__", "_")
        return f"{cleaned}_{self.arch}"

    @property
    def is_blackwell_datacenter(self) -> bool:
        return self.compute_capability.startswith("10.")


#: B200 values for runs without an attached device (filter tests, docs, CI).
B200_CAPS = DeviceCaps(
    name="NVIDIA B200 (assumed)",
    compute_capability="10.0",
    total_memory_bytes=183_359 * 1024**2,
    sm_count=148,
    max_shared_memory_per_block=232_448,
    shared_memory_per_sm=233_472,
    registers_per_sm=65_536,
    max_threads_per_sm=2048,
    warp_size=32,
    l2_cache_bytes=126 * 1024 * 1024,
    measured=False,
)


def device_caps(device: torch.device | str | int | None = None) -> DeviceCaps:
    """Capabilities of an attached CUDA device, or the B200 stand-in without one."""
    if not torch.cuda.is_available():
        return B200_CAPS
    if device is None:
        index = torch.cuda.current_device()
    elif isinstance(device, int):
        index = device
    else:
        dev = torch.device(device)
        index = dev.index if dev.index is not None else torch.cuda.current_device()
    props = torch.cuda.get_device_properties(index)
    return DeviceCaps(
        name=props.name,
        compute_capability=f"{props.major}.{props.minor}",
        total_memory_bytes=int(props.total_memory),
        sm_count=int(props.multi_processor_count),
        max_shared_memory_per_block=int(
            getattr(props, "shared_memory_per_block_optin", getattr(props, "shared_memory_per_block", 49152))
        ),
        shared_memory_per_sm=int(getattr(props, "shared_memory_per_multiprocessor", 65536)),
        registers_per_sm=int(getattr(props, "regs_per_multiprocessor", 65536)),
        max_threads_per_sm=int(getattr(props, "max_threads_per_multi_processor", 2048)),
        warp_size=int(getattr(props, "warp_size", 32)),
        l2_cache_bytes=int(getattr(props, "L2_cache_size", 0)) or 4 * 1024 * 1024,
    )


def device_key(device: torch.device | str | int | None = None) -> str:
    """Cache key of the attached device; ``"cpu"`` when there is none."""
    if not torch.cuda.is_available():
        return "cpu"
    return device_caps(device).key


def _driver_version() -> str | None:
    try:
        raw = torch._C._cuda_getDriverVersion()  # type: ignore[attr-defined]
    except Exception:
        raw = None
    if isinstance(raw, int) and raw > 0:
        return f"{raw // 1000}.{(raw % 1000) // 10}"
    if shutil.which("nvidia-smi") is None:
        return None
    try:
        out = subprocess.run(
            ["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader"],
            capture_output=True,
            text=True,
            timeout=10,
            check=True,
        )
    except (subprocess.SubprocessError, OSError):
        return None
    lines = out.stdout.strip().splitlines()
    return lines[0].strip() if lines else None


def _native_version() -> str | None:
    try:
        from kernelo_b200.runtime import native

        return native.version()
    except Exception:
        return None


@dataclass(frozen=True)
class Environment:
    timestamp: str
    hostname: str
    platform: str
    python_version: str
    torch_version: str
    triton_version: str | None  # kept for schema compatibility; holds the native library version
    cuda_version: str | None
    driver_version: str | None
    gpu_name: str | None
    gpu_arch: str | None
    gpu_memory_bytes: int | None
    sm_count: int | None
    device_key: str

    def as_dict(self) -> dict[str, object]:
        return asdict(self)

    def render(self) -> str:
        rows = [
            ("GPU", self.gpu_name or "none (CPU only)"),
            ("Compute capability", self.gpu_arch or "-"),
            ("SM count", str(self.sm_count) if self.sm_count else "-"),
            ("VRAM", f"{self.gpu_memory_bytes / 1024**3:.1f} GiB" if self.gpu_memory_bytes else "-"),
            ("CUDA", self.cuda_version or "-"),
            ("Driver", self.driver_version or "-"),
            ("PyTorch", self.torch_version),
            ("Native library", self.triton_version or "not loaded"),
            ("Python", self.python_version),
            ("Platform", self.platform),
            ("Host", self.hostname),
            ("Timestamp", self.timestamp),
        ]
        width = max(len(k) for k, _ in rows)
        return "\n".join(f"{k:<{width}}  {v}" for k, v in rows)


def capture_environment(device: torch.device | str | int | None = None) -> Environment:
    has_cuda = torch.cuda.is_available()
    caps = device_caps(device) if has_cuda else None
    return Environment(
        timestamp=datetime.now(timezone.utc).isoformat(timespec="seconds"),
        hostname=socket.gethostname(),
        platform=platform.platform(),
        python_version=sys.version.split()[0],
        torch_version=torch.__version__,
        triton_version=_native_version() if has_cuda else None,
        cuda_version=torch.version.cuda if has_cuda else None,
        driver_version=_driver_version() if has_cuda else None,
        gpu_name=caps.name if caps else None,
        gpu_arch=caps.compute_capability if caps else None,
        gpu_memory_bytes=caps.total_memory_bytes if caps else None,
        sm_count=caps.sm_count if caps else None,
        device_key=device_key(device),
    )


def require_cuda() -> torch.device:
    """Fail loudly rather than time CPU work as if it were the GPU path."""
    if not torch.cuda.is_available():
        raise RuntimeError(
            "KernelForge-B200 kernels require a CUDA device. torch.cuda.is_available() returned False."
        )
    return torch.device("cuda", torch.cuda.current_device())
