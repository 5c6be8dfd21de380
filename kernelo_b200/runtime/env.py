"""Device capabilities and run provenance.

Two value objects with the reference's field names (``kernelforge/runtime/env.py:21-222``),
since the search-space filters, the SQLite ``runs`` table and the cache keys
are defined by them:

* :class:`DeviceCaps` -- what the candidate filters reason about. Filters take
  it as an argument, so they can be tested against a GPU that is not attached.
  Besides the reference's fields it carries the Blackwell resources the
  sm_100a filters need: TMEM columns per SM and the portable cluster size.
  Without a device, :func:`device_caps` answers with B200 values marked
  ``measured=False``.
* :class:`Environment` -- the provenance stamped on every tuning run and
  benchmark row.

Device properties never change while a process runs, so they are read once
per device index and memoised.
"""

from __future__ import annotations

import functools
import platform
import re
import socket
import sys
from dataclasses import asdict, dataclass, fields
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
        board = re.sub(r"[^0-9A-Za-z]+", "_", self.name).strip("_")
        return f"{board}_{self.arch}"

    @property
    def is_blackwell_datacenter(self) -> bool:
        return self.compute_capability.split(".")[0] == "10"

    @classmethod
    def from_properties(cls, props) -> DeviceCaps:
        """From ``torch.cuda.get_device_properties``; the opt-in shared-memory
        limit is the one a kernel can request with dynamic shared memory."""
        def prop(name: str, default: int) -> int:
            return int(getattr(props, name, default) or default)

        return cls(
            name=props.name,
            compute_capability=f"{props.major}.{props.minor}",
            total_memory_bytes=int(props.total_memory),
            sm_count=int(props.multi_processor_count),
            max_shared_memory_per_block=prop("shared_memory_per_block_optin",
                                             prop("shared_memory_per_block", 49152)),
            shared_memory_per_sm=prop("shared_memory_per_multiprocessor", 65536),
            registers_per_sm=prop("regs_per_multiprocessor", 65536),
            max_threads_per_sm=prop("max_threads_per_multi_processor", 2048),
            warp_size=prop("warp_size", 32),
            l2_cache_bytes=prop("L2_cache_size", 4 * 1024 * 1024),
            # TMEM and clusters exist from sm_90 (clusters) and sm_100 (TMEM) on
            tmem_columns_per_sm=512 if props.major >= 10 else 0,
            max_cluster_size=8 if props.major >= 9 else 1,
        )


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


def _device_index(device: torch.device | str | int | None) -> int:
    if isinstance(device, int):
        return device
    if device is None:
        return torch.cuda.current_device()
    dev = torch.device(device)
    return dev.index if dev.index is not None else torch.cuda.current_device()


@functools.lru_cache(maxsize=None)
def _caps_of(index: int) -> DeviceCaps:
    return DeviceCaps.from_properties(torch.cuda.get_device_properties(index))


def device_caps(device: torch.device | str | int | None = None) -> DeviceCaps:
    """Capabilities of an attached CUDA device, or the B200 stand-in without one."""
    if not torch.cuda.is_available():
        return B200_CAPS
    return _caps_of(_device_index(device))


def device_key(device: torch.device | str | int | None = None) -> str:
    """Cache key of the attached device; ``"cpu"`` when there is none."""
    return device_caps(device).key if torch.cuda.is_available() else "cpu"


def _driver_version() -> str | None:
    """The NVIDIA driver's version: NVML's string when NVML is importable,
    else torch's integer (1000 * major + 10 * minor) formatted."""
    try:
        import pynvml

        pynvml.nvmlInit()
        try:
            version = pynvml.nvmlSystemGetDriverVersion()
        finally:
            pynvml.nvmlShutdown()
        return version.decode() if isinstance(version, bytes) else str(version)
    except Exception:  # noqa: BLE001 - NVML missing or unusable: fall back
        pass
    try:
        raw = int(torch._C._cuda_getDriverVersion())  # type: ignore[attr-defined]
    except Exception:  # noqa: BLE001
        return None
    return f"{raw // 1000}.{raw % 1000 // 10}" if raw > 0 else None


def _native_version() -> str | None:
    try:
        from kernelo_b200.runtime import native

        return native.version()
    except Exception:  # noqa: BLE001 - the library is not loadable here
        return None


@dataclass(frozen=True)
class Environment:
    timestamp: str
    hostname: str
    platform: str
    python_version: str
    torch_version: str
    triton_version: str | None  # the schema's column; holds the native library's version here
    cuda_version: str | None
    driver_version: str | None
    gpu_name: str | None
    gpu_arch: str | None
    gpu_memory_bytes: int | None
    sm_count: int | None
    device_key: str

    #: How :meth:`render` labels and formats each field, in display order.
    _DISPLAY = (
        ("gpu_name", "GPU", lambda v: v or "none (CPU only)"),
        ("gpu_arch", "Compute capability", lambda v: v or "-"),
        ("sm_count", "SM count", lambda v: str(v) if v else "-"),
        ("gpu_memory_bytes", "VRAM", lambda v: f"{v / 2**30:.1f} GiB" if v else "-"),
        ("cuda_version", "CUDA", lambda v: v or "-"),
        ("driver_version", "Driver", lambda v: v or "-"),
        ("torch_version", "PyTorch", str),
        ("triton_version", "Native library", lambda v: v or "not loaded"),
        ("python_version", "Python", str),
        ("platform", "Platform", str),
        ("hostname", "Host", str),
        ("timestamp", "Timestamp", str),
    )

    def as_dict(self) -> dict[str, object]:
        return asdict(self)

    def render(self) -> str:
        pairs = [(label, fmt(getattr(self, name))) for name, label, fmt in self._DISPLAY]
        pad = max(len(label) for label, _ in pairs)
        return "\n".join(f"{label.ljust(pad)}  {value}" for label, value in pairs)


def capture_environment(device: torch.device | str | int | None = None) -> Environment:
    facts: dict[str, object] = {
        "timestamp": datetime.now(timezone.utc).isoformat(timespec="seconds"),
        "hostname": socket.gethostname(),
        "platform": platform.platform(),
        "python_version": platform.python_version() or sys.version.split()[0],
        "torch_version": torch.__version__,
        "device_key": device_key(device),
    }
    gpu_fields = ("triton_version", "cuda_version", "driver_version", "gpu_name", "gpu_arch", "gpu_memory_bytes",
                  "sm_count")
    facts.update(dict.fromkeys(gpu_fields))
    if torch.cuda.is_available():
        caps = device_caps(device)
        facts.update(triton_version=_native_version(), cuda_version=torch.version.cuda,
                     driver_version=_driver_version(), gpu_name=caps.name, gpu_arch=caps.compute_capability,
                     gpu_memory_bytes=caps.total_memory_bytes, sm_count=caps.sm_count)
    assert set(facts) == {f.name for f in fields(Environment)}
    return Environment(**facts)


def require_cuda() -> torch.device:
    """Fail loudly rather than time CPU work as if it were the GPU path."""
    if not torch.cuda.is_available():
        raise RuntimeError(
            "KernelForge-B200 kernels require a CUDA device. torch.cuda.is_available() returned False."
        )
    return torch.device("cuda", torch.cuda.current_device())
