from __future__ import annotations

from kernelo_b200.runtime.env import DeviceCaps, Environment, capture_environment, device_caps, require_cuda

__all__ = ["DeviceCaps", "Environment", "capture_environment", "device_caps", "require_cuda"]
