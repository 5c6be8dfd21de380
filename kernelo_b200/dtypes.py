"""Short dtype names and their codes in the C ABI.

The names (``fp16``, ``bf16``, ``fp32``) are what appear in cache keys,
database rows and command-line flags, so they must round-trip exactly
(mirrors ``kernelforge/dtypes.py:13-45``). The integer codes are the
``kf_dtype`` enum of ``include/kernelo_b200.h``.
"""

from __future__ import annotations

import torch

_BY_NAME: dict[str, torch.dtype] = {
    "fp16": torch.float16,
    "bf16": torch.bfloat16,
    "fp32": torch.float32,
}
_BY_DTYPE: dict[torch.dtype, str] = {dtype: name for name, dtype in _BY_NAME.items()}

#: ``kf_dtype`` codes of the native library.
NATIVE_CODES: dict[torch.dtype, int] = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}

SUPPORTED_DTYPES: tuple[str, ...] = tuple(_BY_NAME)


def parse_dtype(name: str | torch.dtype) -> torch.dtype:
    """``"fp16"`` / ``torch.float16`` -> ``torch.float16``; anything else raises."""
    if isinstance(name, torch.dtype):
        if name in _BY_DTYPE:
            return name
        raise ValueError(f"unsupported dtype {name!r}; expected one of {SUPPORTED_DTYPES}")
    dtype = _BY_NAME.get(str(name).lower())
    if dtype is None:
        raise ValueError(f"unsupported dtype {name!r}; expected one of {SUPPORTED_DTYPES}")
    return dtype


def dtype_name(dtype: torch.dtype) -> str:
    name = _BY_DTYPE.get(dtype)
    if name is None:
        raise ValueError(f"unsupported dtype {dtype!r}")
    return name


def itemsize(dtype: torch.dtype) -> int:
    return torch.tensor([], dtype=dtype).element_size()


def native_code(dtype: torch.dtype) -> int:
    code = NATIVE_CODES.get(dtype)
    if code is None:
        raise ValueError(f"dtype mismatch: {dtype} has no native kernel (fp16/bf16/fp32 only)")
    return code
