"""ctypes binding of ``libkernelo_b200.so`` (the C ABI in ``include/kernelo_b200.h``).

This is the seam where the reference's wrappers launched Triton kernels
(``kernelforge/kernels/matmul.py:138-154`` and siblings). Here the wrappers
pass raw device pointers, element strides, a dtype code, a config struct and
torch's current stream to the native library; the library never allocates,
never synchronises and returns a status code that is mapped to the exception
classes the tuner classifies (``kernelforge/tuning/tuner.py:60-72``):

    KF_ERR_INVALID_ARGUMENT / WORKSPACE -> KernelArgumentError (a ValueError)
    KF_ERR_INVALID_CONFIG / UNALIGNED / UNSUPPORTED -> OutOfResources (compile_error)
    KF_ERR_TIMEOUT                      -> KernelTimeoutError
    KF_ERR_LAUNCH / NO_DEVICE           -> KernelLaunchError / NoDeviceError

There is no fallback: if the library cannot be loaded, every kernel call
raises. The library is built from ``kernelo_b200/csrc`` on first use when it
is missing or its recorded source hash no longer matches.
"""

from __future__ import annotations

import ctypes
import functools
import os
import threading
from dataclasses import dataclass

import torch

from kernelo_b200.dtypes import native_code

KF_OK = 0
KF_ERR_INVALID_ARGUMENT = 1
KF_ERR_INVALID_CONFIG = 2
KF_ERR_UNALIGNED = 3
KF_ERR_LAUNCH = 4
KF_ERR_TIMEOUT = 5
KF_ERR_UNSUPPORTED = 6
KF_ERR_WORKSPACE = 7
KF_ERR_NO_DEVICE = 8

KF_EPI_NONE = 0
KF_EPI_BIAS = 1
KF_EPI_BIAS_GELU_TANH = 2
KF_EPI_BIAS_GELU_ERF = 3

KF_GEMM_AUTO = 0
KF_GEMM_TCGEN05 = 1
KF_GEMM_SIMT = 2

#: Every symbol the header declares; tests check the library exports them all.
EXPORTED_SYMBOLS = (
    "kf_abi_version",
    "kf_version",
    "kf_last_error",
    "kf_sm_count",
    "kf_device_status",
    "kf_gemm",
    "kf_linear_bias_act",
    "kf_gemv",
    "kf_gemm_workspace_bytes",
    "kf_gemm_workspace_bytes_for",
    "kf_gemv_workspace_bytes",
    "kf_query_gemm_config",
    "kf_softmax_rows",
    "kf_rmsnorm_rows",
    "kf_selftest_bounded_wait",
    "kf_gemv_noalloc",
    "kf_linear_bias_act_allgather",
    "kf_linear_bias_act_allgather_sync",
    "kf_peer_barrier",
    "kf_peer_barrier_counted",
    "kf_ipc_handle",
    "kf_ipc_open",
    "kf_ipc_close",
)


class KernelLibraryError(RuntimeError):
    """Base class of failures reported by the native library."""

    def __init__(self, message: str, status: int) -> None:
        super().__init__(message)
        self.status = status


class KernelArgumentError(ValueError):
    def __init__(self, message: str, status: int = KF_ERR_INVALID_ARGUMENT) -> None:
        super().__init__(message)
        self.status = status


class OutOfResources(KernelLibraryError):
    """The config cannot run on this device for these operands.

    Named like Triton's exception so the tuner files it as ``compile_error``.
    """


class KernelLaunchError(KernelLibraryError):
    pass


class KernelTimeoutError(KernelLibraryError):
    pass


class NoDeviceError(KernelLibraryError):
    pass


class KfGemmConfig(ctypes.Structure):
    _fields_ = [
        ("kernel", ctypes.c_int32),
        ("block_m", ctypes.c_int32),
        ("block_n", ctypes.c_int32),
        ("block_k", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("group_m", ctypes.c_int32),
        ("stream_k", ctypes.c_int32),
        ("swap_ab", ctypes.c_int32),
        ("cluster_m", ctypes.c_int32),
        ("cluster_n", ctypes.c_int32),
        ("num_ctas", ctypes.c_int32),
        ("epi_store", ctypes.c_int32),
        ("overlap", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 3),
    ]


class KfRowsConfig(ctypes.Structure):
    _fields_ = [
        ("num_warps", ctypes.c_int32),
        ("rows_per_cta", ctypes.c_int32),
        ("cluster", ctypes.c_int32),
        ("kernel", ctypes.c_int32),
        ("row_groups", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 2),
    ]


class KfPeerSync(ctypes.Structure):
    _fields_ = [
        ("local_signals", ctypes.c_void_p),
        ("peer_signals", ctypes.POINTER(ctypes.c_void_p)),
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("epoch_counter", ctypes.c_void_p),
        ("arrivals", ctypes.c_void_p),
        ("timeout_us", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


_i32, _i64, _vp, _f32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_float
_GP = ctypes.POINTER(KfGemmConfig)
_RP = ctypes.POINTER(KfRowsConfig)

_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "kf_abi_version": (_i32, []),
    "kf_version": (ctypes.c_char_p, []),
    "kf_last_error": (ctypes.c_char_p, []),
    "kf_sm_count": (_i32, [_i32]),
    "kf_device_status": (_i32, [_i32, ctypes.POINTER(_i32)]),
    "kf_gemm": (_i32, [_i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64,
                       _GP, _vp, _i64, _vp]),
    "kf_linear_bias_act": (_i32, [_i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i64,
                                  _i64, _i64, _i64, _i32, _GP, _vp, _i64, _vp]),
    "kf_gemv": (_i32, [_i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64,
                       _GP, _vp, _i64, _vp]),
    "kf_gemm_workspace_bytes": (_i64, [_i32, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _GP]),
    "kf_gemm_workspace_bytes_for": (_i64, [_i32, _i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64,
                                           _i64, _i64, _GP]),
    "kf_gemv_workspace_bytes": (_i64, [_i32, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _GP]),
    "kf_query_gemm_config": (_i32, [_i32, _GP, ctypes.POINTER(_i64), ctypes.POINTER(_i32)]),
    "kf_softmax_rows": (_i32, [_i32, _vp, _i64, _vp, _i64, _i64, _i64, _RP, _vp]),
    "kf_rmsnorm_rows": (_i32, [_i32, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _f32, _RP, _vp]),
    "kf_selftest_bounded_wait": (_i32, [_i32, _vp]),
    "kf_gemv_noalloc": (_i32, [_i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64,
                               _vp]),
    "kf_linear_bias_act_allgather": (_i32, [_i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i64,
                                            _i64, _i64, _i64, _i32, ctypes.POINTER(_vp), _i32, _GP, _vp, _i64,
                                            _vp]),
    "kf_linear_bias_act_allgather_sync": (_i32, [_i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i64,
                                                 _i64, _i64, _i64, _i32, ctypes.POINTER(_vp), _i32,
                                                 ctypes.POINTER(KfPeerSync), _GP, _vp, _i64, _vp]),
    "kf_peer_barrier": (_i32, [_vp, ctypes.POINTER(_vp), _i32, _i32, ctypes.c_uint32, _i32, _vp]),
    "kf_peer_barrier_counted": (_i32, [_vp, ctypes.POINTER(_vp), _i32, _i32, _vp, _i32, _vp]),
    "kf_ipc_handle": (_i32, [_vp, _vp, ctypes.POINTER(_i64)]),
    "kf_ipc_open": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "kf_ipc_close": (_i32, [_vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> str:
    from kernelo_b200.csrc import build

    return str(build.LIB_PATH)


def load(*, build_if_needed: bool = True) -> ctypes.CDLL:
    """Load (building first if needed) the native library; cached per process."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        from kernelo_b200.csrc import build

        if build_if_needed and os.environ.get("KERNELO_B200_NO_BUILD") != "1" and build.is_stale():
            build.build()
        if not build.LIB_PATH.exists():
            raise RuntimeError(
                f"{build.LIB_PATH} is missing; run `python -m kernelo_b200.csrc.build` "
                "(there is no CPU fallback for the kernels)"
            )
        lib = ctypes.CDLL(str(build.LIB_PATH))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def version() -> str:
    return load().kf_version().decode()


def last_error() -> str:
    return (load().kf_last_error() or b"").decode(errors="replace")


def check(status: int, what: str) -> None:
    """Raise the exception class that corresponds to a native status code."""
    if status == KF_OK:
        return
    message = f"{what}: {last_error() or 'status ' + str(status)}"
    if status in (KF_ERR_INVALID_ARGUMENT, KF_ERR_WORKSPACE):
        raise KernelArgumentError(message, status)
    if status in (KF_ERR_INVALID_CONFIG, KF_ERR_UNALIGNED, KF_ERR_UNSUPPORTED):
        raise OutOfResources(message, status)
    if status == KF_ERR_TIMEOUT:
        raise KernelTimeoutError(message, status)
    if status == KF_ERR_NO_DEVICE:
        raise NoDeviceError(message, status)
    raise KernelLaunchError(message, status)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def current_stream_handle(device: torch.device) -> int:
    """The current CUDA stream of ``device`` as a raw handle (the cheap accessor
    torch's own extensions use, when this torch build has it)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ----------------------------------------------------------------------- configs
@dataclass(frozen=True)
class GemmLaunch:
    """Native GEMM parameters in KernelConfig vocabulary (0 = library default)."""

    kernel: int = 0
    block_m: int = 0
    block_n: int = 0
    block_k: int = 0
    stages: int = 0
    group_m: int = 0
    stream_k: int = 0
    swap_ab: int = 0
    cluster_m: int = 0
    cluster_n: int = 0
    num_ctas: int = 0
    epi_store: int = 0
    overlap: int = 0

    @classmethod
    def from_config(cls, config) -> GemmLaunch:
        if config is None:
            return _DEFAULT_LAUNCH
        get = config.get
        return cls(
            kernel=get("KERNEL", 0),
            block_m=get("BLOCK_M", 0),
            block_n=get("BLOCK_N", 0),
            block_k=get("BLOCK_K", 0),
            stages=get("num_stages", 0),
            group_m=get("GROUP_M", 0),
            stream_k=get("STREAM_K", 0),
            swap_ab=get("SWAP_AB", 0),
            cluster_m=get("CLUSTER_M", 0),
            cluster_n=get("CLUSTER_N", 0),
            num_ctas=get("NUM_CTAS", 0),
            epi_store=get("EPI_STORE", 0),
            overlap=get("OVERLAP", 0),
        )

    def struct(self) -> KfGemmConfig:
        """The C struct (built once per distinct launch and shared: the library
        only reads it)."""
        return _gemm_struct(self)

    def _build(self) -> KfGemmConfig:
        s = KfGemmConfig()
        for name in (
            "kernel",
            "block_m",
            "block_n",
            "block_k",
            "stages",
            "group_m",
            "stream_k",
            "swap_ab",
            "cluster_m",
            "cluster_n",
            "num_ctas",
            "epi_store",
            "overlap",
        ):
            setattr(s, name, getattr(self, name))
        return s


_DEFAULT_LAUNCH = GemmLaunch()


@functools.lru_cache(maxsize=1024)
def _gemm_struct(launch: GemmLaunch) -> KfGemmConfig:
    return launch._build()


_AUTO_ROWS = None


def rows_struct(config) -> KfRowsConfig:
    global _AUTO_ROWS
    if config is None:
        if _AUTO_ROWS is None:
            _AUTO_ROWS = KfRowsConfig()  # all zero: the library's own choice (only read)
        return _AUTO_ROWS
    s = KfRowsConfig()
    if config is not None:
        s.num_warps = config.get("num_warps", 0)
        s.rows_per_cta = config.get("ROWS_PER_PROGRAM", 0)
        s.cluster = config.get("CLUSTER", 0)
        s.kernel = config.get("ROW_KERNEL", 0)
        s.row_groups = config.get("ROW_GROUPS", 0)
        s.stages = config.get("num_stages", 0)
    return s


def query_gemm_config(dtype: torch.dtype, launch: GemmLaunch) -> tuple[int, int, int, str]:
    """(status, shared-memory bytes, TMEM columns, message) of a GEMM config; needs no GPU."""
    lib = load()
    smem = ctypes.c_int64(0)
    tmem = ctypes.c_int32(0)
    cfg = launch.struct()
    status = lib.kf_query_gemm_config(native_code(dtype), ctypes.byref(cfg), ctypes.byref(smem),
                                      ctypes.byref(tmem))
    message = last_error() if status != KF_OK else ""
    return status, smem.value, tmem.value, message


# ----------------------------------------------------------------------- workspace
class _WorkspacePool:
    """Zero-initialised workspaces, one per (device, stream), grown on demand.

    Stream-K kernels leave their counters at zero when they finish, so a
    workspace is reused without re-clearing. Calls on one stream are ordered,
    so sharing within a stream is safe; different streams get different buffers.
    """

    def __init__(self) -> None:
        self._buffers: dict[tuple[int, int], torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, stream: int, nbytes: int) -> torch.Tensor | None:
        if nbytes <= 0:
            return None
        key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
        with self._lock:
            buf = self._buffers.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 0 if buf is None else 2 * buf.numel())
                buf = torch.zeros(size, dtype=torch.uint8, device=device)
                self._buffers[key] = buf
            return buf

    def reset(self) -> None:
        """Drop every workspace (after a device error left counters unknown)."""
        with self._lock:
            self._buffers.clear()


workspaces = _WorkspacePool()
_workspace_sizes: dict[tuple, int] = {}


# ----------------------------------------------------------------------- calls
def gemm(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, *, bias: torch.Tensor | None = None,
         epilogue: int = KF_EPI_NONE, launch: GemmLaunch | None = None) -> None:
    """``c = epilogue(a @ b (+ bias))`` for 2-D a[M,K], b[K,N], c[M,N] (any strides)."""
    lib = load()
    launch = launch or GemmLaunch()
    cfg = launch.struct()
    dev = c.device
    stream = current_stream_handle(dev)
    code = native_code(a.dtype)
    m, k = a.shape
    n = b.shape[1]
    a_ptr, b_ptr, c_ptr = a.data_ptr(), b.data_ptr(), c.data_ptr()
    sa, sb, sc = a.stride(), b.stride(), c.stride()
    # The plan depends on sizes, strides, the pointers' 16-byte phase and the
    # config only: sized once per distinct call shape.
    key = (dev.index, code, m, n, k, sa, sb, sc, a_ptr & 15, b_ptr & 15, c_ptr & 15, launch)
    ws_bytes = _workspace_sizes.get(key)
    if ws_bytes is None:
        ws_bytes = lib.kf_gemm_workspace_bytes_for(dev.index or 0, code, a_ptr, sa[0], sa[1], b_ptr, sb[0], sb[1],
                                                   c_ptr, sc[0], sc[1], m, n, k, ctypes.byref(cfg))
        if ws_bytes < 0:
            check(int(-ws_bytes), "kf_gemm_workspace_bytes_for")
        if len(_workspace_sizes) > 4096:
            _workspace_sizes.clear()
        _workspace_sizes[key] = ws_bytes
    ws = workspaces.get(dev, stream, ws_bytes)
    ws_ptr = _ptr(ws)
    if epilogue == KF_EPI_NONE:
        status = lib.kf_gemm(code, a_ptr, sa[0], sa[1], b_ptr, sb[0], sb[1], c_ptr, sc[0], sc[1], m, n, k,
                             ctypes.byref(cfg), ws_ptr, max(ws_bytes, 0), stream)
        if status:
            check(status, "kf_gemm")
    else:
        status = lib.kf_linear_bias_act(code, a_ptr, sa[0], sa[1], b_ptr, sb[0], sb[1], _ptr(bias), c_ptr,
                                        sc[0], sc[1], m, n, k, epilogue, ctypes.byref(cfg), ws_ptr,
                                        max(ws_bytes, 0), stream)
        if status:
            check(status, "kf_linear_bias_act")


def peer_sync_struct(local_signals: int, peer_signals: list[int], rank: int, world: int, epoch_counter: int,
                     arrivals: int, timeout_us: int = 2_000_000) -> KfPeerSync:
    """The kf_peer_sync struct of one rank (keeps its peer-pointer array alive)."""
    arr = (_vp * max(1, len(peer_signals)))(*[ctypes.c_void_p(int(p)) for p in peer_signals])
    s = KfPeerSync(local_signals, ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)), rank, world, epoch_counter,
                   arrivals, timeout_us, 0)
    s._keep = arr
    return s


def linear_bias_act_allgather(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, peers: list[int], *,
                              bias: torch.Tensor | None, epilogue: int, launch: GemmLaunch | None = None,
                              sync: KfPeerSync | None = None) -> None:
    """``c = epilogue(a @ b + bias)``, every output tile also stored at the same
    offsets from each address in ``peers`` (peer-mapped copies of c's buffer).
    ``bias`` may be None with ``KF_EPI_NONE`` (the plain sharded GEMM/GEMV).
    With ``sync`` the bounded peer barrier that completes the all-gather
    follows in the same call (inside the kernel on the tile GEMV path)."""
    lib = load()
    launch = launch or GemmLaunch()
    cfg = launch.struct()
    dev = c.device
    stream = current_stream_handle(dev)
    code = native_code(a.dtype)
    m, k = a.shape
    n = b.shape[1]
    ws_bytes = lib.kf_gemm_workspace_bytes(dev.index or 0, code, a.stride(0), a.stride(1),
                                           b.stride(0), b.stride(1), m, n, k, ctypes.byref(cfg))
    if ws_bytes < 0:
        check(int(-ws_bytes), "kf_gemm_workspace_bytes")
    ws = workspaces.get(dev, stream, ws_bytes)
    arr = (_vp * max(1, len(peers)))(*[ctypes.c_void_p(int(p)) for p in peers])
    if sync is None:
        status = lib.kf_linear_bias_act_allgather(code, a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(),
                                                  b.stride(0), b.stride(1), _ptr(bias), c.data_ptr(), c.stride(0),
                                                  c.stride(1), m, n, k, epilogue, arr, len(peers),
                                                  ctypes.byref(cfg), _ptr(ws), max(ws_bytes, 0), stream)
        check(status, "kf_linear_bias_act_allgather")
        return
    status = lib.kf_linear_bias_act_allgather_sync(code, a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(),
                                                   b.stride(0), b.stride(1), _ptr(bias), c.data_ptr(), c.stride(0),
                                                   c.stride(1), m, n, k, epilogue, arr, len(peers),
                                                   ctypes.byref(sync), ctypes.byref(cfg), _ptr(ws),
                                                   max(ws_bytes, 0), stream)
    check(status, "kf_linear_bias_act_allgather_sync")


def peer_barrier(local_signals: int, peer_signals: list[int], rank: int, world: int, epoch: int,
                 *, timeout_us: int = 2_000_000, device: torch.device | None = None) -> None:
    """Enqueue the bounded cross-GPU barrier (kf_peer_barrier) on the current stream."""
    lib = load()
    dev = device or torch.device("cuda", torch.cuda.current_device())
    arr = (_vp * max(1, len(peer_signals)))(*[ctypes.c_void_p(int(p)) for p in peer_signals])
    status = lib.kf_peer_barrier(ctypes.c_void_p(int(local_signals)), arr, rank, world, epoch, timeout_us,
                                 current_stream_handle(dev))
    check(status, "kf_peer_barrier")


def peer_barrier_counted(local_signals: int, peer_signals: list[int], rank: int, world: int, epoch_counter: int,
                         *, timeout_us: int = 2_000_000, device: torch.device | None = None) -> None:
    """Enqueue the bounded cross-GPU barrier whose epoch is a device counter
    (kf_peer_barrier_counted): capturable in a CUDA graph, every replay
    advances the epoch."""
    lib = load()
    dev = device or torch.device("cuda", torch.cuda.current_device())
    arr = (_vp * max(1, len(peer_signals)))(*[ctypes.c_void_p(int(p)) for p in peer_signals])
    status = lib.kf_peer_barrier_counted(ctypes.c_void_p(int(local_signals)), arr, rank, world,
                                         ctypes.c_void_p(int(epoch_counter)), timeout_us,
                                         current_stream_handle(dev))
    check(status, "kf_peer_barrier_counted")


IPC_HANDLE_BYTES = 64


def ipc_handle(t: torch.Tensor) -> tuple[bytes, int]:
    """(CUDA IPC handle of the allocation holding t, t's byte offset in it)."""
    lib = load()
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    off = ctypes.c_int64(0)
    check(lib.kf_ipc_handle(ctypes.c_void_p(t.data_ptr()), buf, ctypes.byref(off)), "kf_ipc_handle")
    return buf.raw, off.value


def ipc_open(handle: bytes) -> int:
    """Map another process's allocation on the current device; returns its base address."""
    lib = load()
    base = ctypes.c_void_p(0)
    check(lib.kf_ipc_open(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES), ctypes.byref(base)),
          "kf_ipc_open")
    return int(base.value)


def ipc_close(base: int) -> None:
    check(load().kf_ipc_close(ctypes.c_void_p(base)), "kf_ipc_close")


def gemv(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, *, w_layout: str = "nk",
         launch: GemmLaunch | None = None) -> None:
    """Decode-shape ``y[M,N] = x[M,K] . W^T`` with W stored [N,K] (``"nk"``) or [K,N] (``"kn"``)."""
    lib = load()
    launch = launch or _DEFAULT_LAUNCH
    cfg = launch.struct()
    dev = y.device
    stream = current_stream_handle(dev)
    code = native_code(x.dtype)
    m, k = x.shape
    if w_layout == "nk":
        n = w.shape[0]
        sw_n, sw_k = w.stride(0), w.stride(1)
    elif w_layout == "kn":
        n = w.shape[1]
        sw_k, sw_n = w.stride(0), w.stride(1)
    else:
        raise ValueError(f"w_layout must be 'nk' or 'kn', got {w_layout!r}")
    sx = x.stride()
    key = ("gemv", dev.index, code, m, n, k, sx, sw_n, sw_k, launch)
    ws_bytes = _workspace_sizes.get(key)
    if ws_bytes is None:
        ws_bytes = lib.kf_gemv_workspace_bytes(dev.index or 0, code, sx[0], sx[1], sw_n, sw_k, m, n, k,
                                               ctypes.byref(cfg))
        if ws_bytes < 0:
            check(int(-ws_bytes), "kf_gemv_workspace_bytes")
        if len(_workspace_sizes) > 4096:
            _workspace_sizes.clear()
        _workspace_sizes[key] = ws_bytes
    ws = workspaces.get(dev, stream, ws_bytes)
    status = lib.kf_gemv(code, x.data_ptr(), sx[0], sx[1], w.data_ptr(), sw_n, sw_k,
                         y.data_ptr(), y.stride(0), y.stride(1), m, n, k, ctypes.byref(cfg),
                         _ptr(ws), max(ws_bytes, 0), stream)
    if status:
        check(status, "kf_gemv")


def softmax_rows(x: torch.Tensor, y: torch.Tensor, config=None) -> None:
    lib = load()
    cfg = rows_struct(config)
    rows, cols = x.shape
    status = lib.kf_softmax_rows(native_code(x.dtype), x.data_ptr(), x.stride(0), y.data_ptr(),
                                 y.stride(0), rows, cols, ctypes.byref(cfg),
                                 current_stream_handle(y.device))
    if status:
        check(status, "kf_softmax_rows")


def rmsnorm_rows(x: torch.Tensor, gamma: torch.Tensor, y: torch.Tensor, eps: float,
                 config=None) -> None:
    lib = load()
    cfg = rows_struct(config)
    rows, cols = x.shape
    status = lib.kf_rmsnorm_rows(native_code(x.dtype), x.data_ptr(), x.stride(0), gamma.data_ptr(),
                                 y.data_ptr(), y.stride(0), rows, cols, float(eps),
                                 ctypes.byref(cfg), current_stream_handle(y.device))
    if status:
        check(status, "kf_rmsnorm_rows")


def device_status(device: int | None = None) -> int:
    """Read and clear the device status word (synchronises the device)."""
    lib = load()
    idx = torch.cuda.current_device() if device is None else int(device)
    out = ctypes.c_int32(0)
    check(lib.kf_device_status(idx, ctypes.byref(out)), "kf_device_status")
    return out.value


def raise_on_device_status(device: int | None = None) -> None:
    """Turn a recorded bounded-wait timeout into :class:`KernelTimeoutError`."""
    value = device_status(device)
    if value:
        workspaces.reset()
        code, site = value & 0xFF, value >> 8
        raise KernelTimeoutError(
            f"a device-side wait gave up (status {code}, wait site {site})", code
        )


def selftest_bounded_wait(timeout_us: int = 20000) -> None:
    lib = load()
    check(lib.kf_selftest_bounded_wait(int(timeout_us), current_stream_handle(torch.device(
        "cuda", torch.cuda.current_device()))), "kf_selftest_bounded_wait")


def sm_count(device: int | None = None) -> int:
    idx = torch.cuda.current_device() if device is None else int(device)
    value = load().kf_sm_count(idx)
    if value < 0:
        check(-value, "kf_sm_count")
    return value
