"""Headline benchmark: fused linear + bias + exact-erf GELU, 4096 x 11008 x 4096 bf16.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

One step = ``Y = gelu(X @ W^T + b)`` over the whole workload (X [4096,4096],
W [11008,4096] stored nn.Linear-style, b [11008]; X ~ N(0,1), W ~ N(0,1/4096),
b ~ N(0,0.1); synthetic, seeded). With N GPUs (torchrun, one process per GPU)
the weight is column-sharded by N and the GEMM's epilogue stores every output
tile into all ranks' copies of Y over NVLink, followed by a bounded peer
barrier (strong scaling: the total work is fixed).

Printed (rank 0, one JSON line): whole-job TFLOP/s over K timed steps (device
time, CUDA events, max over ranks, barrier + synchronize on both sides), the
end-to-end figure through the public API with host<->device copies, the
dominant kernel's roofline against the measured peak, SM clocks sampled during
the timed region, the reference's CPU path timed on this host's cores, and the
memory-bound rows (RMSNorm, softmax, decode GEMV) as secondary lines.

``--impl reference`` times the reference's own CPU implementation of the path
(the oracle's restatement of ``linear_gelu_reference``, torch on host cores,
fp32) on a bounded sample of the same workload, and prints the same line with
``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch
import torch.distributed as dist

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

M, N, K = 4096, 11008, 4096
FLOP = 2 * M * N * K
METRIC = "fused_linear_gelu TFLOP/s (4096x11008x4096 bf16, erf GELU)"
UNIT = "TFLOP/s"
WORKLOAD = "fused_linear bias+erf-GELU M=4096 N=11008 K=4096 bf16, W [N,K]"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def measure_peer_copy_gbs(device: torch.device, world: int, rank: int, nbytes: int = 256 << 20,
                          reps: int = 5) -> dict:
    """One-way NVLink copy rate measured in this run: every rank copies
    ``nbytes`` from its own HBM into the next rank's buffer (a ring, all ranks
    at once, one cudaMemcpyAsync through the CUDA IPC mapping), best of
    ``reps``; the slowest rank's time counts. This is the denominator of the
    all-gathering kernel's NVLink roofline."""
    from cuda.bindings import runtime as cudart

    from kernelo_b200.runtime import native

    src = torch.ones(nbytes, dtype=torch.uint8, device=device)
    dst = torch.zeros(nbytes, dtype=torch.uint8, device=device)
    torch.cuda.synchronize(device)
    everyone: list = [None] * world
    dist.all_gather_object(everyone, native.ipc_handle(dst))
    peer = (rank + 1) % world
    base = native.ipc_open(everyone[peer][0])
    peer_ptr = base + everyone[peer][1]
    stream = torch.cuda.current_stream(device)
    best = float("inf")
    try:
        for _ in range(reps + 1):
            dist.barrier()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            (err,) = cudart.cudaMemcpyAsync(peer_ptr, src.data_ptr(), nbytes,
                                            cudart.cudaMemcpyKind.cudaMemcpyDeviceToDevice, stream.cuda_stream)
            end.record(stream)
            torch.cuda.synchronize(device)
            if err != cudart.cudaError_t.cudaSuccess:
                raise RuntimeError(f"peer copy failed: {err}")
            best = min(best, start.elapsed_time(end))
        ms = max_over_ranks(best, world)
    finally:
        torch.cuda.synchronize(device)
        dist.barrier()
        native.ipc_close(base)
    return {"gbs": round(nbytes / (ms * 1e-3) / 1e9, 1), "bytes": nbytes, "ms": round(ms, 4),
            "how": "ring of one-way cudaMemcpyAsync peer copies, all ranks at once, best of "
                   f"{reps}, slowest rank"}


def allgather_roofline(flop_rank: float, link_bytes: int, kernel_ms: float, tensor_peak: float,
                       tensor_peak_kind: str, link_gbs_peak: float) -> dict:
    """Roofline of the GEMM + all-gather kernel: the target time is the slower
    of the shard's FLOPs at the GEMM peak and the bytes each rank must send over
    NVLink (its shard to every peer) at the peer-copy rate measured in this
    run; ``frac`` is target / measured, in the units of the binding resource."""
    t_tensor = flop_rank / (tensor_peak * 1e12)
    t_link = link_bytes / (link_gbs_peak * 1e9)
    tflops = flop_rank / (kernel_ms * 1e-3) / 1e12
    link_gbs = link_bytes / (kernel_ms * 1e-3) / 1e9
    target_ms = max(t_tensor, t_link) * 1e3
    nvlink_bound = t_link > t_tensor
    return {"bound": "nvlink" if nvlink_bound else "tensor",
            "achieved": round(link_gbs if nvlink_bound else tflops, 1),
            "peak": link_gbs_peak if nvlink_bound else tensor_peak,
            "unit": "GB/s" if nvlink_bound else "TFLOP/s",
            "frac": round(target_ms / kernel_ms, 4), "target_ms": round(target_ms, 4),
            "tensor_tflops": round(tflops, 1), "tensor_peak": tensor_peak, "tensor_peak_kind": tensor_peak_kind,
            "nvlink_gbs": round(link_gbs, 1), "nvlink_bytes_per_rank": link_bytes,
            "nvlink_peak": link_gbs_peak, "nvlink_peak_kind": "peer copy per direction measured in this run",
            "traffic": None, "kernel": "tc_gemm_kernel<bf16,erf,all-gather>", "kernel_ms": round(kernel_ms, 4)}


def peaks() -> tuple[dict, str]:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def profile_traffic(kernel: str) -> float | None:
    """Per-launch DRAM bytes recorded from an ncu capture (profiles/<kernel>.txt)."""
    path = REPO / "profiles" / f"{kernel}.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def tensor_peak_for_run(pk: dict, pk_kind: str, clocks: dict, region_s: float) -> tuple[float, str]:
    """The GEMM peak that applies to this timed region.

    The burst figure (cuBLAS timed alone, at full clocks) unless the region
    ran for seconds under the power cap: only then does the sustained figure
    (cuBLAS back to back for seconds, ``sw_power_cap`` active) describe the
    conditions the kernel ran under."""
    capped = "sw_power_cap" in (clocks.get("reasons") or [])
    sustained = pk.get("bf16_tflops_sustained")
    if capped and region_s >= 1.0 and sustained:
        return sustained, f"{pk_kind} sustained bf16 (timed region {region_s:.2f} s under sw_power_cap)"
    why = "no sw_power_cap sample" if not capped else f"timed region of {region_s * 1e3:.1f} ms"
    return pk["bf16_tflops"], f"{pk_kind} burst bf16 ({why})"


def pcie_rates(device: torch.device, nbytes: int = 64 << 20, reps: int = 5) -> dict:
    """Pinned host<->device copy rates measured in this run (best of ``reps``
    single copies each way), to state the bound of the end-to-end figure."""
    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    out = {}
    for name, dst, src in (("h2d_gbs", dev, host), ("d2h_gbs", host, dev)):
        best = float("inf")
        for _ in range(reps + 1):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            dst.copy_(src, non_blocking=True)
            end.record(stream)
            end.synchronize()
            best = min(best, start.elapsed_time(end))
        out[name] = round(nbytes / (best * 1e-3) / 1e9, 1)
    return out


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock, power and clock-event reasons sampled every 2 ms through NVML
    (read-only queries) on a background thread during the timed region;
    nvidia-smi polling when NVML is not importable. The first sample is taken
    as the region starts and one more as it ends, so a region of a few
    milliseconds still has its clocks on record."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, period_s: float = 0.002) -> None:
        self.device_index = device_index
        self.period_s = period_s
        self.rows: list[tuple[float, float, float, int]] = []  # (sm MHz, max MHz, watts, reason bits)
        self._stop = threading.Event()
        self._thread = None
        self._proc = None
        self._smi_out = ""

    def _nvml_handle(self):
        import pynvml

        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.device_index).uuid)
        return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)

    def _sample(self, nvml, handle, max_mhz: float) -> None:
        try:
            mhz = float(nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM))
            watts = nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
            bits = int(nvml.nvmlDeviceGetCurrentClocksEventReasons(handle))
            self.rows.append((mhz, max_mhz, watts, bits))
        except Exception:  # noqa: BLE001 - a failed read is a missing sample
            pass

    def _loop(self, nvml, handle) -> None:
        max_mhz = float(nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM))
        while True:
            self._sample(nvml, handle, max_mhz)
            if self._stop.wait(self.period_s):
                self._sample(nvml, handle, max_mhz)  # as the region ends
                return

    def __enter__(self):
        try:
            nvml, handle = self._nvml_handle()
            self._thread = threading.Thread(target=self._loop, args=(nvml, handle), daemon=True)
            self._thread.start()
        except Exception:  # noqa: BLE001 - NVML unavailable: poll nvidia-smi instead
            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                     "-i", str(self.device_index)],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except OSError:
                self._proc = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._smi_out, _ = self._proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
            for line in (self._smi_out or "").splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    flags = [f.lower() == "active" for f in parts[5:9]]
                    bits = sum(b for (_, b), on in zip(self.REASONS[:4], flags) if on)
                    self.rows.append((float(parts[1]), float(parts[2]), float(parts[3]), bits))
                except ValueError:
                    continue

    def summary(self) -> dict:
        rows = list(self.rows)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [r for r in rows if r[2] > 200.0] or rows
        reasons = sorted({name for r in loaded for name, bit in self.REASONS if r[3] & bit})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": rows[0][1], "reasons": reasons,
                "samples": len(loaded), "power_w_max": max(r[2] for r in rows),
                "source": "nvml" if self._thread is not None else "nvidia-smi"}


# ------------------------------------------------------------------ helpers
def dist_setup(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if gpus != world:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        # NCCL carries the timing reductions, the gate and, where it measures
        # faster than the fused gather at this N, the all-gather; without NVLS
        # no buffer is ever bound to an NVLink multicast object, so a rank that
        # fails cannot take its peers' GPUs down with it.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world: int) -> None:
    if world > 1:
        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_inputs(device, rank: int, world: int):
    """X replicated on every rank; each rank builds only its W/b slice."""
    from kernelo_b200.distributed import shard_chunk

    gen = torch.Generator(device=device).manual_seed(1234)
    x = torch.randn(M, K, device=device, generator=gen, dtype=torch.float32).to(torch.bfloat16)
    chunk = shard_chunk(N, world) if world > 1 else N
    wgen = torch.Generator(device=device).manual_seed(99 + rank)
    w = (torch.randn(chunk, K, device=device, generator=wgen) * K ** -0.5).to(torch.bfloat16)
    b = (torch.randn(chunk, device=device, generator=wgen) * math.sqrt(0.1)).to(torch.bfloat16)
    if world > 1:  # zero the padding rows of the last shard
        valid = max(0, min(chunk, N - rank * chunk))
        w[valid:] = 0
        b[valid:] = 0
    return x, w, b, chunk


def cpu_operands(rows: int = M):
    """The CPU path's operands: X [rows, K] bf16 (the step's input), and W and b
    as resident fp32 parameters -- converted once, outside any timed call, as
    a CPU deployment of the reference's fp32 path would hold them."""
    gen = torch.Generator().manual_seed(7)
    x = torch.randn(rows, K, generator=gen).bfloat16()
    w = (torch.randn(N, K, generator=gen) * K ** -0.5).bfloat16()
    b = (torch.randn(N, generator=gen) * math.sqrt(0.1)).bfloat16()
    return x, w.float().t(), b.float()


def cpu_baseline(budget_s: float = 10.0) -> dict:
    """The reference's CPU path (oracle restatement, torch on host cores, fp32)
    over the whole workload (all 4096 rows of X), as many calls as fit in
    ``budget_s``."""
    from oracle.cpu_reference import torch_cpu

    torch.set_num_threads(os.cpu_count() or 1)
    x, wt, b = cpu_operands()
    torch_cpu.linear_gelu(x[:64], wt, b, "none")  # warm the BLAS
    calls, start = 0, time.perf_counter()
    while True:
        torch_cpu.linear_gelu(x, wt, b, "none")
        calls += 1
        elapsed = time.perf_counter() - start
        if elapsed >= budget_s or calls >= 50:
            break
    return {"value": FLOP * calls / elapsed / 1e12, "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{calls} calls of the full {M}x{N}x{K} step (fp32 math; W and b held in fp32, "
                      f"X converted per call) in {elapsed:.1f} s",
            "host_cpus": os.cpu_count()}


# ------------------------------------------------------------------ secondary rows
class ReferenceKernels:
    """The reference's own GPU kernels, for comparison lines only: its Triton
    kernels (JIT-compiled for this GPU by the Triton in this image) and its
    hand-written CUDA RMSNorm (built with torch's extension loader), imported
    from the reference package installed under ``baseline/_ref``. Nothing in
    ``kernelo_b200`` uses them."""

    AUTOTUNE_TOP = ((128, 256, 64, 8, 3), (128, 128, 32, 4, 4), (64, 256, 32, 4, 4), (128, 64, 32, 4, 4))

    def __init__(self) -> None:
        self.error = None
        path = REPO / "baseline" / "_ref"
        if not (path / "kernelforge").is_dir():
            self.error = "reference package not installed under baseline/_ref"
            return
        if str(path) not in sys.path:
            sys.path.append(str(path))
        try:
            import kernelforge.kernels.fused_linear as fl
            import kernelforge.kernels.matmul as mm
            import kernelforge.kernels.rmsnorm as rn
            import kernelforge.kernels.softmax as sm
            from kernelforge.tuning.config import KernelConfig as RefConfig
        except Exception as exc:  # noqa: BLE001 - report, do not fail the bench
            self.error = f"import failed: {type(exc).__name__}: {exc}"
            return
        self.fl, self.mm, self.rn, self.sm, self.Config = fl, mm, rn, sm, RefConfig
        self._cuda_rms = None

    def fused_best_config(self, x, w_kn, b, single_ms):
        """The best of the reference's top autotune configs on its fused kernel."""
        best = None
        for bm, bn, bk, warps, stages in self.AUTOTUNE_TOP:
            cfg = self.Config("fused_linear", BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk, GROUP_M=8, num_warps=warps,
                              num_stages=stages)
            try:
                ms = single_ms(lambda cfg=cfg: self.fl.fused_linear_gelu(x, w_kn, b, config=cfg), iters=3)
            except Exception:  # noqa: BLE001 - a config Triton cannot build is skipped
                continue
            if best is None or ms < best[0]:
                best = (ms, cfg)
        return None if best is None else best[1]

    def cuda_rmsnorm(self):
        if self._cuda_rms is None:
            from kernelforge.kernels import cuda_rmsnorm as ext

            if not ext.available():
                raise RuntimeError("no CUDA toolkit for the reference's extension")
            ext.load()
            self._cuda_rms = ext.cuda_rmsnorm
        return self._cuda_rms


def secondary_lines(pk: dict, flush, *, reference_kernels: bool = True) -> list[dict]:
    """Every other BASELINE configuration at N=1: the plain GEMM (config 0)
    and the fp16 fused linear in TFLOP/s against the burst GEMM peak, and the
    memory-bound rows (RMSNorm, softmax in every dtype and width, decode GEMV)
    in GB/s against the HBM copy peak.

    ``value`` is device time per launch from a CUDA graph of back-to-back
    launches that cycle through input sets together larger than twice the L2
    (no launch finds its inputs cached, no host overhead or event gap inside);
    ``single_launch`` is one launch between two events after an L2 flush (clean
    lines), which adds the ~6 us launch-and-event floor. Comparison figures on
    the same inputs and timing: cuBLAS (torch) where it has the op, and the
    reference's own kernels (``vs_reference_triton``: our time's speed-up over
    theirs; ``vs_reference_cuda`` for its CUDA RMSNorm).
    """
    from kernelo_b200.benchmark.metrics import gemv_bytes, matmul_flops, rmsnorm_bytes, softmax_bytes
    from kernelo_b200.benchmark.runner import graph_time_per_launch, rotation_sets
    from kernelo_b200.kernels.fused_linear import fused_linear_gelu
    from kernelo_b200.kernels.gemv import gemv
    from kernelo_b200.kernels.matmul import matmul
    from kernelo_b200.kernels.rmsnorm import rmsnorm
    from kernelo_b200.kernels.softmax import softmax

    dev = torch.device("cuda")
    out = []
    ref = ReferenceKernels() if reference_kernels else None

    def single_ms(fn, iters=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
        for s, e in ev:
            flush()
            s.record()
            fn()
            e.record()
        torch.cuda.synchronize()
        return statistics.median(s.elapsed_time(e) for s, e in ev)

    def compare(entry, key, make_calls, ms):
        """Time another implementation's calls the same way; record its speed
        and our speed-up over it (or why it could not run)."""
        if make_calls is None:
            return
        try:
            other = graph_time_per_launch(make_calls())
            entry[key] = {"us_per_launch": round(other * 1e3, 2), "speedup": round(other / ms, 3)}
        except Exception as exc:  # noqa: BLE001 - a comparison never fails the bench
            entry[key] = {"unavailable": f"{type(exc).__name__}: {str(exc)[:160]}"}

    def line(metric, work, calls, sets, *, unit="GB/s", peak=None, peak_kind="measured HBM copy",
             cublas=None, reference=None, reference_cuda=None, reference_note=None):
        ms = graph_time_per_launch(calls)
        one = single_ms(calls[0])
        rate = work / ms / (1e6 if unit == "GB/s" else 1e9)
        peak = peak if peak is not None else pk["hbm_gbs"]
        entry = {"metric": metric, "value": round(rate, 1), "unit": unit, "frac": round(rate / peak, 3),
                 "peak": peak, "peak_kind": peak_kind, "us_per_launch": round(ms * 1e3, 2),
                 ("single_launch_gbs" if unit == "GB/s" else "single_launch_tflops"):
                     round(work / one / (1e6 if unit == "GB/s" else 1e9), 1),
                 "timing": f"CUDA graph of {len(calls)} launches over {sets} rotating input sets (> 2x L2)"}
        compare(entry, "vs_cublas", cublas, ms)
        if ref is not None:
            if ref.error is not None:
                entry["vs_reference_triton"] = {"unavailable": ref.error}
            elif reference_note is not None:
                entry["vs_reference_triton"] = {"unavailable": reference_note}
            else:
                compare(entry, "vs_reference_triton", reference, ms)
                compare(entry, "vs_reference_cuda", reference_cuda, ms)
        out.append(entry)
        return entry

    g = torch.Generator(device=dev).manual_seed(5)
    burst = pk["bf16_tflops"]
    ok = ref is not None and ref.error is None

    # config 0: plain GEMM 2048 x 4096 x 4096 fp16, row-major (K, N) B
    sets = rotation_sets((2048 * 4096 + 4096 * 4096 + 2048 * 4096) * 2, dev)
    As = [torch.randn(2048, 4096, device=dev, generator=g).half() for _ in range(sets)]
    Bs = [torch.randn(4096, 4096, device=dev, generator=g).half() for _ in range(sets)]
    pairs = list(zip(As, Bs)) * 4  # each call allocates its output, as the reference's wrapper does
    line("matmul 2048x4096x4096 fp16 (config 0)", matmul_flops(2048, 4096, 4096),
         [lambda a=a, b=b: matmul(a, b) for a, b in pairs], sets, unit="TFLOP/s", peak=burst,
         peak_kind="measured burst bf16 (cuBLAS; fp16 runs at the same tensor rate)",
         cublas=lambda: [lambda a=a, b=b: torch.mm(a, b) for a, b in pairs],
         reference=(lambda: [lambda a=a, b=b: ref.mm.matmul_triton_autotune(a, b) for a, b in pairs])
         if ok else None)
    del As, Bs, pairs

    # config 1 in fp16 (erf GELU, W [N, K]); the reference's fused kernel is
    # the tanh form, so its comparison is against this kernel's tanh epilogue
    sets = rotation_sets((M * K + N * K + M * N) * 2, dev)
    xs = [torch.randn(M, K, device=dev, generator=g).half() for _ in range(sets)]
    ws = [(torch.randn(N, K, device=dev, generator=g) * K ** -0.5).half() for _ in range(sets)]
    bs = [(torch.randn(N, device=dev, generator=g) * math.sqrt(0.1)).half() for _ in range(sets)]
    ys = [torch.empty(M, N, device=dev, dtype=torch.float16) for _ in range(sets)]
    quad = list(zip(xs, ws, bs, ys)) * 2
    import torch.nn.functional as F

    line(f"fused_linear erf 4096x{N}x4096 fp16", FLOP,
         [lambda x=x, w=w, b=b, y=y: fused_linear_gelu(x, w.t(), b, approximate="none", out=y)
          for x, w, b, y in quad], sets, unit="TFLOP/s", peak=burst,
         peak_kind="measured burst bf16 (cuBLAS; fp16 runs at the same tensor rate)",
         cublas=lambda: [lambda x=x, w=w, b=b: F.gelu(torch.addmm(b, x, w.t()), approximate="none")
                         for x, w, b, _ in quad], reference_note="the reference's fused kernel is tanh-only")
    ref_fused = None
    if ok:
        try:
            cfg = ref.fused_best_config(xs[0], ws[0].t(), bs[0], single_ms)
            if cfg is not None:
                ref_fused = (lambda: [lambda x=x, w=w, b=b: ref.fl.fused_linear_gelu(x, w.t(), b, config=cfg)
                                      for x, w, b, _ in quad])
        except Exception:  # noqa: BLE001
            ref_fused = None
    entry = line(f"fused_linear tanh 4096x{N}x4096 fp16", FLOP,
                 [lambda x=x, w=w, b=b, y=y: fused_linear_gelu(x, w.t(), b, approximate="tanh", out=y)
                  for x, w, b, y in quad], sets, unit="TFLOP/s", peak=burst,
                 peak_kind="measured burst bf16 (cuBLAS; fp16 runs at the same tensor rate)",
                 cublas=lambda: [lambda x=x, w=w, b=b: F.gelu(torch.addmm(b, x, w.t()), approximate="tanh")
                                 for x, w, b, _ in quad], reference=ref_fused,
                 reference_note=None if ref_fused is not None or not ok else "no reference config built")
    if ok and ref_fused is not None:
        entry["vs_reference_triton"]["config"] = "best of the reference's top-4 autotune configs"
    del xs, ws, bs, ys, quad

    for dt in (torch.float16, torch.bfloat16):
        for cols in (4096, 8192):
            nbytes = rmsnorm_bytes(16384, cols, 2)
            sets = rotation_sets(nbytes, dev)
            xs = [torch.randn(16384, cols, device=dev, generator=g).to(dt) for _ in range(sets)]
            gamma = (torch.randn(cols, device=dev, generator=g) * 0.1 + 1).to(dt)
            calls = [lambda x=x: rmsnorm(x, gamma, eps=1e-6) for x in xs] * 2
            line(f"rmsnorm 16384x{cols} {str(dt)[6:]}", nbytes, calls, sets,
                 cublas=None,
                 reference=(lambda: [lambda x=x: ref.rn.rmsnorm(x, gamma, eps=1e-6) for x in xs] * 2) if ok else None,
                 reference_cuda=(lambda: [lambda x=x, f=ref.cuda_rmsnorm(): f(x, gamma, eps=1e-6) for x in xs] * 2)
                 if ok else None)
            del xs, calls
    for dt in (torch.float16, torch.bfloat16, torch.float32):
        item = torch.empty(0, dtype=dt).element_size()
        for cols in (1000, 4096, 4097, 32000):
            nbytes = softmax_bytes(32768, cols, item)
            sets = rotation_sets(nbytes, dev)
            xs = [(torch.randn(32768, cols, device=dev, generator=g) * 4).to(dt) for _ in range(sets)]
            calls = [lambda x=x: softmax(x) for x in xs] * (2 if nbytes < (1 << 30) else 1)
            line(f"softmax 32768x{cols} {str(dt)[6:]}", nbytes, calls, sets,
                 reference=(lambda: [lambda x=x: ref.sm.softmax(x) for x in xs] * (2 if nbytes < (1 << 30) else 1))
                 if ok and cols <= 16384 else None,
                 reference_note="the reference's kernel refuses rows over 16384 columns" if cols > 16384 else None)
            del xs, calls
    wbytes = N * K * 2
    sets = rotation_sets(wbytes, dev)
    ws = [(torch.randn(N, K, device=dev, generator=g) * K ** -0.5).half() for _ in range(sets)]
    def with_overlap(entry, work, make_calls):
        """The same launches with overlap=True (weights are not written by the
        kernel before each call): programmatic dependent launch lets each GEMV
        stream its weight while its predecessor's last tiles finish, as in a
        decode loop of back-to-back layers."""
        try:
            ms = graph_time_per_launch(make_calls())
            rate = work / ms / 1e6
            entry["with_overlap"] = {"value": round(rate, 1), "frac": round(rate / pk["hbm_gbs"], 3),
                                     "us_per_launch": round(ms * 1e3, 2)}
        except Exception as exc:  # noqa: BLE001 - a variant never fails the bench
            entry["with_overlap"] = {"unavailable": f"{type(exc).__name__}: {str(exc)[:160]}"}

    for m in (1, 4, 16):
        xx = torch.randn(m, K, device=dev, generator=g).half()
        calls = [lambda w=w: gemv(xx, w) for w in ws] * 4
        entry = line(f"gemv M={m} N={N} K={K} fp16", gemv_bytes(m, N, K, 2), calls, sets,
                     cublas=lambda: [lambda w=w: torch.mm(xx, w.t()) for w in ws] * 4,
                     reference=(lambda: [lambda w=w: ref.mm.matmul_triton_autotune(xx, w.t()) for w in ws] * 4)
                     if ok else None)
        with_overlap(entry, gemv_bytes(m, N, K, 2), lambda: [lambda w=w: gemv(xx, w, overlap=True) for w in ws] * 4)
    del ws
    # Not a BASELINE config: the MLP down-projection's decode shape (the
    # transpose of config 2's weight, long K), where the library takes the
    # streamed tile kernel beyond 8 rows of x.
    n2, k2 = K, N
    sets = rotation_sets(n2 * k2 * 2, dev)
    ws = [(torch.randn(n2, k2, device=dev, generator=g) * k2 ** -0.5).half() for _ in range(sets)]
    for m in (1, 16):
        xx = torch.randn(m, k2, device=dev, generator=g).half()
        entry = line(f"gemv M={m} N={n2} K={k2} fp16 (down-projection shape)", gemv_bytes(m, n2, k2, 2),
                     [lambda w=w: gemv(xx, w) for w in ws] * 4, sets,
                     cublas=lambda: [lambda w=w: torch.mm(xx, w.t()) for w in ws] * 4)
        with_overlap(entry, gemv_bytes(m, n2, k2, 2), lambda: [lambda w=w: gemv(xx, w, overlap=True) for w in ws] * 4)
    del ws
    return out


# ------------------------------------------------------------------ arms
def run_reference(args, world: int, rank: int) -> int:
    if rank != 0:
        return 0
    # Every host thread the box has: torchrun sets OMP_NUM_THREADS=1 for its
    # workers, which would time the reference's CPU path on one core.
    torch.set_num_threads(os.cpu_count() or 1)
    from oracle.cpu_reference import torch_cpu

    # Each step is the whole workload -- all 4096 rows, about a third of a
    # second on 16 cores, W and b resident in fp32 -- unless K + W such steps
    # would exceed three minutes; then each step is the largest multiple of
    # 64 rows that keeps the run within that bound.
    x, w, b = cpu_operands()
    t0 = time.perf_counter()
    torch_cpu.linear_gelu(x, w, b, "none")
    full_s = time.perf_counter() - t0
    calls = args.steps + max(args.warmup, 1)
    if full_s * calls > 180.0:
        x = x[: max(64, int(M * 180.0 / (full_s * calls)) // 64 * 64)]
    rows = x.shape[0]
    for _ in range(max(args.warmup, 1)):
        torch_cpu.linear_gelu(x, w, b, "none")
    start = time.perf_counter()
    for _ in range(args.steps):
        torch_cpu.linear_gelu(x, w, b, "none")
    elapsed = time.perf_counter() - start
    value = 2 * rows * N * K * args.steps / elapsed / 1e12
    sample = (f"each step {'the full' if rows == M else f'{rows} of the {M} rows of the'} {M}x{N}x{K} "
              "workload (torch fp32 on host cores; W and b held in fp32, X converted per step)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample_rows": rows, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_native(args, world: int, rank: int, local: int) -> int:
    from kernelo_b200.distributed import ShardedFusedLinear
    from kernelo_b200.kernels.fused_linear import fused_linear_gelu, fused_linear_gelu_host
    from kernelo_b200.runtime import native

    dev = torch.device("cuda", local)
    pk, pk_kind = peaks()
    x, w, b, chunk = make_inputs(dev, rank, world)
    mode = "single"
    if world > 1:
        layer = ShardedFusedLinear(None, None, out_features=N, shard_weight=w, shard_bias=b, approximate="none",
                                   gather="auto")
        written: list[torch.Tensor] = []

        # layer(x) in two parts, so the timed loop can bracket the kernel alone:
        # the GEMM whose epilogue also stores every output tile into the peers'
        # copies of Y over NVLink, then the bounded cross-GPU barrier
        def launch_kernel():
            written[:] = [layer.fused_kernel(x)]

        def finish_step():
            layer.fused_publish(x)
            return written[0][:, :N]
    else:
        y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)

        def launch_kernel():
            fused_linear_gelu(x, w.t(), b, approximate="none", out=y)

        def finish_step():
            return y

    def step():
        launch_kernel()
        return finish_step()

    # correctness gate on a sample before timing (never inside the timed region)
    out = step()
    torch.cuda.synchronize()
    rows = torch.arange(0, M, 97, device=dev)[:32]
    if world == 1:
        ref = torch.nn.functional.gelu(x[rows].float() @ w.float().t() + b.float(), approximate="none")
        err = float((out[rows].float() - ref).abs().max() / ref.abs().max())
        if not err < 2e-2:
            raise SystemExit(f"fused linear failed the bf16 gate before timing: err={err:.3e}")
    else:
        # every rank's tiles must have arrived: the same layer gathered by NCCL
        nccl = ShardedFusedLinear(None, None, out_features=N, shard_weight=w, shard_bias=b, approximate="none",
                                  gather="nccl")
        differs = float(not torch.equal(out, nccl(x)))
        torch.cuda.synchronize()
        del nccl
        if max_over_ranks(differs, world) > 0:  # every rank takes the same exit
            raise SystemExit("the fused all-gather differs from the NCCL all-gather before timing")
        # The layer's own choice of gather at this N, by measurement (collective;
        # every rank sees the slowest rank's times, so all choose alike).
        mode = layer.gather_mode(x)
        if mode == "nccl":
            # the local GEMM is the bracketed kernel; NCCL's all-gather follows
            def launch_kernel():
                layer.nccl_kernel(x)

            def finish_step():
                return layer.nccl_publish(x)
    if max_over_ranks(float(native.device_status(local) != 0), world) > 0:
        raise SystemExit("device status word set before timing")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream(dev)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    # every launch of the dominant kernel bracketed on its own stream, inside the timed region
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        barrier(world)
        start.record(stream)
        for ks, ke in kev:
            ks.record(stream)
            launch_kernel()
            ke.record(stream)
            finish_step()
        end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    if max_over_ranks(float(native.device_status(local) != 0), world) > 0:
        raise SystemExit(f"device status word {native.device_status(local):#x} after the timed loop")
    ms_total = max_over_ranks(start.elapsed_time(end), world)
    ms_step = ms_total / args.steps
    value = FLOP * args.steps / (ms_total * 1e-3) / 1e12

    # the dominant kernel's average launch duration over the timed region
    kernel_ms = max_over_ranks(sum(ks.elapsed_time(ke) for ks, ke in kev) / len(kev), world)
    flop_rank = 2 * M * chunk * K  # this rank's column shard (padded to the shard width)
    achieved = flop_rank / (kernel_ms * 1e-3) / 1e12
    clock_summary = clocks.summary()
    # The denominator follows the run: burst for a short region at full
    # clocks, sustained only for seconds under the power cap.
    peak, peak_kind = tensor_peak_for_run(pk, pk_kind, clock_summary, ms_total * 1e-3)
    burst, sustained = pk["bf16_tflops"], pk.get("bf16_tflops_sustained")
    if world == 1:
        roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                    "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                    "frac_of_burst": round(achieved / burst, 4),
                    "frac_of_sustained": round(achieved / sustained, 4) if sustained else None,
                    "traffic": profile_traffic("tc_gemm_fused_linear_erf_bf16"),
                    "kernel": "tc_gemm_kernel<bf16,erf>", "kernel_ms": round(kernel_ms, 4)}
    else:
        link = measure_peer_copy_gbs(dev, world, rank)
        if mode == "fused":
            roofline = allgather_roofline(flop_rank, M * chunk * 2 * (world - 1), kernel_ms, peak, peak_kind,
                                          link["gbs"])
        else:
            # the bracketed kernel is the shard's GEMM alone; NCCL gathers after it
            roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": None,
                        "kernel": "tc_gemm_kernel<bf16,erf> (shard; NCCL all-gather follows)",
                        "kernel_ms": round(kernel_ms, 4), "step_ms": round(ms_step, 4)}
        roofline["nvlink_measurement"] = link
        roofline["gather"] = {"chosen": mode, "ms_per_3_calls": layer.gather_timings.get(M)}

    # end to end through the public API: pinned host X in, Y back to pinned host
    e2e_steps = max(3, min(20, args.steps))
    x_host = x.cpu().pin_memory()
    y_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        if world > 1:
            # each rank moves 1/world of X in and of Y out over its own PCIe link
            layer.forward_host(x_host, y_host)
        else:
            # the host-buffer entry point: row chunks overlap H2D, the kernel and D2H
            fused_linear_gelu_host(x_host, w.t(), b, approximate="none", out=y_host)

    e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    ee.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(es.elapsed_time(ee), world)
    e2e_value = FLOP * e2e_steps / (e2e_ms * 1e-3) / 1e12
    # The host link bounds the end-to-end figure: each step moves X in and Y
    # out (the two directions overlap on separate copy engines), split over
    # the ranks' own PCIe links at N > 1.
    pcie = pcie_rates(dev)
    h2d_s = x.numel() * 2 / world / (pcie["h2d_gbs"] * 1e9)
    d2h_s = M * N * 2 / world / (pcie["d2h_gbs"] * 1e9)
    pcie_bound = FLOP / max(h2d_s, d2h_s) / 1e12

    secondary = []
    baseline = None
    if rank == 0 and world == 1 and not args.no_secondary:
        from kernelo_b200.benchmark.runner import L2Flush

        flush = L2Flush(dev)
        secondary = secondary_lines(pk, flush, reference_kernels=not args.no_reference_kernels)
        del flush
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        baseline = cpu_baseline()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) X, N(0,1/4096) W, N(0,0.1) b; random init)",
            "config": {"workload": WORKLOAD, "M": M, "N": N, "K": K, "gelu": "erf",
                       "parallelism": ("single GPU" if world == 1 else
                                       f"N-sharded columns x{world}, all-gather fused into the GEMM epilogue "
                                       "(NVLink peer stores) + bounded peer barrier" if mode == "fused" else
                                       f"N-sharded columns x{world}, local GEMM + NCCL all_gather_into_tensor "
                                       "(chosen over the fused gather by measurement at this N)"),
                       "l2": "inputs exceed L2 (X 32 MiB + W 86 MiB + Y 86 MiB > 126 MiB), no flush"},
            "roofline": roofline,
            "clocks": clock_summary,
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": x.numel() * 2,
                    "d2h_bytes_per_step": M * N * 2, "steps": e2e_steps,
                    "bound": {"by": "host link (PCIe), pinned copies measured in this run on rank 0",
                              **pcie, "tflops_if_copies_alone": round(pcie_bound, 1),
                              "frac": round(e2e_value / pcie_bound, 3)},
                    "api": ("fused_linear_gelu_host (pinned X in, pinned Y out, row chunks (a 256-row first one) overlapping "
                            "copies and kernel)" if world == 1 else
                            "ShardedFusedLinear.forward_host: each rank copies 1/N of X's rows in and 1/N of "
                            f"Y's rows out (bytes summed over ranks), X all-gathered over NVLink, "
                            f"{max(1, 8 // world)} row chunk(s) pipelined")},
            "gpu_launches": args.steps * (2 if mode == "fused" else 1),
            "cpu_baseline": baseline,
            "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        layer.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    p.add_argument("--no-secondary", action="store_true", help="skip the memory-bound rows")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-reference-kernels", action="store_true",
                   help="skip the comparison with the reference's own GPU kernels")
    args = p.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return run_reference(args, world, rank)
    world, rank, local = dist_setup(args.gpus)
    return run_native(args, world, rank, local)


if __name__ == "__main__":
    sys.exit(main())
