"""GPU runtime pieces: bounded device waits, the timing harness, the tuner
and cache-backed dispatch on real kernels.

Failure detection is tested without a fault: a kernel waits on an mbarrier
that nothing completes, gives up after a short limit, records KF_ERR_TIMEOUT
(with its site) in the device status word and returns; the context stays
usable and the next kernels run normally.
"""

from __future__ import annotations

import pytest
import torch

from kernelo_b200.benchmark.runner import benchmark, cross_check_median_ms
from kernelo_b200.runtime import native
from kernelo_b200.tuning.config import Problem

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports_its_site(device):
    assert native.device_status(device.index) == 0
    native.selftest_bounded_wait(20_000)  # 20 ms
    torch.cuda.synchronize(device)
    value = native.device_status(device.index)
    assert value & 0xFF == native.KF_ERR_TIMEOUT and value >> 8 == 6
    assert native.device_status(device.index) == 0  # read-and-clear
    # The context is intact: a real kernel still runs and verifies.
    from kernelo_b200.kernels.softmax import softmax

    x = torch.randn(4, 1000, device=device)
    assert torch.allclose(softmax(x), torch.softmax(x, -1), atol=1e-6)


def test_a_recorded_timeout_surfaces_as_an_exception(device):
    native.selftest_bounded_wait(5_000)
    with pytest.raises(native.KernelTimeoutError, match="wait site 6"):
        native.raise_on_device_status(device.index)


def test_counted_peer_barrier_advances_its_device_epoch(device):
    """The graph-replayable barrier on one GPU, as rank 0 of 2 with a "peer"
    signal array that is another local buffer. The peer's arrival is planted
    in advance (this rank's slot for rank 1 already holds a later epoch), so
    no launch waits on another: each barrier takes counter + 1 as its epoch,
    stores it back and signals the peer with it, eagerly and on every replay
    of a captured graph; a barrier whose peer never reaches the epoch gives
    up after its limit with the barrier's site in the status word."""
    local = torch.zeros(2, dtype=torch.int32, device=device)
    peer = torch.zeros(2, dtype=torch.int32, device=device)
    counter = torch.zeros(1, dtype=torch.int32, device=device)
    local[1] = 100  # rank 1 "arrived" up to epoch 100

    def barrier():
        native.peer_barrier_counted(local.data_ptr(), [peer.data_ptr()], 0, 2, counter.data_ptr(),
                                    timeout_us=1_000_000, device=device)

    barrier()
    barrier()
    torch.cuda.synchronize(device)
    assert counter.item() == 2 and peer.tolist() == [2, 0]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        barrier()
        barrier()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(device)
    del graph
    assert counter.item() == 8 and peer.tolist() == [8, 0]
    assert native.device_status(device.index) == 0
    # rank 1 stopped at epoch 100: the barrier of epoch 101 times out (20 ms)
    counter.fill_(100)
    native.peer_barrier_counted(local.data_ptr(), [peer.data_ptr()], 0, 2, counter.data_ptr(),
                                timeout_us=20_000, device=device)
    torch.cuda.synchronize(device)
    value = native.device_status(device.index)
    assert value & 0xFF == native.KF_ERR_TIMEOUT and value >> 8 == 7
    assert counter.item() == 101 and peer[0].item() == 101
    with pytest.raises(ValueError, match="null epoch counter"):
        native.peer_barrier_counted(local.data_ptr(), [peer.data_ptr()], 0, 2, 0, device=device)


def test_native_library_is_the_in_tree_build(device):
    import os

    from kernelo_b200.csrc import build

    lib = native.load()
    assert os.path.samefile(lib._name, build.LIB_PATH)
    assert native.sm_count(device.index) == torch.cuda.get_device_properties(device).multi_processor_count


def test_harness_uses_cuda_events_and_the_flush_matters(device):
    x = torch.randn(4096, 4096, device=device)
    r = benchmark(lambda: x * 2, warmup=5, iterations=20, device=device)
    assert r.timer == "cuda_event" and r.flushed_l2 and r.median_ms > 0
    # Kernel-dominated on purpose: a GEMM of a few microseconds is launch-bound on
    # a B200, and without the flush's memset ahead of it the measured interval
    # would include host launch gaps rather than the kernel. 4096^3 runs ~0.1 ms
    # with 32 MiB operands that stay L2-resident unless flushed.
    a = torch.randn(4096, 4096, device=device, dtype=torch.bfloat16)
    b = torch.randn(4096, 4096, device=device, dtype=torch.bfloat16)
    warm = benchmark(lambda: a @ b, warmup=10, iterations=50, device=device, flush_l2=False)
    cold = benchmark(lambda: a @ b, warmup=10, iterations=50, device=device, flush_l2=True)
    assert cold.median_ms >= warm.median_ms * 0.95


def test_harness_agrees_with_torch_benchmark(device):
    """Both timers over a similar span of back-to-back GEMMs (~10 ms each): a
    loop of half a second reaches the 1 kW power cap and runs at lower clocks
    (measured 0.101 against 0.119 ms), which is the GPU, not the harness."""
    from kernelo_b200.kernels.matmul import matmul

    a = torch.randn(4096, 4096, device=device, dtype=torch.bfloat16)
    b = torch.randn(4096, 4096, device=device, dtype=torch.bfloat16)
    ours = benchmark(lambda: matmul(a, b), warmup=10, iterations=100, device=device, flush_l2=False)
    theirs = cross_check_median_ms(lambda: matmul(a, b), min_run_time=0.01)
    assert ours.median_ms == pytest.approx(theirs, rel=0.15)


def test_tuning_writes_a_cache_entry_dispatch_reads(device, tmp_path):
    from kernelo_b200.db import ResultsDB
    from kernelo_b200.kernels import get_operator
    from kernelo_b200.runtime.dispatch import SOURCE_CACHE, SOURCE_DEFAULT, select_config
    from kernelo_b200.tuning.cache import ConfigCache
    from kernelo_b200.tuning.tuner import Tuner

    for name, problem in (
        ("rmsnorm", Problem.create("rmsnorm", "fp16", rows=512, cols=1024)),
        ("matmul", Problem.create("matmul", "bf16", M=512, N=512, K=1024)),
    ):
        op = get_operator(name)
        path = tmp_path / f"{name}.json"
        assert select_config(op, problem, cache=ConfigCache(path)).source == SOURCE_DEFAULT
        db = ResultsDB(tmp_path / "r.db")
        result = Tuner(warmup=3, iterations=10, max_candidates=6, cache=ConfigCache(path), db=db).tune(op, problem)
        assert result.best is not None and result.correct >= 1
        assert all(o.ok or o.status != "incorrect" for o in result.outcomes), result.status_counts()
        picked = select_config(op, problem, cache=ConfigCache(path))
        assert picked.source == SOURCE_CACHE and picked.config == result.best_config
        db.close()


def test_tuned_winner_is_no_slower_than_the_default(device):
    from kernelo_b200.kernels import get_operator
    from kernelo_b200.tuning.tuner import Tuner

    op = get_operator("matmul")
    problem = Problem.create("matmul", "fp16", M=2048, N=2048, K=2048)
    result = Tuner(warmup=5, iterations=30, max_candidates=8).tune(op, problem)
    default = result.baselines.get("kernelforge_default")
    assert result.best is not None
    if default is not None:
        assert result.best.median_ms <= default.median_ms * 1.05


def test_tile_gemv_runs_the_peer_barrier_in_its_last_cta(device):
    """kf_linear_bias_act_allgather_sync on the tile GEMV (M <= 32) as rank 0
    of 2, with the "peer" signal array and Y copy in local memory and rank 1's
    arrival planted in advance: each call stores Y and the peer copy, its last
    CTA advances the device epoch by one and signals the peer slot, and the
    arrival word is back at zero; a peer that never reaches the epoch makes
    the in-kernel wait give up after its limit with the barrier's site in the
    status word, the context still usable."""
    from kernelo_b200.kernels.gemv import gemv

    gen = torch.Generator().manual_seed(11)
    x = torch.randn(4, 512, generator=gen).half().to(device)
    w = (torch.randn(1000, 512, generator=gen) * 0.04).half().to(device)
    y = torch.empty(4, 1000, device=device, dtype=torch.float16)
    peer_y = torch.zeros_like(y)
    local = torch.zeros(2, dtype=torch.int32, device=device)
    peer_sig = torch.zeros(2, dtype=torch.int32, device=device)
    counter = torch.zeros(1, dtype=torch.int32, device=device)
    arrivals = torch.zeros(1, dtype=torch.int32, device=device)
    local[1] = 100  # rank 1 "arrived" up to epoch 100
    sync = native.peer_sync_struct(local.data_ptr(), [peer_sig.data_ptr()], 0, 2, counter.data_ptr(),
                                   arrivals.data_ptr(), timeout_us=1_000_000)
    for _ in range(3):
        native.linear_bias_act_allgather(x, w.t(), y, [peer_y.data_ptr()], bias=None,
                                         epilogue=native.KF_EPI_NONE, sync=sync)
    torch.cuda.synchronize(device)
    assert counter.item() == 3 and arrivals.item() == 0 and peer_sig.tolist() == [3, 0]
    assert native.device_status(device.index) == 0
    assert torch.equal(y, peer_y) and torch.equal(y, gemv(x, w))
    counter.fill_(100)  # rank 1 stopped at epoch 100: epoch 101 times out
    sync = native.peer_sync_struct(local.data_ptr(), [peer_sig.data_ptr()], 0, 2, counter.data_ptr(),
                                   arrivals.data_ptr(), timeout_us=20_000)
    native.linear_bias_act_allgather(x, w.t(), y, [peer_y.data_ptr()], bias=None, epilogue=native.KF_EPI_NONE,
                                     sync=sync)
    torch.cuda.synchronize(device)
    value = native.device_status(device.index)
    assert value & 0xFF == native.KF_ERR_TIMEOUT and value >> 8 == 7
    assert counter.item() == 101 and arrivals.item() == 0
    assert torch.equal(y, gemv(x, w))  # still usable
