"""Multi-process host logic on CPU: two gloo ranks.

Covers the parts of ``kernelo_b200.distributed`` that need no GPU: the shard
arithmetic and its validation, the row split, the sharded fused linear's and
decode GEMV's gather/permute paths (with the native kernel replaced by a CPU
stand-in in the child processes), and the tuner sweep dealt over ranks with
rank 0 as the single writer -- including a rank whose candidates all fail.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kernelo_b200 import distributed as kd


def test_shard_chunk_and_row_range():
    assert kd.shard_chunk(11008, 8) == 1376 and kd.shard_chunk(11008, 2) == 5504
    assert kd.shard_chunk(100, 3) == 48  # rounded to 16, padded
    spans = [kd.row_range(10, 4, r) for r in range(4)]
    assert spans == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert sum(b - a for a, b in (kd.row_range(32768, 8, r) for r in range(8))) == 32768
    with pytest.raises(ValueError):
        kd.row_range(10, 2, 2)


def test_forward_host_refuses_a_cpu_layer():
    """The host-to-host path runs the all-gathering kernel: a CPU layer is an
    error up front, not a failure deep inside torch."""
    w = torch.zeros(32, 16)
    layer = kd.ShardedFusedLinear(w, torch.zeros(32))
    with pytest.raises(ValueError, match="CUDA device"):
        layer.forward_host(torch.zeros(4, 16), torch.zeros(4, 32))


def test_shards_too_small_for_the_output_are_refused():
    with pytest.raises(ValueError, match="cannot hold"):
        kd.ShardedGemv(None, out_features=100, shard_weight=torch.zeros(64, 16))
    layer = kd.ShardedGemv(None, out_features=64, shard_weight=torch.zeros(64, 16))
    assert layer.b is None and layer.chunk == 64


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))


def _sharded_linear_worker(rank: int, world: int, port: int, out_q) -> None:
    _init(rank, world, port)
    try:
        import torch.nn.functional as F

        import kernelo_b200.distributed as mod

        # CPU stand-in for the native kernel: same signature, exact math.
        def fake_fused(x, w_t, b, *, approximate, config, out=None):
            y = F.gelu(x.float() @ w_t.float() + b.float(), approximate="none").to(x.dtype)
            if out is None:
                return y
            out.copy_(y)
            return out

        mod.fused_linear_gelu = fake_fused
        gen = torch.Generator().manual_seed(0)
        x = torch.randn(6, 32, generator=gen)
        w = torch.randn(50, 32, generator=gen) * 0.2  # N=50: padded to 2 x 64
        b = torch.randn(50, generator=gen)
        layer = mod.ShardedFusedLinear(w, b, approximate="none")
        y = layer(x)
        expected = F.gelu(x @ w.t() + b, approximate="none")
        out_q.put((rank, tuple(y.shape), float((y - expected).abs().max())))
    finally:
        dist.destroy_process_group()


def _sharded_gemv_worker(rank: int, world: int, port: int, out_q) -> None:
    _init(rank, world, port)
    try:
        import kernelo_b200.distributed as mod

        # CPU stand-in for the native GEMV: same signature, exact math.
        def fake_gemv(x, w, *, config=None, out=None):
            y = (x.double() @ w.double().t()).to(x.dtype)
            if out is None:
                return y
            out.copy_(y)
            return out

        mod.gemv = fake_gemv
        gen = torch.Generator().manual_seed(1)
        w = torch.randn(50, 32, generator=gen)  # N=50: padded to 2 x 64
        layer = mod.ShardedGemv(w, gather="nccl")
        errs = []
        for m in (1, 4, 16):
            x = torch.randn(m, 32, generator=gen)
            y = layer(x)
            errs.append((tuple(y.shape), float((y - x @ w.t()).abs().max())))
        refused = False
        try:
            layer(torch.zeros(257, 32))
        except ValueError:
            refused = True
        out_q.put((rank, layer.b is None, errs, refused))
    finally:
        dist.destroy_process_group()


def _tune_worker(rank: int, world: int, port: int, tmpdir: str, out_q) -> None:
    _init(rank, world, port)
    try:
        from kernelo_b200.db import ResultsDB
        from kernelo_b200.tuning.cache import ConfigCache
        from kernelo_b200.tuning.tuner import Tuner
        from tests.test_tuner import PROBLEM, _FakeOperator

        db = ResultsDB(os.path.join(tmpdir, "r.db")) if rank == 0 else None
        cache = ConfigCache(os.path.join(tmpdir, "c.json")) if rank == 0 else None
        tuner = Tuner(warmup=1, iterations=3, flush_l2=False, db=db, cache=cache)
        result = kd.distributed_tune(tuner, _FakeOperator(), PROBLEM, device="cpu", finalists=2)
        out_q.put((rank, result.tested, result.correct, result.best.config["MODE"]))
    finally:
        dist.destroy_process_group()


def _resume_worker(rank: int, world: int, port: int, tmpdir: str, out_q) -> None:
    """Tune once, then again with resume=True: the second sweep measures nothing."""
    _init(rank, world, port)
    try:
        from kernelo_b200.db import ResultsDB
        from kernelo_b200.tuning.tuner import Tuner
        from tests.test_tuner import PROBLEM, _FakeOperator

        db = ResultsDB(os.path.join(tmpdir, "r.db")) if rank == 0 else None
        first = kd.distributed_tune(Tuner(warmup=1, iterations=3, flush_l2=False, measure_baselines=False, db=db),
                                    _FakeOperator(), PROBLEM, device="cpu", finalists=0)
        calls = []

        class _Counting(_FakeOperator):
            def run(self, config, x):
                calls.append(config)
                return super().run(config, x)

        # only rank 0 holds the database, so only its tuner asks to resume; it
        # decides for every rank what is already done
        tuner = Tuner(warmup=1, iterations=3, flush_l2=False, measure_baselines=False, db=db,
                      resume=db is not None)
        second = kd.distributed_tune(tuner, _Counting(), PROBLEM, device="cpu", finalists=0)
        rows = db.counts()["results"] if db is not None else None
        out_q.put((rank, len(calls), first.tested, second.tested,
                   (first.best.config["MODE"], second.best.config["MODE"]), rows))
    finally:
        dist.destroy_process_group()


def _mismatched_shard_worker(rank: int, world: int, port: int, out_q) -> None:
    """Two ranks whose weight shards differ in size: the peer-mapped output
    would be laid out differently on each, so both must refuse before any
    buffer is allocated, mapped or written."""
    _init(rank, world, port)
    try:
        chunk = 32 if rank == 0 else 48
        layer = kd.ShardedFusedLinear(None, None, out_features=64, shard_weight=torch.zeros(chunk, 16),
                                      shard_bias=torch.zeros(chunk), gather="fused")
        try:
            layer.fused_kernel(torch.zeros(4, 16))
            out_q.put((rank, "no error"))
        except ValueError as exc:
            out_q.put((rank, str(exc)))
    finally:
        dist.destroy_process_group()


def _run(target, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, 2, port, *args, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(results)


def test_sharded_fused_linear_gathers_columns_on_two_ranks():
    for rank, shape, err in _run(_sharded_linear_worker):
        assert shape == (6, 50)
        assert err < 1e-5


def test_sharded_gemv_gathers_columns_on_two_ranks():
    """The decode GEMV sharded by weight rows: no bias anywhere, each rank's
    slice gathered into [M, N] (N padded to the shard grid, padding dropped),
    and more rows than the GEMV operator takes refused up front."""
    for rank, no_bias, errs, refused in _run(_sharded_gemv_worker):
        assert no_bias and refused
        for (shape, err), m in zip(errs, (1, 4, 16)):
            assert shape == (m, 50)
            assert err < 1e-5


def test_resumed_distributed_sweep_measures_nothing_twice(tmp_path):
    results = _run(_resume_worker, str(tmp_path))
    for rank, calls, first_tested, second_tested, (first_best, second_best), rows in results:
        assert calls == 0, f"rank {rank} re-ran {calls} stored candidates"
        assert second_tested == first_tested == 6
        assert second_best == first_best, "the stored outcomes rank as they did when measured"
    assert results[0][5] == 6  # rank 0's database: the first sweep's rows, none added


def test_tuning_sweep_is_dealt_over_ranks_and_written_once(tmp_path):
    results = _run(_tune_worker, str(tmp_path))
    # Both ranks see the merged outcome list: all 6 feasible candidates, 2 correct.
    assert [r[1:] for r in results] == [(6, 2, 0), (6, 2, 0)]
    from kernelo_b200.db import ResultsDB
    from kernelo_b200.tuning.cache import ConfigCache
    from tests.test_tuner import PROBLEM

    db = ResultsDB(tmp_path / "r.db")
    assert db.counts()["runs"] == 1  # a single writer
    entries = ConfigCache(tmp_path / "c.json").entries()
    assert len(entries) == 1 and entries[0].config["MODE"] == 0
    db.close()
    del PROBLEM


def test_ranks_with_different_shard_sizes_are_refused_before_any_peer_store():
    for rank, message in _run(_mismatched_shard_worker):
        assert "disagree" in message and "chunk=32" in message and "chunk=48" in message, (rank, message)
