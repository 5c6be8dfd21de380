"""Multi-GPU partitioning of the hot path (one process per GPU, torch.distributed).

Three shardings, each where the work splits naturally:

* :class:`ShardedFusedLinear` -- the fused linear is column-sharded by N: rank r
  holds rows [r*chunk, (r+1)*chunk) of the [N, K] weight and of the bias and
  computes its [M, chunk] slice of ``gelu(x @ W^T + b)`` with the native
  kernel. With ``gather="fused"`` the kernel's epilogue
  stores every output tile into all ranks' copies of Y over NVLink (peer
  pointers, mapped by CUDA IPC, into double-buffered copies) and a bounded cross-GPU
  barrier kernel publishes completion: no collective, no copy, and the
  transfer overlaps the math tile by tile. ``gather="nccl"`` (and ``"auto"``
  off CUDA) exchanges the slices with one ``all_gather_into_tensor`` of the
  group's backend and permutes them into [M, N]. ``gather="auto"`` (the
  default) on CUDA times both on the first call of each M and keeps the
  faster, by the slowest rank's time, so every rank picks the same. N is padded to ``world * chunk`` with zero weight rows (their
  columns are dropped).
* :class:`ShardedGemv` -- the decode GEMV ``x @ W^T`` sharded the same way:
  each rank streams 1/world of the weight (the HBM-bound part) through the
  16-row tile kernel, whose stores also write every peer's copy of Y; the
  bounded barrier publishes it. The gathered Y is at most a few hundred KB,
  so the exchange costs about the barrier's latency.
* :func:`row_range` -- softmax / RMSNorm rows split evenly; no exchange.
* :func:`distributed_tune` -- the tuner's budgeted candidates dealt round-robin
  to one worker per GPU; outcomes are gathered on rank 0, which alone writes
  the database and the cache, after re-timing the finalists on its own GPU
  (timings from different GPUs are never ranked against each other).

The reference has no multi-GPU code; this module is new. No TMA multicast is
used anywhere: the fused gather is plain stores to peer memory.
"""

from __future__ import annotations

from dataclasses import replace

import torch
import torch.distributed as dist

from kernelo_b200.kernels.fused_linear import _EPILOGUES, fused_linear_gelu
from kernelo_b200.kernels.gemv import MAX_ROWS as MAX_GEMV_ROWS
from kernelo_b200.kernels.gemv import gemv


def world_info(group=None) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def shard_chunk(total: int, world: int, align: int = 16) -> int:
    """Equal per-rank chunk (a multiple of ``align``) covering ``total``."""
    if world < 1 or total < 1:
        raise ValueError("total and world must be positive")
    per = -(-total // world)
    return -(-per // align) * align


def row_range(rows: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [start, stop) of ``rank`` when ``rows`` are split as evenly as possible."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class ShardedFusedLinear:
    """``gelu(x @ W^T + b)`` with W [N, K] column-sharded over the process group.

    ``weight`` and ``bias`` are the FULL tensors (each rank keeps only its
    slice); pass ``shard_weight``/``shard_bias`` instead to build directly from
    a rank-local slice of ``chunk`` rows.
    """

    _plain = False  # ShardedGemv: x @ W^T with no bias and no activation

    def __init__(
        self,
        weight: torch.Tensor | None,
        bias: torch.Tensor | None,
        *,
        out_features: int | None = None,
        shard_weight: torch.Tensor | None = None,
        shard_bias: torch.Tensor | None = None,
        approximate: str = "none",
        group=None,
        config=None,
        gather: str = "auto",
        barrier_timeout_us: int = 2_000_000,
    ) -> None:
        if gather not in ("auto", "fused", "nccl"):
            raise ValueError("gather must be 'auto', 'fused' or 'nccl'")
        if not self._plain and approximate not in _EPILOGUES:
            raise ValueError(f"approximate must be 'tanh', 'none' or 'erf', got {approximate!r}")
        self.group = group
        self.world, self.rank = world_info(group)
        self.approximate = approximate
        self.config = config
        self.gather = gather
        self.barrier_timeout_us = barrier_timeout_us
        self._symm: dict[int, _PeerOutput] = {}
        self._host: dict = {}  # forward_host state per M: X staging, peer output, copy streams
        self._host_out: dict[int, torch.Tensor] = {}
        if shard_weight is not None:
            if out_features is None or (shard_bias is None and not self._plain):
                raise ValueError("shard_weight needs out_features and shard_bias")
            self.n = out_features
            self.chunk = shard_weight.shape[0]
            if self.world * self.chunk < self.n:
                raise ValueError(f"{self.world} shards of {self.chunk} rows cannot hold {self.n} output features")
            self.w = shard_weight
            self.b = shard_bias
        else:
            if weight is None or (bias is None and not self._plain):
                raise ValueError("pass weight and bias, or shard_weight and shard_bias")
            self.n = weight.shape[0]
            self.chunk = shard_chunk(self.n, self.world)
            start = self.rank * self.chunk
            stop = min(self.n, start + self.chunk)
            k = weight.shape[1]
            w = torch.zeros(self.chunk, k, device=weight.device, dtype=weight.dtype)
            b = None if bias is None else torch.zeros(self.chunk, device=bias.device, dtype=bias.dtype)
            if stop > start:
                w[: stop - start].copy_(weight[start:stop])
                if b is not None:
                    b[: stop - start].copy_(bias[start:stop])
            self.w, self.b = w, b
        self._gather_buf: torch.Tensor | None = None
        self._auto: dict[int, str] = {}  # M -> the gather "auto" chose
        #: M -> {"fused": ms, "nccl": ms}, the measurements behind each choice
        self.gather_timings: dict[int, dict[str, float]] = {}

    def _epilogue(self) -> int:
        from kernelo_b200.runtime import native

        return native.KF_EPI_NONE if self._plain else _EPILOGUES[self.approximate]

    def local(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's [M, chunk] slice of the output."""
        return fused_linear_gelu(x, self.w.t(), self.b, approximate=self.approximate,
                                 config=self.config, out=out)

    def gather_mode(self, x: torch.Tensor) -> str:
        """"fused" or "nccl": fixed by ``gather``, or for ``"auto"`` on CUDA the
        faster of the two for this M, measured once (collective: every rank
        calls it with the same M)."""
        if self.gather != "auto":
            return self.gather
        if not x.is_cuda:
            return "nccl"
        m = x.shape[0]
        if m not in self._auto:
            self._auto[m] = self._measure_gathers(x)
        return self._auto[m]

    def _measure_gathers(self, x: torch.Tensor, calls: int = 3) -> str:
        """Median-free and cheap: one untimed call of each mode, then ``calls``
        timed back to back; each mode's time is the slowest rank's."""
        stream = torch.cuda.current_stream(x.device)
        spent = {}
        for mode in ("fused", "nccl"):
            run = self.fused_step if mode == "fused" else self.nccl_step
            run(x)
            torch.cuda.synchronize(x.device)
            dist.barrier(group=self.group)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for _ in range(calls):
                run(x)
            end.record(stream)
            end.synchronize()
            t = torch.tensor([start.elapsed_time(end)], device=x.device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            spent[mode] = float(t.item())
        self.gather_timings[x.shape[0]] = spent
        return min(spent, key=spent.get)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return self.local(x)[:, : self.n]
        if self.gather_mode(x) == "fused":
            return self.fused_step(x)
        return self.nccl_step(x)

    def nccl_step(self, x: torch.Tensor) -> torch.Tensor:
        """The local GEMM, then one all-gather of the group's backend and a permute into [M, N]."""
        self.nccl_kernel(x)
        return self.nccl_publish(x)

    def nccl_kernel(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's GEMM into its slot of the gather buffer (the first half of :meth:`nccl_step`)."""
        m = x.shape[0]
        if self._gather_buf is None or self._gather_buf.shape != (self.world, m, self.chunk):
            self._gather_buf = torch.empty(self.world, m, self.chunk, device=x.device, dtype=x.dtype)
        mine = self._gather_buf[self.rank]
        self.local(x, out=mine)
        return mine

    def nccl_publish(self, x: torch.Tensor) -> torch.Tensor:
        """The all-gather and the permute into [M, N] (the second half of :meth:`nccl_step`)."""
        m = x.shape[0]
        mine = self._gather_buf[self.rank]
        dist.all_gather_into_tensor(self._gather_buf.view(-1), mine.reshape(-1), group=self.group)
        full = self._gather_buf.permute(1, 0, 2).reshape(m, self.world * self.chunk)
        return full[:, : self.n]


    # ---------------------------------------------------------------- fused all-gather
    def fused_kernel(self, x: torch.Tensor, *, sync: bool = False) -> torch.Tensor:
        """Launch this rank's GEMM whose epilogue also writes every peer's Y;
        returns the buffer it wrote (valid on all ranks after :meth:`fused_publish`,
        or at once with ``sync``: the barrier follows in the same call, inside
        the kernel on the tile GEMV path)."""
        from kernelo_b200.runtime import native

        m = x.shape[0]
        sym = self._symm.get(m)
        if sym is None:
            sym = self._symm[m] = _PeerOutput(m, self.world * self.chunk, x.dtype, x.device, self.group,
                                              chunk=self.chunk)
        buf, peers = sym.next_buffer(self.rank * self.chunk)
        mine = buf[:, self.rank * self.chunk:(self.rank + 1) * self.chunk]
        native.linear_bias_act_allgather(x, self.w.t(), mine, peers, bias=self.b, epilogue=self._epilogue(),
                                         launch=native.GemmLaunch.from_config(self.config),
                                         sync=sym.sync(self.rank, self.world, self.barrier_timeout_us) if sync
                                         else None)
        return buf

    def fused_publish(self, x: torch.Tensor) -> None:
        """Enqueue the bounded cross-GPU barrier that completes the gather."""
        self._symm[x.shape[0]].barrier(self.rank, self.world, self.barrier_timeout_us)

    def forward_host(self, x_host: torch.Tensor, out: torch.Tensor, *, chunks: int | None = None) -> torch.Tensor:
        """The layer from host memory to host memory, the PCIe traffic split
        over the ranks: each rank copies 1/world of X's rows in (its own PCIe
        link), X is all-gathered over NVLink, every rank computes its column
        shard for all rows with the all-gathering kernel, and each rank copies
        its 1/world of Y's rows (all N columns) back out. Row chunks pipeline
        the copies, the gather and the kernels.

        ``chunks`` defaults to 8 / world (at least 1): the host copies are the
        limit here, and each chunk adds two cross-rank synchronisations (the X
        gather and the barrier) -- on B200 at 4096 x 11008 x 4096 the
        per-call time was lowest with 4 chunks at 2 GPUs, 2 at 4 and 1 at 8.

        ``x_host`` [M, K] and ``out`` [M, N] are pinned host tensors; on return
        (after synchronizing this rank's current stream) this rank's rows of
        ``out`` hold the result -- rank r owns rows [a + r*q, a + (r+1)*q) of
        every chunk [a, a + world*q). Collective: every rank calls it with the
        same shapes. CUDA only (the all-gathering kernel).
        """
        from kernelo_b200.runtime import native

        if not self.w.is_cuda:
            raise ValueError("forward_host runs the all-gathering kernel: the layer must be on a CUDA device")
        if not (x_host.is_pinned() and out.is_pinned()):
            raise ValueError("forward_host needs pinned host tensors")
        m, k = x_host.shape
        if out.shape != (m, self.n):
            raise ValueError(f"out must be [{m}, {self.n}]")
        dev = self.w.device
        world, rank = self.world, self.rank
        if chunks is None:
            chunks = max(1, 8 // world)
        chunks = max(1, min(chunks, m // max(1, world)))
        q = -(-m // (world * chunks))  # rows per rank per chunk
        step = q * world
        key = ("host", m)
        state = self._host.get(key)
        if state is None:
            x_dev = torch.empty(step * chunks, k, device=dev, dtype=x_host.dtype)
            sym = (_PeerOutput(m, world * self.chunk, x_host.dtype, dev, self.group, chunk=self.chunk)
                   if world > 1 else None)
            state = self._host[key] = (x_dev, sym, torch.cuda.Stream(dev), torch.cuda.Stream(dev))
        x_dev, sym, h2d, d2h = state
        compute = torch.cuda.current_stream(dev)
        if sym is not None:
            buf = sym.bufs[sym.parity]
            parity = sym.parity
            sym.parity ^= 1
        else:
            buf = self._host_out.get(m)
            if buf is None:
                buf = self._host_out[m] = torch.empty(m, self.chunk, device=dev, dtype=x_host.dtype)
        launch = native.GemmLaunch.from_config(self.config)
        h2d.wait_stream(compute)  # x_dev is free once the previous call's kernels ran
        elt = buf.element_size()
        for c in range(chunks):
            a = c * step
            if a >= m:
                break
            b = min(m, a + step)
            mine0 = min(b, a + rank * q)
            mine1 = min(b, a + (rank + 1) * q)
            with torch.cuda.stream(h2d):
                if mine1 > mine0:
                    x_dev[mine0:mine1].copy_(x_host[mine0:mine1], non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(h2d)
            compute.wait_event(ready)
            if world > 1:
                dist.all_gather_into_tensor(x_dev[a:a + step], x_dev[a + rank * q:a + (rank + 1) * q],
                                            group=self.group)
                cols = slice(rank * self.chunk, (rank + 1) * self.chunk)
                peers = [sym.peer_ptrs[parity][j] + (a * buf.shape[1] + rank * self.chunk) * elt
                         for j in range(world) if j != rank]
                native.linear_bias_act_allgather(x_dev[a:b], self.w.t(), buf[a:b, cols], peers, bias=self.b,
                                                 epilogue=self._epilogue(), launch=launch)
                sym.barrier(rank, world, self.barrier_timeout_us)
                rows_out = buf[mine0:mine1, : self.n]
            else:
                self.local(x_dev[a:b], out=buf[a:b])
                rows_out = buf[mine0:mine1, : self.n]
            done = torch.cuda.Event()
            done.record(compute)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                if mine1 > mine0:
                    out[mine0:mine1].copy_(rows_out, non_blocking=True)
        # later barrier signals (which let peers overwrite this buffer) follow
        # this call's reads of it
        compute.wait_stream(d2h)
        return out

    def close(self) -> None:
        """Unmap the peers' output buffers. Collective: call on every rank, after
        the last use of a fused result; the process group stays usable."""
        for sym in self._symm.values():
            sym.close()
        for _, sym, _, _ in self._host.values():
            if sym is not None:
                sym.close()
        self._symm.clear()
        self._host.clear()
        if self.world > 1:
            dist.barrier(group=self.group)

    def fused_step(self, x: torch.Tensor, *, check_status: bool = False) -> torch.Tensor:
        """``gelu(x @ W^T + b)`` as a full [M, N] view of the peer-mapped output.

        Two buffers alternate between calls, so the result stays valid until
        the call after next; consume it (on this stream) before then.

        The barrier that publishes the result gives up after
        ``barrier_timeout_us`` when a peer does not answer: it records
        ``KF_ERR_TIMEOUT`` in the device status word and still advances its
        epoch, so later calls run on without the guarantee that a peer has
        consumed a buffer before it is overwritten, and their results cannot
        be trusted. ``check_status=True`` synchronizes the stream after the
        barrier and raises if the status word is set (a host round trip per
        call); otherwise read :func:`kernelo_b200.runtime.native.device_status`
        at a point of your choosing."""
        buf = self.fused_kernel(x, sync=True)
        if check_status:
            from kernelo_b200.runtime import native

            native.raise_on_device_status(x.device.index)
        return buf[:, : self.n]


class ShardedGemv(ShardedFusedLinear):
    """Decode GEMV ``x @ W^T`` (no bias, no activation) with W [N, K]
    column-sharded over the process group.

    Each rank reads only its ``chunk`` rows of the weight -- 1/world of the
    HBM traffic that bounds the single-GPU GEMV -- through the 16-row tile
    kernel for up to 32 rows of x (the tcgen05 GEMM above that, up to the
    GEMV operator's 256 rows).
    With ``gather="fused"`` that kernel's stores also write every peer's copy
    of Y and the bounded barrier publishes it; at M = 16, N = 11008 the whole
    gathered Y is 352 KB. ``gather="nccl"`` runs
    :func:`kernelo_b200.kernels.gemv.gemv` locally and all-gathers the slices;
    ``"auto"`` measures both on the first call of each M and keeps the faster.
    ``forward_host`` and ``close`` behave as for the fused linear.

    The reference has no dedicated GEMV and no multi-GPU code: single-GPU
    decode is its ``matmul`` at M in {1, 4, 16}
    (kernelforge/kernels/matmul.py:132-155).
    """

    _plain = True

    def __init__(
        self,
        weight: torch.Tensor | None,
        *,
        out_features: int | None = None,
        shard_weight: torch.Tensor | None = None,
        group=None,
        config=None,
        gather: str = "auto",
        barrier_timeout_us: int = 2_000_000,
    ) -> None:
        super().__init__(weight, None, out_features=out_features, shard_weight=shard_weight, group=group,
                         config=config, gather=gather, barrier_timeout_us=barrier_timeout_us)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[0] > MAX_GEMV_ROWS:
            raise ValueError(f"gemv takes at most {MAX_GEMV_ROWS} rows, got {x.shape[0]}; use matmul")
        return super().__call__(x)

    def local(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's [M, chunk] slice of ``x @ W^T``."""
        return gemv(x, self.w, config=self.config, out=out)


def check_peer_geometry(m: int, n_total: int, dtype: torch.dtype, chunk: int, group=None) -> None:
    """Raise ``ValueError`` on every rank unless all ranks agree on the peer
    output's geometry.

    Each rank stores its tiles at columns ``[rank*chunk, (rank+1)*chunk)`` of
    every peer's [m, n_total] buffer, computed from its own ``chunk``; a rank
    whose shard (or M, or dtype) differs would write past the end of another
    GPU's buffer. The check runs before any buffer is allocated, mapped or
    written. Collective over ``group``.
    """
    world = dist.get_world_size(group)
    mine = (int(m), int(n_total), str(dtype), torch.empty(0, dtype=dtype).element_size(), int(chunk))
    everyone: list = [None] * world
    dist.all_gather_object(everyone, mine, group=group)
    if any(g != everyone[0] for g in everyone):
        detail = ", ".join(f"rank {r}: m={g[0]} n_total={g[1]} dtype={g[2]} chunk={g[4]}"
                           for r, g in enumerate(everyone))
        raise ValueError(f"ranks disagree on the sharded output's geometry ({detail})")
    if chunk * world != n_total:
        raise ValueError(f"{world} shards of {chunk} columns do not tile {n_total} output columns")


class _PeerOutput:
    """Two copies of Y [M, n_total] and a signal array on every rank, each
    mapped into every other rank by CUDA IPC handles (exchanged over the
    process group's store); no NVLink multicast object is created.

    Double buffering: call i writes buffer i % 2 on every rank. A rank cannot
    start call i + 2 (and overwrite a peer's buffer i % 2) before that peer has
    signalled the barrier of call i + 1, which it enqueues after whatever it
    did with the result of call i.
    """

    def __init__(self, m: int, n_total: int, dtype: torch.dtype, device: torch.device, group, *,
                 chunk: int) -> None:
        from kernelo_b200.runtime import native

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        check_peer_geometry(m, n_total, dtype, chunk, group)
        self.bufs = [torch.empty((m, n_total), dtype=dtype, device=device) for _ in range(2)]
        self.signals = torch.zeros((self.world,), dtype=torch.int32, device=device)
        # this rank's barrier epoch, advanced on the device by each barrier,
        # and the arrival word of the in-kernel barrier (left at zero)
        self.counter = torch.zeros((1,), dtype=torch.int32, device=device)
        self.arrivals = torch.zeros((1,), dtype=torch.int32, device=device)
        self._sync = None
        torch.cuda.synchronize(device)
        mine = [native.ipc_handle(t) for t in (*self.bufs, self.signals)]
        everyone: list = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self._opened: list[int] = []
        bases: dict[tuple[int, int], int] = {}
        self.peer_ptrs: list[list[int]] = [[0] * self.world for _ in range(3)]
        for j in range(self.world):
            for i, (handle, offset) in enumerate(everyone[j]):
                if j == self.rank:
                    addr = (self.bufs + [self.signals])[i].data_ptr()
                else:
                    key = (j, handle)
                    if key not in bases:
                        bases[key] = native.ipc_open(handle)
                        self._opened.append(bases[key])
                    addr = bases[key] + offset
                self.peer_ptrs[i][j] = addr
        dist.barrier(group=group)  # every rank's signal array is zero before any peer signals
        self.parity = 0

    def next_buffer(self, col_offset: int) -> tuple[torch.Tensor, list[int]]:
        """The buffer of this call and the peers' addresses of element (0, col_offset)."""
        i = self.parity
        self.parity ^= 1
        buf = self.bufs[i]
        off = col_offset * buf.element_size()
        return buf, [self.peer_ptrs[i][j] + off for j in range(self.world) if j != self.rank]

    def signal_ptrs(self) -> tuple[int, list[int]]:
        return self.signals.data_ptr(), [self.peer_ptrs[2][j] for j in range(self.world) if j != self.rank]

    def sync(self, rank: int, world: int, timeout_us: int):
        """The barrier's arguments as one kf_peer_sync struct (built once)."""
        from kernelo_b200.runtime import native

        if self._sync is None:
            local, peers = self.signal_ptrs()
            self._sync = native.peer_sync_struct(local, peers, rank, world, self.counter.data_ptr(),
                                                 self.arrivals.data_ptr(), timeout_us)
        return self._sync

    def barrier(self, rank: int, world: int, timeout_us: int) -> None:
        """Enqueue the bounded barrier; its epoch lives on the device, so a
        CUDA graph that captured it stays correct on every replay."""
        from kernelo_b200.runtime import native

        local, peers = self.signal_ptrs()
        native.peer_barrier_counted(local, peers, rank, world, self.counter.data_ptr(), timeout_us=timeout_us,
                                    device=self.signals.device)

    def close(self) -> None:
        """Unmap the peers' buffers (all ranks should be done with them)."""
        from kernelo_b200.runtime import native

        torch.cuda.synchronize(self.signals.device)
        for base in self._opened:
            native.ipc_close(base)
        self._opened = []


def distributed_tune(tuner, operator, problem, *, device=None, group=None, finalists: int = 3):
    """Tune with the candidate list dealt round-robin over the group's ranks.

    Every rank returns the merged :class:`TuningResult`; only rank 0 persists
    it (the tuner's ``db``/``cache`` are ignored on other ranks). With
    ``resume`` on rank 0's tuner, candidates its database already holds for
    this problem and device are not measured again on any rank. Rank 0 re-times
    its best ``finalists`` candidates locally before ranking, so the winner is
    chosen from measurements taken on one GPU.
    """
    world, rank = world_info(group)
    if world == 1:
        return tuner.tune(operator, problem, device=device)
    db, cache, resume = tuner.db, tuner.cache, tuner.resume
    # Resuming (rank 0's tuner decides, rank 0 being the database's only reader
    # and writer): rank 0 looks up the candidates already measured on this
    # device and tells every rank to skip them; their stored outcomes rejoin
    # the merged list on rank 0.
    reused: dict = {}
    if resume and rank == 0:
        from kernelo_b200.runtime.env import capture_environment, device_caps
        from kernelo_b200.tuning.tuner import _outcome_from_row

        target = torch.device(device) if device is not None else None
        key = capture_environment(target).device_key
        cset = operator.search_space().generate(problem, device_caps(target),
                                                max_candidates=tuner.max_candidates)
        for c in cset.candidates:
            row = db.latest_result(problem, c, device_key=key)
            if row is not None:
                reused[c] = _outcome_from_row(c, row)
    done = [sorted(c.digest for c in reused) if rank == 0 else None]
    dist.broadcast_object_list(done, src=0, group=group)
    skip = set(done[0])
    saved_filter = tuner.candidate_filter
    tuner.db = tuner.cache = None
    tuner.resume = False
    fresh_index: dict = {}

    def deal(i, c):  # round-robin over the candidates not measured yet
        if c.digest in skip:
            return False
        j = fresh_index.setdefault(c.digest, len(fresh_index))
        return j % world == rank

    tuner.candidate_filter = deal
    try:
        local = tuner.tune(operator, problem, device=device)
    finally:
        tuner.candidate_filter = saved_filter
        tuner.db, tuner.cache, tuner.resume = db, cache, resume
    gathered: list = [None] * world
    dist.all_gather_object(gathered, local.outcomes, group=group)
    merged = [o for part in gathered for o in part] + list(reused.values())
    result = replace(local, outcomes=tuple(merged))
    if rank == 0:
        correct = sorted((o for o in merged if o.ok and o.timing is not None), key=lambda o: o.median_ms)
        if correct and finalists > 0:
            retimed = _retime(tuner, operator, problem, [o for o in correct[:finalists]], device)
            keep = {id(o) for o in correct[:finalists]}
            others = [o for o in merged if id(o) not in keep]
            result = replace(result, outcomes=tuple(retimed + others))
        tuner._persist(result, result.environment, skip=set(reused))
    # Every rank returns rank 0's ranking (the one measured on a single GPU).
    final = [result.outcomes if rank == 0 else None]
    dist.broadcast_object_list(final, src=0, group=group)
    return replace(result, outcomes=tuple(final[0]))


def _retime(tuner, operator, problem, outcomes, device):
    target = torch.device(device) if device is not None else None
    inputs = operator.make_inputs(problem, target or torch.device("cuda"), seed=tuner.seed)
    return [tuner._time_candidate(operator, replace(o, timing=None), inputs, target or inputs[0].device)
            for o in outcomes]
