"""Multi-GPU partitioning of the hot path (one process per GPU, torch.distributed).

Three shardings, each where the work splits naturally:

* :class:`ShardedFusedLinear` -- the fused linear is column-sharded by N: rank r
  holds rows [r*chunk, (r+1)*chunk) of the [N, K] weight and of the bias,
  computes its [M, chunk] slice of ``gelu(x @ W^T + b)`` with the native
  kernel, and the slices are exchanged with one NCCL ``all_gather_into_tensor``
  over NVLink. N is padded to ``world * chunk`` with zero weight rows (their
  columns are dropped), since the collective needs equal chunks.
* :func:`row_range` -- softmax / RMSNorm rows split evenly; no exchange.
* :func:`distributed_tune` -- the tuner's budgeted candidates dealt round-robin
  to one worker per GPU; outcomes are gathered on rank 0, which alone writes
  the database and the cache, after re-timing the finalists on its own GPU
  (timings from different GPUs are never ranked against each other).

The reference has no multi-GPU code; this module is new. No TMA multicast is
used anywhere (the collective is NCCL's).
"""

from __future__ import annotations

from dataclasses import replace

import torch
import torch.distributed as dist

from kernelo_b200.kernels.fused_linear import fused_linear_gelu


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
    ) -> None:
        self.group = group
        self.world, self.rank = world_info(group)
        self.approximate = approximate
        self.config = config
        if shard_weight is not None:
            if out_features is None or shard_bias is None:
                raise ValueError("shard_weight needs out_features and shard_bias")
            self.n = out_features
            self.chunk = shard_weight.shape[0]
            self.w = shard_weight
            self.b = shard_bias
        else:
            if weight is None or bias is None:
                raise ValueError("pass weight and bias, or shard_weight and shard_bias")
            self.n = weight.shape[0]
            self.chunk = shard_chunk(self.n, self.world)
            start = self.rank * self.chunk
            stop = min(self.n, start + self.chunk)
            k = weight.shape[1]
            w = torch.zeros(self.chunk, k, device=weight.device, dtype=weight.dtype)
            b = torch.zeros(self.chunk, device=bias.device, dtype=bias.dtype)
            if stop > start:
                w[: stop - start].copy_(weight[start:stop])
                b[: stop - start].copy_(bias[start:stop])
            self.w, self.b = w, b
        self._gather_buf: torch.Tensor | None = None

    def local(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's [M, chunk] slice of the output."""
        return fused_linear_gelu(x, self.w.t(), self.b, approximate=self.approximate,
                                 config=self.config, out=out)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        m = x.shape[0]
        if self.world == 1:
            return self.local(x)[:, : self.n]
        if self._gather_buf is None or self._gather_buf.shape != (self.world, m, self.chunk):
            self._gather_buf = torch.empty(self.world, m, self.chunk, device=x.device, dtype=x.dtype)
        mine = self._gather_buf[self.rank]
        self.local(x, out=mine)
        dist.all_gather_into_tensor(self._gather_buf.view(-1), mine.reshape(-1), group=self.group)
        full = self._gather_buf.permute(1, 0, 2).reshape(m, self.world * self.chunk)
        return full[:, : self.n]


def distributed_tune(tuner, operator, problem, *, device=None, group=None, finalists: int = 3):
    """Tune with the candidate list dealt round-robin over the group's ranks.

    Every rank returns the merged :class:`TuningResult`; only rank 0 persists
    it (the tuner's ``db``/``cache`` are ignored on other ranks). Rank 0 re-times
    its best ``finalists`` candidates locally before ranking, so the winner is
    chosen from measurements taken on one GPU.
    """
    world, rank = world_info(group)
    if world == 1:
        return tuner.tune(operator, problem, device=device)
    db, cache = tuner.db, tuner.cache
    saved_filter = tuner.candidate_filter
    tuner.db = tuner.cache = None
    tuner.candidate_filter = lambda i, c: i % world == rank
    try:
        local = tuner.tune(operator, problem, device=device)
    finally:
        tuner.candidate_filter = saved_filter
        tuner.db, tuner.cache = db, cache
    gathered: list = [None] * world
    dist.all_gather_object(gathered, local.outcomes, group=group)
    merged = [o for part in gathered for o in part]
    result = replace(local, outcomes=tuple(merged))
    if rank == 0:
        correct = sorted((o for o in merged if o.ok and o.timing is not None), key=lambda o: o.median_ms)
        if correct and finalists > 0:
            retimed = _retime(tuner, operator, problem, [o for o in correct[:finalists]], device)
            keep = {id(o) for o in correct[:finalists]}
            others = [o for o in merged if id(o) not in keep]
            result = replace(result, outcomes=tuple(retimed + others))
        tuner._persist(result, result.environment)
    # Every rank returns rank 0's ranking (the one measured on a single GPU).
    final = [result.outcomes if rank == 0 else None]
    dist.broadcast_object_list(final, src=0, group=group)
    return replace(result, outcomes=tuple(final[0]))


def _retime(tuner, operator, problem, outcomes, device):
    target = torch.device(device) if device is not None else None
    inputs = operator.make_inputs(problem, target or torch.device("cuda"), seed=tuner.seed)
    return [tuner._time_candidate(operator, replace(o, timing=None), inputs, target or inputs[0].device)
            for o in outcomes]
