"""Row-sharded codebook fits across ranks (one process per GPU).

A projection's expert-major rows are split into contiguous row ranges, one per
rank in rank order (``expert_row_range``); every rank calls the ordinary
``fit`` on its own rows inside ``with row_sharded(group):``. Each k-means
problem (one per column block) then has its points spread over the ranks:

* assign and the centroid update run locally; the per-iteration centroid sums
  (n_blocks x K x bs f32) and counts (n_blocks x K int32) are summed with one
  ``all_reduce`` each, so every rank finalises identical centroids and all
  ranks stop at the same iteration;
* the empty-cluster reseed gathers every rank's worst-fit candidates
  (``all_gather`` of at most n_empty per problem) and all ranks pick the same
  global worst points, ordered by score and global point index exactly as the
  single-process reseed (kmeans.py:161-172, 219-231);
* Forgy initialisation draws ``randperm(n_global)`` identically on every rank
  (seed every rank the same); the owner of each chosen point contributes it
  and one ``all_reduce`` assembles the initial centroids;
* the spherical negative-scale flip ORs its per-block flags over ranks.

Row-local work (row zero masks, SSVQ signs, scales, residual errors, the
scale re-fit, remainders) needs no communication, so each rank ends with the
CWR of its own rows and the same codebooks as every other rank. Shared
codebooks and training subsamples (``max_train_samples``) are not supported
in this mode and raise.
"""

from __future__ import annotations

from collections.abc import Iterator
from contextlib import contextmanager

import torch
import torch.distributed as dist

INT64_MAX = (1 << 63) - 1

_CURRENT: RowShard | None = None


class RowShard:
    """Collectives of a row-sharded fit over ``group`` (NCCL on GPUs; gloo
    also works, through host copies)."""

    def __init__(self, group: dist.ProcessGroup | None = None) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.host_staged = dist.get_backend(group) == "gloo"

    def _stage(self, t: torch.Tensor) -> torch.Tensor:
        return t.cpu() if self.host_staged and t.is_cuda else t

    def all_reduce_sum_(self, t: torch.Tensor) -> torch.Tensor:
        from skcq_b200._engine import TIMER

        s = self._stage(t)
        # the timer (off unless a benchmark enables it) records the bytes reduced
        TIMER.run("allreduce", lambda: dist.all_reduce(s, op=dist.ReduceOp.SUM, group=self.group),
                  work=float(s.numel() * s.element_size()))
        if s is not t:
            t.copy_(s)
        return t

    def all_reduce_max_(self, t: torch.Tensor) -> torch.Tensor:
        s = self._stage(t)
        dist.all_reduce(s, op=dist.ReduceOp.MAX, group=self.group)
        if s is not t:
            t.copy_(s)
        return t

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        """(world, *t.shape) on t's device."""
        s = self._stage(t.contiguous())
        out = [torch.empty_like(s) for _ in range(self.world)]
        dist.all_gather(out, s, group=self.group)
        return torch.stack(out).to(t.device)


def current() -> RowShard | None:
    """The row-sharding context of the calling thread's fit, if any."""
    return _CURRENT


@contextmanager
def row_sharded(group: dist.ProcessGroup | None = None) -> Iterator[RowShard]:
    """Fits inside this context treat their input rows as this rank's slice of
    a matrix split over ``group`` in rank order."""
    global _CURRENT
    prev = _CURRENT
    _CURRENT = RowShard(group)
    try:
        yield _CURRENT
    finally:
        _CURRENT = prev


def expert_row_range(num_experts: int, out_dim: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [start, end) of rank ``rank``: whole experts, split as evenly as
    possible (the first ``num_experts % world`` ranks get one more)."""
    base, extra = divmod(num_experts, world)
    e0 = rank * base + min(rank, extra)
    e1 = e0 + base + (1 if rank < extra else 0)
    return e0 * out_dim, e1 * out_dim


def global_counts(shard: RowShard, n_local: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(n_global int64 [nblk], gofs int64 [nblk]): points of every problem over
    all ranks, and the global index of this rank's first point."""
    all_n = shard.all_gather(n_local.to(torch.int64))
    return all_n.sum(0), all_n[: shard.rank].sum(0)


def owned_init(X: torch.Tensor, perm: torch.Tensor, k: torch.Tensor, gofs: torch.Tensor,
               n_local: torch.Tensor) -> torch.Tensor:
    """This rank's share of the Forgy centroids ``X_global[b][perm[b][:k[b]]]``:
    rows it owns are copied, others are zero ([nblk, k_pad, bs])."""
    nblk, k_pad = perm.shape
    loc = perm - gofs[:, None]
    cols = torch.arange(k_pad, device=perm.device)[None, :]
    own = (loc >= 0) & (loc < n_local[:, None].to(loc.dtype)) & (cols < k[:, None].to(cols.dtype))
    idx = torch.where(own, loc, torch.zeros_like(loc))
    C = torch.gather(X, 1, idx[..., None].expand(nblk, k_pad, X.shape[2]))
    return C * own[..., None].to(C.dtype)


def empty_clusters(counts: torch.Tensor, k: torch.Tensor, active: torch.Tensor) -> torch.Tensor:
    """Mask [nblk, k_pad] of empty clusters of active problems (global counts)."""
    cols = torch.arange(counts.shape[1], device=counts.device)[None, :]
    return (counts == 0) & (cols < k[:, None].to(cols.dtype)) & (active[:, None] != 0)


def merge_reseed(keys_all: torch.Tensor, vecs_all: torch.Tensor, empty: torch.Tensor, sums: torch.Tensor) -> None:
    """Seed the empty clusters of ``sums`` from the ranks' candidates.

    keys_all [G, nblk, m] int64 (selection order = ascending; padding
    INT64_MAX), vecs_all [G, nblk, m, bs]. The i-th smallest key of problem b
    seeds the i-th empty cluster of b in ascending cluster order."""
    G, nblk, m = keys_all.shape
    bs = vecs_all.shape[-1]
    keys = keys_all.permute(1, 0, 2).reshape(nblk, G * m)
    vecs = vecs_all.permute(1, 0, 2, 3).reshape(nblk, G * m, bs)
    order = torch.argsort(keys, dim=1)
    ranked = torch.gather(vecs, 1, order[..., None].expand(nblk, G * m, bs))
    b_idx, c_idx = empty.nonzero(as_tuple=True)
    if b_idx.numel() == 0:
        return
    pos = (empty.to(torch.int64).cumsum(1) - 1)[b_idx, c_idx]
    sums[b_idx, c_idx] = ranked[b_idx, pos].to(sums.dtype)


def or_over_ranks(shard: RowShard, flags: torch.Tensor) -> torch.Tensor:
    """Bitwise OR of int64 flags over ranks."""
    g = shard.all_gather(flags)
    out = g[0].clone()
    for r in range(1, g.shape[0]):
        out |= g[r]
    return out
