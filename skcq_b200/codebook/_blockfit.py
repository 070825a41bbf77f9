"""Per-block k-means of a weight matrix, batched over all blocks.

Shared by the spherical and euclidean codecs: the reference's
``for b in range(n_blocks): _cluster_block(raw[:, b*bs:(b+1)*bs])`` loop
(skcq/codebook/spherical.py:162-176, euclidean.py:401-415) becomes one
problem set whose blocks iterate together on the device.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from skcq_b200 import _engine, distributed
from skcq_b200.codebook.events import Experiment
from skcq_b200.codebook.kmeans import emit_run_events, sobol_first_orthant


@dataclass
class BlockFit:
    pts: _engine.PointSet  # every non-zero point (the final assignment set)
    run: _engine.KmeansRun | None  # None when no block has points
    labels: torch.Tensor  # int32 [nblk, n_pad] labels of `pts`
    idxs: torch.Tensor  # int64 (n_blocks, n_rows)
    k_cent: int  # centroids per block in the stacked codebook tensor


def fit_blocks(
    owner: Experiment,
    raw: torch.Tensor,
    *,
    metric: int,
    bs: int,
    K: int,
    shared: bool,
    max_iters: int,
    norm_threshold: float,
    skip_zeros: bool,
    max_train_samples: int,
    name: str,
) -> BlockFit:
    """Cluster every block of ``raw`` (f32, CUDA, row-major) and emit each
    block's k-means events from ``owner`` in block order."""
    dev = raw.device
    n_rows, in_dim = raw.shape
    n_blocks = in_dim // bs
    shard = distributed.current()
    if shard is not None and shared:
        raise NotImplementedError("row-sharded fits support per-block codebooks only (shared=False)")
    pts = _engine.gather_block_points(raw, bs, n_blocks, shared, norm_threshold, skip_zeros, metric)
    nblk = pts.nblk
    n_global = gofs = None
    n_all = pts.n_host
    if shard is not None:
        n_global, gofs = distributed.global_counts(shard, pts.n)
        n_all = [int(v) for v in n_global.tolist()]
    # Centroid count each block would stack (spherical.py:250-256, euclidean.py:462-468):
    # empty blocks give min(K, 1) (spherical) or K (euclidean) zero centroids.
    empty_k = min(K, 1) if metric == _engine.COSINE else K
    k_each = [min(K, nb) if nb > 0 else empty_k for nb in n_all]
    if len(set(k_each)) != 1:
        raise RuntimeError(
            f"stack expects each tensor to be equal size, but blocks have {sorted(set(k_each))} centroids"
        )
    k_cent = k_each[0]
    # Random draws in the reference's order: per block, the training subsample
    # permutation (if any) and then the Forgy permutation (euclidean only).
    sub_perms: list[torch.Tensor | None] = []
    init_perms: list[torch.Tensor | None] = []
    any_sub = False
    for nb in n_all:
        sp = None
        if nb > 0 and max_train_samples > 0 and nb > max_train_samples:
            if shard is not None:
                raise NotImplementedError("row-sharded fits do not subsample (max_train_samples)")
            sp = torch.randperm(nb, device=dev)
            any_sub = True
        sub_perms.append(sp)
        n_train = min(nb, max_train_samples) if sp is not None else nb
        if metric == _engine.L2 and nb > 0:
            init_perms.append(torch.randperm(n_train, device=dev))
        else:
            init_perms.append(None)
    train = _engine.subsample_points(raw, bs, n_blocks, shared, pts, sub_perms, max_train_samples) if any_sub else pts
    if max(n_all) == 0:
        run = None
        labels = torch.zeros(nblk, pts.n_pad, dtype=torch.int32, device=dev)
    else:
        run = _engine.lloyd(
            train, K, max_iters,
            init_cosine=lambda k, d: sobol_first_orthant(k, d, dev),
            init_perms=init_perms, shard=shard, n_global=n_global, gofs=gofs,
        )
        labels = _engine.assign(pts, run) if any_sub else run.labels
        metric_name = "cosine" if metric == _engine.COSINE else "euclidean"
        n_train = n_all if shard is not None else train.n_host
        for b in range(nblk):
            if n_all[b] == 0:
                continue
            emit_run_events(
                owner, run, b,
                name if shared else f"{name} blk={b}",
                metric_name, max_iters, n_train[b],
                0 if shared else b, 1 if shared else n_blocks,
            )
    idxs = _engine.scatter_labels(pts, labels, shared, n_rows, n_blocks)
    return BlockFit(pts=pts, run=run, labels=labels, idxs=idxs, k_cent=k_cent)


def stacked_centroids(fit: BlockFit, bs: int) -> torch.Tensor:
    """(n_blocks | 1, bs, K) bf16 codebook tensor; empty blocks stay zero."""
    nblk = fit.pts.nblk
    if fit.run is None:
        return torch.zeros(nblk, bs, fit.k_cent, dtype=torch.bfloat16, device=fit.idxs.device)
    return _engine.centroids_bf16(fit.run.C, fit.run.k_pad, bs, fit.k_cent)
