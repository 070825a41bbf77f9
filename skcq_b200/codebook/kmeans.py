"""Lloyd k-means on B200 (interface of skcq/codebook/kmeans.py).

``assign_cosine`` / ``assign_l2`` / ``KmeansExperiment`` keep the reference's
signatures and results; the work runs in the batched device engine (one
problem here) -- tensor-core assignment with the arg-max fused into the
epilogue, segmented-sum update, reseed and finalisation kernels.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from skcq_b200 import _engine
from skcq_b200.codebook.base import DistanceMetric
from skcq_b200.codebook.events import Experiment, KmeansDoneEvent, KmeansIterEvent, KmeansStartEvent

logger = logging.getLogger(__name__)

_METRIC = {"cosine": _engine.COSINE, "euclidean": _engine.L2}


def _single_problem(data: torch.Tensor, raw: torch.Tensor | None, metric: int, dev: torch.device) -> _engine.PointSet:
    """Wrap an (n, d) matrix as a one-problem point set (no zero skipping)."""
    x = _engine.to_device_f32(data, dev)
    n, d = x.shape
    pts = _engine.gather_block_points(x, d, 1, False, 0.0, False, metric)
    if metric == _engine.COSINE and raw is not None:
        r = _engine.to_device_f32(raw, dev)
        rp = _engine.gather_block_points(r, d, 1, False, 0.0, False, _engine.L2)
        pts.R = rp.X
    return pts


def _assign(data: torch.Tensor, centroids: torch.Tensor, metric: int) -> torch.Tensor:
    dev = _engine.cuda_device(centroids.device if centroids.is_cuda else None, data)
    d, k = centroids.shape
    pts = _single_problem(data, None, metric, dev)
    k_pad = _engine.round_up(k, _engine.CENT_TILE)
    C = torch.zeros(1, k_pad, d, dtype=torch.float32, device=dev)
    C[0, :k] = centroids.to(device=dev, dtype=torch.float32).t()
    run = _engine.KmeansRun(C=C, k_pad=k_pad, k_host=[k], labels=None, iters_run=[0], converged=[False],
                            moved=None, n_empty=None,
                            cnorm=torch.empty(1, k_pad, dtype=torch.float32, device=dev))
    labels = _engine.assign(pts, run)
    return labels[0, : data.shape[0]].to(device=data.device, dtype=torch.long)


def assign_cosine(data: torch.Tensor, centroids: torch.Tensor, chunk_size: int, device: torch.device) -> torch.Tensor:
    """Index of the largest ``data @ centroids`` per row (kmeans.py:25-43).

    ``centroids`` is ``(d, k)``. ``chunk_size`` only bounded memory in the
    reference; here the distance matrix never exists, so it is ignored.
    Labels are returned on ``data.device``.
    """
    return _assign(data, centroids, _engine.COSINE)


def assign_l2(data: torch.Tensor, centroids: torch.Tensor, chunk_size: int, device: torch.device) -> torch.Tensor:
    """Index of the smallest ``||c||^2 - 2 data @ centroids`` per row (kmeans.py:46-66)."""
    return _assign(data, centroids, _engine.L2)


def sobol_first_orthant(k: int, d: int, device: torch.device) -> torch.Tensor:
    """k unit directions in the first orthant: scrambled Sobol points (seed 42),
    clamped at 1e-6 and normalised -- the reference's initial centroids
    (kmeans.py:69-74), drawn with torch's own Sobol engine."""
    sobol = torch.quasirandom.SobolEngine(dimension=d, scramble=True, seed=42)
    points = sobol.draw(k).to(device).clamp(min=1e-6)
    return F.normalize(points, dim=-1)


@dataclass
class KmeansConfig:
    """Configuration of one k-means run (kmeans.py:82-92)."""

    metric: DistanceMetric
    k: int
    max_iters: int
    device: torch.device
    name: str
    chunk_size: int
    raw_data: torch.Tensor | None = None
    block_idx: int = 0
    n_blocks: int = 1


def emit_run_events(exp: Experiment, run: _engine.KmeansRun, b: int, name: str, metric: str, max_iters: int,
                    n_points: int, block_idx: int, n_blocks: int) -> None:
    """The Start / Iter* / Done sequence of problem ``b`` (kmeans.py:115-192)."""
    exp._emit(KmeansStartEvent(name=name, metric=metric, k=run.k_host[b], max_iters=max_iters, n_points=n_points,
                               block_idx=block_idx, n_blocks=n_blocks))
    if exp.listens(KmeansIterEvent):  # one event per iteration: built only for a listener
        for it in range(run.iters_run[b]):
            exp._emit(KmeansIterEvent(iter=it, max_iters=max_iters, moved=float(run.moved[it, b]),
                                      n_empty=int(run.n_empty[it, b])))
    exp._emit(KmeansDoneEvent(iters_run=run.iters_run[b], final_moved=run.final_moved(b),
                              converged=run.converged[b]))


class KmeansExperiment(Experiment):
    """One k-means run (kmeans.py:95-259). ``fit(data)`` returns
    ``(centroids (k_eff, d) f32, labels (n,) int64)`` on ``config.device``;
    cosine data is normalised internally and ``config.raw_data`` (if given)
    drives the norm-weighted update."""

    def __init__(self, config: KmeansConfig) -> None:
        super().__init__()
        self.config = config
        self._centroids: torch.Tensor | None = None
        self._labels: torch.Tensor | None = None

    def fit(self, data: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        cfg = self.config
        metric = _METRIC[cfg.metric]
        dev = _engine.cuda_device(cfg.device, data)
        n, d = data.shape
        k_eff = min(cfg.k, n)
        pts = _single_problem(data, cfg.raw_data if metric == _engine.COSINE else None, metric, dev)
        if metric == _engine.COSINE:
            run = _engine.lloyd(pts, cfg.k, cfg.max_iters, init_cosine=lambda kk, dd: sobol_first_orthant(kk, dd, dev))
        else:
            perm = torch.randperm(n, device=data.device)[:k_eff]
            run = _engine.lloyd(pts, cfg.k, cfg.max_iters, init_perms=[perm])
        if n > 0:
            emit_run_events(self, run, 0, cfg.name, cfg.metric, cfg.max_iters, n, cfg.block_idx, cfg.n_blocks)
        out_dev = torch.device(cfg.device) if cfg.device is not None else data.device
        self._centroids = run.C[0, :k_eff].to(out_dev)
        self._labels = run.labels[0, :n].to(device=data.device, dtype=torch.long)
        return self._centroids, self._labels

    @property
    def centroids(self) -> torch.Tensor:
        assert self._centroids is not None, "fit() not called yet"
        return self._centroids

    @property
    def labels(self) -> torch.Tensor:
        assert self._labels is not None, "fit() not called yet"
        return self._labels
