"""Euclidean (l2) codec on B200 (interface of skcq/codebook/euclidean.py).

Per-block (or shared) centroids that carry magnitude; a raw bf16 remainder
for the columns no block covers.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass

import torch

from skcq_b200 import _engine
from skcq_b200.codebook._blockfit import fit_blocks, stacked_centroids
from skcq_b200.codebook.base import WeightsCodebookBase
from skcq_b200.codebook.cwr import EuclideanCWR
from skcq_b200.codebook.events import Experiment

logger = logging.getLogger(__name__)


@dataclass
class EuclideanCodebookConfig:
    """euclidean.py:18-33 (same fields and defaults)."""

    block_size: int
    K: int
    shared: bool = False
    max_iters: int = 100
    norm_threshold: float = 0.001
    skip_zeros: bool = True
    chunk_budget_mb: int = 2048
    device: torch.device | None = None
    max_train_samples: int = 0


class EuclideanCodebook(WeightsCodebookBase[EuclideanCWR], Experiment):
    """Euclidean codec: reconstruction is a direct centroid lookup."""

    def __init__(self, config: EuclideanCodebookConfig) -> None:
        Experiment.__init__(self)
        self.config = config
        self.centroids: torch.Tensor | None = None  # (n_blocks | 1, bs, K) bf16
        self.block_size = config.block_size
        self.shared = config.shared
        self.K = config.K

    def fit(self, w: torch.Tensor) -> EuclideanCWR:
        """euclidean.py:55-101 on the device engine."""
        cfg = self.config
        out_dev = torch.device(cfg.device) if cfg.device is not None else w.device
        dev = _engine.cuda_device(cfg.device, w)
        bs = cfg.block_size
        n_blocks = w.shape[1] // bs
        raw = _engine.to_device_f32(w, dev)
        fit = fit_blocks(
            self, raw, metric=_engine.L2, bs=bs, K=cfg.K, shared=cfg.shared, max_iters=cfg.max_iters,
            norm_threshold=cfg.norm_threshold, skip_zeros=cfg.skip_zeros,
            max_train_samples=cfg.max_train_samples, name="euclidean",
        )
        remainder = _engine.remainder_bf16(raw, n_blocks * bs)
        self.centroids = stacked_centroids(fit, bs).to(out_dev)
        return EuclideanCWR(idxs=fit.idxs.to(out_dev), remainder=remainder.to(out_dev) if remainder is not None else None)

    def views(self, cwr: EuclideanCWR, dev: torch.device) -> list[_engine.CodecView]:
        assert self.centroids is not None, "fit() not called yet"
        cent = self.centroids
        if cent.dtype != torch.bfloat16:
            raise TypeError("euclidean centroids must be bf16 (as stored after fit)")
        idxs = cwr.idxs.to(dev)
        if idxs.dim() == 2 and idxs.shape[0] > 0 and idxs.stride(1) != 1:
            idxs = idxs.contiguous()
        rem = cwr.remainder.to(dev).contiguous() if cwr.remainder is not None else None
        return [_engine.CodecView(
            kind=1, bs=self.block_size, n_blocks=idxs.shape[0], K=cent.shape[-1], shared=self.shared,
            cent=cent.to(dev).contiguous(), idxs=idxs, rem=rem,
        )]

    def reconstruct(self, cwr: EuclideanCWR) -> torch.Tensor:
        """euclidean.py:103-120: ``(n_rows, in_dim)`` f32 on ``cwr.idxs.device``."""
        out_dev = cwr.idxs.device
        dev = _engine.cuda_device(None, cwr.idxs)
        v = self.views(cwr, dev)
        n_rows = cwr.idxs.shape[1]
        in_dim = v[0].n_blocks * v[0].bs + (v[0].rem.shape[1] if v[0].rem is not None else 0)
        return _engine.reconstruct(v, n_rows, in_dim).to(out_dev)

    def quantize_centroids(self, bits: int) -> None:
        """euclidean.py:186-195 (same scheme as the spherical codec)."""
        if bits >= 16 or self.centroids is None:
            return
        out_dev = self.centroids.device
        dev = _engine.cuda_device(None, self.centroids)
        cb = self.centroids.to(device=dev, dtype=torch.bfloat16).contiguous().clone()
        _engine.quantize_centroids_(cb, bits)
        self.centroids = cb.to(out_dev)

    @property
    def centroids_tensor(self) -> torch.Tensor:
        assert self.centroids is not None, "fit() not called yet"
        return self.centroids
