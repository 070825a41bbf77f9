"""AQLM composite on B200 (interface of skcq/codebook/aqlm.py).

primary (spherical, optionally sign-split) + residual chain fitted on the
real error; optional int-N centroid quantisation; full rebuild; least-squares
re-fit of the primary scales. Every error / rebuild is one streaming pass of
the fused multi-codebook decode kernel instead of per-codec, per-block loops.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass

import torch

from skcq_b200 import _engine
from skcq_b200.codebook.base import WeightsCodebookBase
from skcq_b200.codebook.cwr import AQLMCWR, CompressedWeightsRepresentation, SphericalCWR, SSVQCWR, cwr_to
from skcq_b200.codebook.events import (
    CodebookDoneEvent,
    CodebookIterEvent,
    CodebookStartEvent,
    KmeansDoneEvent,
    KmeansIterEvent,
    KmeansStartEvent,
)
from skcq_b200.codebook.spherical import SphericalCodebook
from skcq_b200.codebook.ssvq import SSVQCodebook

logger = logging.getLogger(__name__)


@dataclass
class AQLMCodebookConfig:
    """aqlm.py:24-38 (same fields and defaults)."""

    codebook_bits: int = 16
    norm_threshold: float = 0.001
    device: torch.device | None = None
    out_dim: int | None = None
    num_experts: int | None = None


class AQLMCodebook(WeightsCodebookBase[AQLMCWR]):
    """Primary + residual composite (aqlm.py:40-246)."""

    def __init__(
        self,
        primary: WeightsCodebookBase,
        residuals: list[WeightsCodebookBase],
        config: AQLMCodebookConfig | None = None,
    ) -> None:
        super().__init__()
        self.primary = primary
        self.residuals = residuals
        self.config = config or AQLMCodebookConfig()

    def _all(self) -> list[WeightsCodebookBase]:
        return [self.primary, *self.residuals]

    def fit(self, w: torch.Tensor) -> AQLMCWR:
        """aqlm.py:67-135."""
        cfg = self.config
        out_dev = torch.device(cfg.device) if cfg.device is not None else w.device
        dev = _engine.cuda_device(cfg.device, w)
        n_rows, in_dim = w.shape
        raw = _engine.to_device_f32(w, dev)
        zero_mask = _engine.row_zero_mask(raw, cfg.norm_threshold)
        if logger.isEnabledFor(logging.INFO):
            logger.info("AQLM: %d/%d rows below norm threshold %s", int(zero_mask.sum()), n_rows, cfg.norm_threshold)
        n_codebooks = 1 + len(self.residuals)
        sph, _, _ = self._unwrap_spherical_primary()
        self._emit(CodebookStartEvent(
            n_codebooks=n_codebooks,
            primary_block_size=getattr(self.primary, "block_size", 0),
            primary_k=getattr(self.primary, "K", 0),
            metric="cosine" if sph is not None else "euclidean",
        ))
        # 1. primary
        self._wire_child_events(self.primary, 0, n_codebooks)
        primary_cwr = self.primary.fit(raw)
        self._emit(CodebookDoneEvent(codebook_idx=0, n_codebooks=n_codebooks))
        views = self.primary.views(primary_cwr, dev)
        # 2. residual chain on the real error: error = raw - (p + r1 + ...)
        res_cwrs: list[CompressedWeightsRepresentation] = []
        for i, res_cb in enumerate(self.residuals):
            error = _engine.reconstruct(views, n_rows, in_dim, raw=raw)
            self._wire_child_events(res_cb, i + 1, n_codebooks)
            res_cwr = res_cb.fit(error)
            del error
            res_cwrs.append(res_cwr)
            self._emit(CodebookDoneEvent(codebook_idx=i + 1, n_codebooks=n_codebooks))
            views = views + res_cb.views(res_cwr, dev)
        # 3. centroid quantisation
        if cfg.codebook_bits < 16:
            for cb in self._all():
                cb.quantize_centroids(cfg.codebook_bits)
            logger.info("AQLM: quantized centroids to int%d", cfg.codebook_bits)
        # 4 + 5. rebuild with the final centroids, then the LS primary scale re-fit
        sph, sph_cwr, _ = self._unwrap_spherical_primary_from_cwr(primary_cwr)
        if sph is not None and sph_cwr is not None:
            views = self.primary.views(primary_cwr, dev)
            for res_cb, rc in zip(self.residuals, res_cwrs, strict=True):
                views = views + res_cb.views(rc, dev)
            recon = _engine.reconstruct(views, n_rows, in_dim)
            scales = sph_cwr.scales
            if scales.dtype != torch.float32 or not scales.is_cuda:
                raise RuntimeError("primary scales must be f32 on the device during fit")
            _engine.refit_scales(views[0], raw, recon, zero_mask, scales)
        out = AQLMCWR(primary=primary_cwr, residuals=res_cwrs)
        return out if out_dev.type == "cuda" else cwr_to(out, out_dev)

    def views(self, cwr: AQLMCWR, dev: torch.device) -> list[_engine.CodecView]:
        v = self.primary.views(cwr.primary, dev)
        for res_cb, rc in zip(self.residuals, cwr.residuals, strict=True):
            v = v + res_cb.views(rc, dev)
        return v

    def reconstruct(self, cwr: AQLMCWR) -> torch.Tensor:
        """aqlm.py:137-141 as one fused decode pass."""
        first = cwr.primary.inner if isinstance(cwr.primary, SSVQCWR) else cwr.primary
        out_dev = first.idxs.device
        dev = _engine.cuda_device(None, first.idxs)
        v = self.views(cwr, dev)
        n_rows = first.idxs.shape[1]
        in_dim = v[0].n_blocks * v[0].bs + (v[0].rem.shape[1] if v[0].rem is not None else 0)
        return _engine.reconstruct(v, n_rows, in_dim).to(out_dev)

    def quantize_centroids(self, bits: int) -> None:
        for cb in self._all():
            cb.quantize_centroids(bits)

    def _unwrap_spherical_primary(self):
        """aqlm.py:258-271."""
        if isinstance(self.primary, SSVQCodebook):
            if isinstance(self.primary.inner, SphericalCodebook):
                return self.primary.inner, None, None
        elif isinstance(self.primary, SphericalCodebook):
            return self.primary, None, None
        return None, None, None

    def _unwrap_spherical_primary_from_cwr(self, primary_cwr):
        """aqlm.py:273-285."""
        if isinstance(self.primary, SSVQCodebook):
            inner = self.primary.inner
            if isinstance(inner, SphericalCodebook) and isinstance(primary_cwr, SSVQCWR):
                return inner, primary_cwr.inner, primary_cwr.signs
        elif isinstance(self.primary, SphericalCodebook) and isinstance(primary_cwr, SphericalCWR):
            return self.primary, primary_cwr, None
        return None, None, None

    def _wire_child_events(self, child: WeightsCodebookBase, codebook_idx: int, n_codebooks: int) -> None:
        """aqlm.py:291-319: forward Start/Done, wrap Iter into CodebookIterEvent
        (with the reference's fixed block_idx 0 / n_blocks 1), forward Iter."""
        self._forward_from(child, KmeansStartEvent)
        self._forward_from(child, KmeansDoneEvent)
        metric = "cosine" if isinstance(child, (SphericalCodebook, SSVQCodebook)) else "euclidean"

        def wrap_iter(e: KmeansIterEvent) -> None:
            self._emit(CodebookIterEvent(
                codebook_idx=codebook_idx, n_codebooks=n_codebooks, block_idx=0, n_blocks=1, iter=e.iter,
                max_iters=e.max_iters, moved=e.moved, n_empty=e.n_empty, metric=metric,
            ))

        child.on(KmeansIterEvent, wrap_iter, when=lambda: self.listens(CodebookIterEvent))
        self._forward_from(child, KmeansIterEvent)
