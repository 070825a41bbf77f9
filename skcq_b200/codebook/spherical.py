"""Spherical (cosine) codec on B200 (interface of skcq/codebook/spherical.py).

Unit-norm directions per block, a per-(row, block) scale = <raw block,
direction>, a raw bf16 remainder for the columns no block covers.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass

import torch

from skcq_b200 import _engine, distributed
from skcq_b200._lib import call, ptr, stream
from skcq_b200.codebook._blockfit import fit_blocks, stacked_centroids
from skcq_b200.codebook.base import WeightsCodebookBase
from skcq_b200.codebook.cwr import SphericalCWR
from skcq_b200.codebook.events import Experiment

logger = logging.getLogger(__name__)

_FP8_MAP = {"fp8_e4m3": torch.float8_e4m3fn, "fp8_e5m2": torch.float8_e5m2}


@dataclass
class ScaleQuantState:
    """How stored scales decode to f32 (spherical.py:33-42): a plain cast for
    bf16/fp16/fp8, ``q * q_scale`` for int<N>."""

    scale_dtype: str = "bf16"
    q_scale: torch.Tensor | None = None


def quantize_spherical_scales(cwr: SphericalCWR, cb: SphericalCodebook, scale_dtype: str) -> None:
    """Quantise ``cwr.scales`` in place and record the decode state on ``cb``
    (spherical.py:45-71). int<N>: one global abs-max scale, round half to even."""
    scales = cwr.scales.float()
    if scale_dtype == "bf16":
        cwr.scales = scales.to(torch.bfloat16)
        cb.scale_quant = ScaleQuantState(scale_dtype="bf16")
    elif scale_dtype == "fp16":
        cwr.scales = scales.to(torch.float16)
        cb.scale_quant = ScaleQuantState(scale_dtype="fp16")
    elif scale_dtype in _FP8_MAP:
        cwr.scales = scales.to(_FP8_MAP[scale_dtype])
        cb.scale_quant = ScaleQuantState(scale_dtype=scale_dtype)
    elif scale_dtype.startswith("int"):
        bits = int(scale_dtype[3:])
        out_dev = scales.device
        dev = _engine.cuda_device(None, scales)
        q, q_scale = _engine.quantize_scales_int(scales.to(dev), bits)
        cb.scale_quant = ScaleQuantState(scale_dtype=scale_dtype, q_scale=q_scale.to(out_dev))
        if q is not None:
            cwr.scales = q.to(out_dev)
    else:
        raise ValueError(f"Unknown scale dtype: {scale_dtype}")


def scale_bits_per_elem(dtype: str) -> int:
    """Storage bits of one scale (spherical.py:74-81)."""
    if dtype.startswith("int"):
        return int(dtype[3:])
    if dtype in _FP8_MAP:
        return 8
    if dtype in ("fp16", "bf16"):
        return 16
    raise ValueError(f"Unknown scale dtype: {dtype}")


def parse_scale_dtype(s: str) -> str:
    """Validate a scale dtype name (spherical.py:84-95)."""
    s = s.strip().lower()
    if s.startswith("int"):
        bits = int(s[3:])
        if bits < 2 or bits > 16:
            raise ValueError(f"int bits must be 2-16, got {bits}")
        return s
    if s in ("fp16", "bf16") or s in _FP8_MAP:
        return s
    raise ValueError(f"Unknown scale dtype '{s}'")


@dataclass
class SphericalCodebookConfig:
    """spherical.py:103-120 (same fields and defaults)."""

    block_size: int
    K: int
    shared: bool = False
    max_iters: int = 100
    norm_threshold: float = 0.001
    skip_zeros: bool = True
    chunk_budget_mb: int = 2048
    device: torch.device | None = None
    max_train_samples: int = 0
    scale_dtype: str = "bf16"


def _cuda_view(t: torch.Tensor | None, dev: torch.device) -> torch.Tensor | None:
    return None if t is None else t.to(dev)


class SphericalCodebook(WeightsCodebookBase[SphericalCWR], Experiment):
    """Spherical codec with per-block (or shared) unit directions."""

    def __init__(self, config: SphericalCodebookConfig) -> None:
        Experiment.__init__(self)
        self.config = config
        self.directions: torch.Tensor | None = None  # (n_blocks | 1, bs, K) bf16
        self.block_size = config.block_size
        self.shared = config.shared
        self.K = config.K
        self.scale_quant = ScaleQuantState(scale_dtype="bf16")

    def fit(self, w: torch.Tensor) -> SphericalCWR:
        """spherical.py:140-190 on the device engine."""
        cfg = self.config
        out_dev = torch.device(cfg.device) if cfg.device is not None else w.device
        dev = _engine.cuda_device(cfg.device, w)
        n_rows, in_dim = w.shape
        bs = cfg.block_size
        n_blocks = in_dim // bs
        cov = n_blocks * bs
        raw = _engine.to_device_f32(w, dev)
        row_zero = _engine.row_zero_mask(raw, cfg.norm_threshold)
        fit = fit_blocks(
            self, raw, metric=_engine.COSINE, bs=bs, K=cfg.K, shared=cfg.shared, max_iters=cfg.max_iters,
            norm_threshold=cfg.norm_threshold, skip_zeros=cfg.skip_zeros,
            max_train_samples=cfg.max_train_samples, name="spherical",
        )
        if fit.run is not None:
            self._flip_negative(fit, bs)
            scales = torch.empty(n_rows, n_blocks, dtype=torch.float32, device=dev)
            call("skcq_spherical_scales", ptr(raw), raw.stride(0), n_rows, bs, n_blocks, int(cfg.shared),
                 ptr(fit.run.C), fit.run.k_pad, ptr(fit.idxs), ptr(row_zero), ptr(scales), stream())
        else:
            scales = torch.zeros(n_rows, n_blocks, dtype=torch.float32, device=dev)
        remainder = _engine.remainder_bf16(raw, cov)
        self.directions = stacked_centroids(fit, bs).to(out_dev)
        return SphericalCWR(
            idxs=fit.idxs.to(out_dev), scales=scales.to(out_dev),
            remainder=remainder.to(out_dev) if remainder is not None else None,
        )

    def _flip_negative(self, fit, bs: int) -> None:
        """spherical.py:289-299: negate centroid *dimensions* named by labels of
        points whose scale is negative; a label >= bs is an IndexError there."""
        pts, run = fit.pts, fit.run
        flags = torch.empty(pts.nblk, dtype=torch.int64, device=run.C.device)
        call("skcq_flip_check", ptr(pts.R), ptr(run.C), ptr(fit.labels), pts.nblk, pts.n_pad, run.k_pad, bs,
             ptr(pts.n), ptr(flags), stream())
        shard = distributed.current()
        if shard is not None:  # the flip names labels of any rank's points
            flags = distributed.or_over_ranks(shard, flags)
        host = [int(v) & 0xFFFFFFFFFFFFFFFF for v in flags.cpu().tolist()]
        if any(h >> 63 for h in host):
            raise IndexError(f"index out of range in the negative-scale flip: a label >= block size {bs}")
        if any(host):
            for b, h in enumerate(host):
                if h:
                    logger.info("[spherical blk=%d] flipped %d/%d centroids", b, bin(h).count("1"), run.k_host[b])
            call("skcq_apply_flip", ptr(flags), pts.nblk, run.k_pad, bs, ptr(run.C), stream())

    def views(self, cwr: SphericalCWR, dev: torch.device) -> list[_engine.CodecView]:
        """Device view of this codec and ``cwr`` for the fused decode."""
        assert self.directions is not None, "fit() not called yet"
        cent = self.directions
        if cent.dtype != torch.bfloat16:
            raise TypeError("spherical directions must be bf16 (as stored after fit)")
        idxs = cwr.idxs.to(dev)
        if idxs.dim() == 2 and idxs.shape[0] > 0 and idxs.stride(1) != 1:
            idxs = idxs.contiguous()
        scales, q_scale = self._scales_for_decode(cwr.scales, dev)
        rem = cwr.remainder.to(dev).contiguous() if cwr.remainder is not None else None
        return [_engine.CodecView(
            kind=0, bs=self.block_size, n_blocks=idxs.shape[0], K=cent.shape[-1], shared=self.shared,
            cent=cent.to(dev).contiguous(), idxs=idxs, scales=scales, q_scale=q_scale, rem=rem,
        )]

    def _scales_for_decode(self, scales: torch.Tensor, dev: torch.device) -> tuple[torch.Tensor, float]:
        """spherical.py:213-223 ``_dequant_scales`` as (tensor, multiplier)."""
        sq = self.scale_quant
        s = scales.to(dev)
        if sq.scale_dtype.startswith("int") and not s.is_floating_point():
            assert sq.q_scale is not None
            return s.contiguous(), float(sq.q_scale)
        if s.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            s = s.float()
        if s.stride(-1) != 1:
            s = s.contiguous()
        return s, 1.0

    def reconstruct(self, cwr: SphericalCWR) -> torch.Tensor:
        """spherical.py:192-211: ``(n_rows, in_dim)`` f32 on ``cwr.idxs.device``."""
        out_dev = cwr.idxs.device
        dev = _engine.cuda_device(None, cwr.idxs)
        v = self.views(cwr, dev)
        n_rows = cwr.idxs.shape[1]
        in_dim = v[0].n_blocks * v[0].bs + (v[0].rem.shape[1] if v[0].rem is not None else 0)
        return _engine.reconstruct(v, n_rows, in_dim).to(out_dev)

    def quantize_centroids(self, bits: int) -> None:
        """spherical.py:306-315: int<bits> fake quantisation, one scale per
        centroid index shared by all blocks and dimensions."""
        if bits >= 16 or self.directions is None:
            return
        out_dev = self.directions.device
        dev = _engine.cuda_device(None, self.directions)
        cb = self.directions.to(device=dev, dtype=torch.bfloat16).contiguous().clone()
        _engine.quantize_centroids_(cb, bits)
        self.directions = cb.to(out_dev)

    @property
    def centroids_tensor(self) -> torch.Tensor:
        assert self.directions is not None, "fit() not called yet"
        return self.directions
