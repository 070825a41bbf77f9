"""One sweep configuration on the B200 codebooks (interface of
skcq/vq/experiment.py:37-307, ``VQRunExperiment``).

``VQRunExperiment(config).fit(W)`` builds the configuration's AQLM codebook
(spherical or euclidean primary, optionally sign-split and shared; euclidean
residuals with per-codebook K, block size and sign split; centroid bits),
fits it on the GPU, quantises the primary scales to ``scale_dtype``, and
returns the reference's result row: scheme label, rel_fro_err, bits per
weight, compression ratio and the configuration fields. The same events are
forwarded (codebook and k-means start / iter / done) and ``VQStartEvent`` /
``VQDoneEvent`` bracket the run. The TCP progress listener of the reference's
sweep workers is not part of this package.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass

import torch

from skcq_b200.codebook.aqlm import AQLMCodebook
from skcq_b200.codebook.base import DistanceMetric
from skcq_b200.codebook.cwr import SSVQCWR, SphericalCWR
from skcq_b200.codebook.events import (
    CodebookDoneEvent,
    CodebookIterEvent,
    CodebookStartEvent,
    Experiment,
    KmeansDoneEvent,
    KmeansIterEvent,
    KmeansStartEvent,
)
from skcq_b200.codebook.spherical import SphericalCodebook, quantize_spherical_scales, scale_bits_per_elem
from skcq_b200.codebook.ssvq import SSVQCodebook
from skcq_b200.config import CodecSpec, _per_codebook, _resolve_residual_ss, assemble_aqlm
from skcq_b200.vq.bpw import bits_per_weight_kmeans

logger = logging.getLogger(__name__)


@dataclass
class VQStartEvent:
    config_id: str
    projection: str
    block_size: int
    K: int
    n_codebooks: int
    metric: DistanceMetric


@dataclass
class VQDoneEvent:
    config_id: str
    row: dict


@dataclass
class VQRunConfig:
    """experiment.py:53-77 (same fields and meaning)."""

    projection: str
    in_dim: int
    num_experts: int
    hidden_size: int
    intermediate_size: int
    block_size: int
    K: int
    n_codebooks: int
    metric: DistanceMetric
    residual_k: int | list[int] | None
    residual_sign_split: bool | list[bool] | None
    shared_codebook: bool
    sign_split: bool
    max_iters: int
    scale_dtype: str
    residual_block_sizes: int | list[int] | None
    codebook_bits: int
    layer_idx: int
    device: torch.device
    chunk_budget_mb: int
    primary_codebook_cache: object | None = None
    cache_key_str: str | None = None


_CHILD_EVENTS = (CodebookStartEvent, CodebookIterEvent, CodebookDoneEvent, KmeansStartEvent, KmeansIterEvent,
                 KmeansDoneEvent)
_NORM_THRESHOLD = 0.001  # the sweep's zero-block threshold (experiment.py:181)
_SHARED_TRAIN_SAMPLES = 1 << 23  # training subsample of a shared primary (experiment.py:183)


@dataclass(frozen=True)
class _Plan:
    """What one sweep configuration fits: per-codebook specs (primary first)
    and the figures its result row reports."""

    specs: list[CodecSpec]
    label: str
    config_id: str
    out_dim: int

    @property
    def block_sizes(self) -> list[int]:
        return [sp.block_size for sp in self.specs]

    @property
    def ks(self) -> list[int]:
        return [sp.K for sp in self.specs]

    @property
    def residual_sign_split(self) -> list[bool]:
        return [sp.sign_split for sp in self.specs[1:]]


def _plan(cfg: VQRunConfig) -> _Plan:
    """Per-codebook block sizes, K and sign splits of a configuration. The
    primary takes the configuration's own values; a residual takes its entry of
    a per-codebook list, else the shared scalar, else the primary's. A zero
    residual K means "same as the primary". Only a spherical primary is
    sign-split; it alone skips zero blocks and subsamples when shared."""
    n = cfg.n_codebooks
    res_k = cfg.residual_k if isinstance(cfg.residual_k, list) else (cfg.residual_k or None)
    ks = _per_codebook(res_k, cfg.K, n)
    bss = _per_codebook(cfg.residual_block_sizes, cfg.block_size, n)
    res_ss = _resolve_residual_ss(cfg.residual_sign_split, n - 1)
    cosine = cfg.metric == "cosine"
    specs = [CodecSpec(cfg.metric, cfg.block_size, cfg.K, sign_split=cosine and cfg.sign_split, skip_zeros=True,
                       shared=cfg.shared_codebook,
                       max_train_samples=_SHARED_TRAIN_SAMPLES if cfg.shared_codebook else 0)]
    specs += [CodecSpec("euclidean", bss[c], ks[c], sign_split=res_ss[c - 1], skip_zeros=False,
                        shared=cfg.shared_codebook) for c in range(1, n)]
    # scheme label: the reference's naming, which sweep tables key on
    parts = "-".join(f"cb{c}_b{sp.block_size}k{sp.K}" for c, sp in enumerate(specs))
    tags = [cfg.metric[:3], "shared" if cfg.shared_codebook else "perblock", "ssvq" if cfg.sign_split else "nosign"]
    label = f"kmeans_{parts}_" + "_".join(tags)
    if cfg.scale_dtype != "bf16":
        label += f"_{cfg.scale_dtype}"
    if cfg.codebook_bits < 16:
        label += f"_cb{cfg.codebook_bits}"
    out_dim = cfg.hidden_size if cfg.projection == "down" else cfg.intermediate_size
    return _Plan(specs, label, f"L{cfg.layer_idx}.{cfg.projection}.{label}", out_dim)


def _spherical_primary(aqlm: AQLMCodebook, cwr) -> tuple[SphericalCodebook, SphericalCWR] | None:
    """The spherical codec and payload under a (possibly sign-split) primary."""
    codec, payload = aqlm.primary, cwr.primary
    if isinstance(codec, SSVQCodebook):
        codec = codec.inner
        payload = payload.inner if isinstance(payload, SSVQCWR) else payload
    if isinstance(codec, SphericalCodebook) and isinstance(payload, SphericalCWR):
        return codec, payload
    return None


class VQRunExperiment(Experiment):
    """One VQ configuration run (experiment.py:87-307): fit, quantise the
    primary scales, measure rel_fro_err and bits per weight, emit the row."""

    def __init__(self, config: VQRunConfig) -> None:
        super().__init__()
        self.config = config
        self._result: dict | None = None

    def _row(self, plan: _Plan, err: float, bpw: float) -> dict:
        cfg = self.config
        extra_bs = [b for b in plan.block_sizes[1:] if b != cfg.block_size]
        return {
            "projection": cfg.projection, "scheme": plan.label, "block_size": cfg.block_size, "K": cfg.K,
            "n_codebooks": cfg.n_codebooks, "metric": cfg.metric, "shared": cfg.shared_codebook,
            "sign_split": cfg.sign_split, "scale_dtype": cfg.scale_dtype, "kmeans_iters": cfg.max_iters,
            "residual_block_sizes": [cfg.block_size, *extra_bs] if extra_bs else [],
            "rel_fro_err": err, "bits_per_weight": bpw, "compression_ratio": 16.0 / bpw,
        }

    def fit(self, W_raw: torch.Tensor) -> dict:  # noqa: N803
        cfg = self.config
        plan = _plan(cfg)
        self._emit(VQStartEvent(config_id=plan.config_id, projection=cfg.projection, block_size=cfg.block_size,
                                K=cfg.K, n_codebooks=cfg.n_codebooks, metric=cfg.metric))
        aqlm = assemble_aqlm(plan.specs, max_iters=cfg.max_iters, norm_threshold=_NORM_THRESHOLD,
                             codebook_bits=cfg.codebook_bits, out_dim=plan.out_dim, num_experts=cfg.num_experts,
                             device=cfg.device, chunk_budget_mb=cfg.chunk_budget_mb)
        for ev in _CHILD_EVENTS:
            self._forward_from(aqlm, ev)
        w = W_raw if cfg.device is None else W_raw.to(cfg.device)
        cwr = aqlm.fit(w)
        if cfg.metric == "cosine" and (sp := _spherical_primary(aqlm, cwr)) is not None:
            quantize_spherical_scales(sp[1], sp[0], cfg.scale_dtype)
        recon = aqlm.reconstruct(cwr)
        ref = W_raw.float().to(recon.device)
        err = (torch.linalg.vector_norm(ref - recon) / torch.linalg.vector_norm(ref)).item()
        del cwr, recon, ref
        bpw = bits_per_weight_kmeans(
            W_raw.shape[0], cfg.in_dim, cfg.in_dim // cfg.block_size, cfg.block_size, cfg.n_codebooks, plan.ks,
            shared_codebook=cfg.shared_codebook, sign_split=cfg.sign_split,
            scale_bits_per_elem=scale_bits_per_elem(cfg.scale_dtype), bs_per_codebook=plan.block_sizes,
            codebook_bits=cfg.codebook_bits, residual_sign_split=plan.residual_sign_split,
            primary_metric=cfg.metric)
        logger.info("  [%s] err=%.6f bpw=%.3f cr=%.2f", cfg.projection, err, bpw, 16.0 / bpw)
        self._result = self._row(plan, err, bpw)
        self._emit(VQDoneEvent(config_id=plan.config_id, row=self._result))
        return self._result

    @property
    def result(self) -> dict:
        assert self._result is not None, "fit() not called yet"
        return self._result
