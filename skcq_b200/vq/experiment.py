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

from skcq_b200.codebook.aqlm import AQLMCodebook, AQLMCodebookConfig
from skcq_b200.codebook.base import DistanceMetric, WeightsCodebookBase
from skcq_b200.codebook.cwr import SSVQCWR, SphericalCWR
from skcq_b200.codebook.euclidean import EuclideanCodebook, EuclideanCodebookConfig
from skcq_b200.codebook.events import (
    CodebookDoneEvent,
    CodebookIterEvent,
    CodebookStartEvent,
    Experiment,
    KmeansDoneEvent,
    KmeansIterEvent,
    KmeansStartEvent,
)
from skcq_b200.codebook.spherical import (
    SphericalCodebook,
    SphericalCodebookConfig,
    quantize_spherical_scales,
    scale_bits_per_elem,
)
from skcq_b200.codebook.ssvq import SSVQCodebook
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


def _per_residual(value, n: int, primary):
    """Per-codebook values: the primary's, then residual c's from a scalar or a
    list indexed c - 1 (experiment.py:97-125)."""
    if value is None:
        return [primary] * n
    if isinstance(value, list):
        return [primary if c == 0 else value[c - 1] for c in range(n)]
    return [primary if c == 0 else value for c in range(n)]


class VQRunExperiment(Experiment):
    """One VQ configuration run (experiment.py:87-307)."""

    def __init__(self, config: VQRunConfig) -> None:
        super().__init__()
        self.config = config
        self._result: dict | None = None

    def fit(self, W_raw: torch.Tensor) -> dict:  # noqa: N803
        cfg = self.config
        device = cfg.device
        n_rows = W_raw.shape[0]
        w_norm = W_raw.float().norm().item()
        n_blocks = cfg.in_dim // cfg.block_size
        k_per = [cfg.K if c == 0 else (cfg.residual_k or cfg.K) for c in range(cfg.n_codebooks)] \
            if isinstance(cfg.residual_k, int | None) else _per_residual(cfg.residual_k, cfg.n_codebooks, cfg.K)
        bs_per = _per_residual(cfg.residual_block_sizes, cfg.n_codebooks, cfg.block_size)
        if cfg.residual_sign_split is None:
            res_ss = [False] * (cfg.n_codebooks - 1)
        elif isinstance(cfg.residual_sign_split, bool):
            res_ss = [cfg.residual_sign_split] * (cfg.n_codebooks - 1)
        else:
            res_ss = list(cfg.residual_sign_split[: cfg.n_codebooks - 1])
            res_ss += [False] * (cfg.n_codebooks - 1 - len(res_ss))
        sign_split = [cfg.sign_split, *res_ss]

        cb_id = "-".join(f"cb{c}_b{bs_per[c]}k{k_per[c]}" for c in range(cfg.n_codebooks))
        scale_tag = f"_{cfg.scale_dtype}" if cfg.scale_dtype != "bf16" else ""
        cb_qtag = f"_cb{cfg.codebook_bits}" if cfg.codebook_bits < 16 else ""
        label = (f"kmeans_{cb_id}_{cfg.metric[:3]}_{'shared' if cfg.shared_codebook else 'perblock'}_"
                 f"{'ssvq' if cfg.sign_split else 'nosign'}{scale_tag}{cb_qtag}")
        out_dim = cfg.intermediate_size if cfg.projection != "down" else cfg.hidden_size
        config_id = f"L{cfg.layer_idx}.{cfg.projection}.{label}"
        self._emit(VQStartEvent(config_id=config_id, projection=cfg.projection, block_size=cfg.block_size, K=cfg.K,
                                n_codebooks=cfg.n_codebooks, metric=cfg.metric))

        sub = 2**23 if cfg.shared_codebook else 0
        primary: WeightsCodebookBase
        if cfg.metric == "cosine":
            primary = SphericalCodebook(SphericalCodebookConfig(
                block_size=cfg.block_size, K=cfg.K, shared=cfg.shared_codebook, max_iters=cfg.max_iters,
                norm_threshold=0.001, skip_zeros=True, chunk_budget_mb=cfg.chunk_budget_mb, device=device,
                max_train_samples=sub))
            if cfg.sign_split:
                primary = SSVQCodebook(primary)
        else:
            primary = EuclideanCodebook(EuclideanCodebookConfig(
                block_size=cfg.block_size, K=cfg.K, shared=cfg.shared_codebook, max_iters=cfg.max_iters,
                norm_threshold=0.001, skip_zeros=True, chunk_budget_mb=cfg.chunk_budget_mb, device=device,
                max_train_samples=sub))
        residuals: list[WeightsCodebookBase] = []
        for c in range(1, cfg.n_codebooks):
            euc: WeightsCodebookBase = EuclideanCodebook(EuclideanCodebookConfig(
                block_size=bs_per[c], K=k_per[c], shared=cfg.shared_codebook, max_iters=cfg.max_iters,
                norm_threshold=0.001, skip_zeros=False, chunk_budget_mb=cfg.chunk_budget_mb, device=device))
            if sign_split[c]:
                euc = SSVQCodebook(euc)
            residuals.append(euc)
        aqlm = AQLMCodebook(primary=primary, residuals=residuals, config=AQLMCodebookConfig(
            codebook_bits=cfg.codebook_bits, norm_threshold=0.001, device=device, out_dim=out_dim,
            num_experts=cfg.num_experts))
        for ev in (CodebookStartEvent, CodebookIterEvent, CodebookDoneEvent, KmeansStartEvent, KmeansIterEvent,
                   KmeansDoneEvent):
            self._forward_from(aqlm, ev)

        cwr = aqlm.fit(W_raw.to(device) if device is not None else W_raw)
        sc_bits = scale_bits_per_elem(cfg.scale_dtype)
        if cfg.metric == "cosine":
            cb, cwr_p = aqlm.primary, cwr.primary
            if isinstance(cb, SSVQCodebook):
                cb, cwr_p = cb.inner, cwr_p.inner if isinstance(cwr_p, SSVQCWR) else cwr_p
            if isinstance(cb, SphericalCodebook) and isinstance(cwr_p, SphericalCWR):
                quantize_spherical_scales(cwr_p, cb, cfg.scale_dtype)
        w_recon = aqlm.reconstruct(cwr)
        err = torch.norm(W_raw.float().to(w_recon.device) - w_recon).item() / w_norm
        bpw = bits_per_weight_kmeans(
            n_rows, cfg.in_dim, n_blocks, cfg.block_size, cfg.n_codebooks, k_per,
            shared_codebook=cfg.shared_codebook, sign_split=cfg.sign_split, scale_bits_per_elem=sc_bits,
            bs_per_codebook=bs_per, codebook_bits=cfg.codebook_bits, residual_sign_split=res_ss,
            primary_metric=cfg.metric)
        logger.info("  [%s] err=%.6f bpw=%.3f cr=%.2f", cfg.projection, err, bpw, 16.0 / bpw)
        del cwr, w_recon
        row = {
            "projection": cfg.projection, "scheme": label, "block_size": cfg.block_size, "K": cfg.K,
            "n_codebooks": cfg.n_codebooks, "metric": cfg.metric, "shared": cfg.shared_codebook,
            "sign_split": cfg.sign_split, "scale_dtype": cfg.scale_dtype, "kmeans_iters": cfg.max_iters,
            "residual_block_sizes": ([cfg.block_size] + [b for b in bs_per[1:] if b != cfg.block_size]
                                     if any(b != cfg.block_size for b in bs_per[1:]) else []),
            "rel_fro_err": err, "bits_per_weight": bpw, "compression_ratio": 16.0 / bpw,
        }
        self._result = row
        self._emit(VQDoneEvent(config_id=config_id, row=row))
        return row

    @property
    def result(self) -> dict:
        assert self._result is not None, "fit() not called yet"
        return self._result
