"""Numpy restatement of SKCQ's codecs: spherical, euclidean, SSVQ and the AQLM
composite (skcq/codebook/{spherical,euclidean,ssvq,aqlm}.py).

Test infrastructure only (see ``oracle/__init__.py``). A codec here is a plain
dict of numpy arrays; a CWR is a dict with the fields of skcq/codebook/cwr.py.
bf16 rounding (``.to(torch.bfloat16)``) is restated as round-to-nearest-even on
the top 16 bits of the float32 pattern.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass, field

import numpy as np

from oracle.kmeans import (
    F32,
    KmeansLog,
    assign_cosine,
    assign_l2,
    fit_cosine,
    fit_euclidean,
    normalize_rows,
)

SobolFn = Callable[[int, int], np.ndarray]  # (k, d) -> (k, d) unit directions
PermFn = Callable[[int], np.ndarray]  # n -> permutation of range(n)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 -> float32, round to nearest even (NaN-free input)."""
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32)
    lsb = (u >> 16) & 1
    r = (u + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)
    return r.view(F32)


def row_norms(x: np.ndarray) -> np.ndarray:
    x = x.astype(F32, copy=False)
    return np.sqrt(np.einsum("nd,nd->n", x, x, dtype=F32)).astype(F32)


# ---------------------------------------------------------------------------
# Spherical codec (skcq/codebook/spherical.py)
# ---------------------------------------------------------------------------


@dataclass
class SphericalCfg:
    """SphericalCodebookConfig (spherical.py:103-120)."""

    block_size: int
    K: int
    shared: bool = False
    max_iters: int = 100
    norm_threshold: float = 0.001
    skip_zeros: bool = True
    max_train_samples: int = 0


@dataclass
class EuclideanCfg:
    """EuclideanCodebookConfig (euclidean.py:18-33)."""

    block_size: int
    K: int
    shared: bool = False
    max_iters: int = 100
    norm_threshold: float = 0.001
    skip_zeros: bool = True
    max_train_samples: int = 0


@dataclass
class Codec:
    """A fitted codec: ``kind`` in {"spherical", "euclidean", "ssvq"}."""

    kind: str
    cfg: object = None
    centroids: np.ndarray | None = None  # (n_blocks|1, bs, K), bf16-valued f32
    inner: Codec | None = None
    scale_dtype: str = "bf16"
    q_scale: float | None = None
    logs: list[KmeansLog] = field(default_factory=list)

    @property
    def block_size(self) -> int:
        return self.inner.block_size if self.kind == "ssvq" else self.cfg.block_size


def _spherical_cluster_block(
    cfg: SphericalCfg, data: np.ndarray, sobol: SobolFn, perm: PermFn, logs: list
) -> tuple[np.ndarray, np.ndarray]:
    """spherical.py:225-304 ``_cluster_block``. Returns (labels_full, centroids (k, d))."""
    n_rows, d = data.shape
    block_zero = row_norms(data) < F32(cfg.norm_threshold)
    if cfg.skip_zeros:
        non_zero = data[~block_zero]
    else:
        non_zero = data
        block_zero = np.zeros(n_rows, dtype=bool)
    if non_zero.shape[0] == 0:
        return np.zeros(n_rows, dtype=np.int64), np.zeros((min(cfg.K, 1), d), dtype=F32)
    k_eff = min(cfg.K, non_zero.shape[0])
    train = non_zero
    if cfg.max_train_samples > 0 and non_zero.shape[0] > cfg.max_train_samples:
        train = non_zero[perm(non_zero.shape[0])[: cfg.max_train_samples]]
    cent, _, log = fit_cosine(train, train, k_eff, cfg.max_iters, sobol(min(k_eff, train.shape[0]), d))
    logs.append(log)
    unit = normalize_rows(non_zero)
    labels_nz = assign_cosine(unit, cent.T)
    scales_nz = np.einsum("nd,nd->n", non_zero, cent[labels_nz], dtype=F32)
    neg = scales_nz < 0
    if neg.any():
        # spherical.py:295-298 indexes dimension 1 of the (k, d) centroid matrix.
        neg_labels = np.unique(labels_nz[neg])
        if neg_labels.max() >= d:
            raise IndexError("negative-scale flip: label out of range for dim 1 (spherical.py:298)")
        cent[:, neg_labels] = -cent[:, neg_labels]
    labels_full = np.zeros(n_rows, dtype=np.int64)
    labels_full[~block_zero] = labels_nz
    return labels_full, cent


def spherical_fit(
    cfg: SphericalCfg, w: np.ndarray, sobol: SobolFn, perm: PermFn | None = None
) -> tuple[Codec, dict]:
    """spherical.py:140-190 ``SphericalCodebook.fit``."""
    raw = w.astype(F32)
    n_rows, in_dim = raw.shape
    bs = cfg.block_size
    n_blocks = in_dim // bs
    cov = n_blocks * bs
    rem = in_dim - cov
    zero_mask = row_norms(raw) < F32(cfg.norm_threshold)
    logs: list[KmeansLog] = []
    if cfg.shared:
        pooled = raw[:, :cov].reshape(n_rows * n_blocks, bs)
        labels, cent = _spherical_cluster_block(cfg, pooled, sobol, perm, logs)
        assignments = labels.reshape(n_rows, n_blocks).T.copy()
        directions = cent.T.copy()[None]
    else:
        lab, cents = [], []
        for b in range(n_blocks):
            labels, cent = _spherical_cluster_block(cfg, raw[:, b * bs : (b + 1) * bs], sobol, perm, logs)
            lab.append(labels)
            cents.append(cent.T.copy())
        if len({c.shape for c in cents}) != 1:
            raise RuntimeError("stack expects each tensor to be equal size (spherical.py:176)")
        assignments = np.stack(lab, 0)
        directions = np.stack(cents, 0)
    scales = np.zeros((n_rows, n_blocks), dtype=F32)
    for b in range(n_blocks):
        cb = directions[0] if cfg.shared else directions[b]
        d = cb.T[assignments[b]].copy()
        d[zero_mask] = 0.0
        scales[:, b] = np.einsum("nd,nd->n", raw[:, b * bs : (b + 1) * bs], d, dtype=F32)
    remainder = bf16_round(raw[:, cov:]) if rem > 0 else None
    codec = Codec("spherical", cfg, centroids=bf16_round(directions), logs=logs)
    return codec, {"idxs": assignments, "scales": scales, "remainder": remainder}


def dequant_scales(codec: Codec, scales: np.ndarray) -> np.ndarray:
    """spherical.py:213-223 ``_dequant_scales``."""
    if codec.scale_dtype.startswith("int"):
        return scales.astype(F32) * F32(codec.q_scale)
    return scales.astype(F32)


def spherical_reconstruct(codec: Codec, cwr: dict) -> np.ndarray:
    """spherical.py:192-211."""
    idxs = cwr["idxs"]
    n_blocks, n_rows = idxs.shape
    bs = codec.cfg.block_size
    cov = n_blocks * bs
    rem = cwr["remainder"].shape[1] if cwr["remainder"] is not None else 0
    recon = np.zeros((n_rows, cov + rem), dtype=F32)
    dirs = codec.centroids.astype(F32)
    scales = dequant_scales(codec, cwr["scales"])
    for b in range(n_blocks):
        cb = dirs[0] if codec.cfg.shared else dirs[b]
        recon[:, b * bs : (b + 1) * bs] = scales[:, b : b + 1] * cb.T[idxs[b]]
    if rem:
        recon[:, cov:] = cwr["remainder"].astype(F32)
    return recon


# ---------------------------------------------------------------------------
# Euclidean codec (skcq/codebook/euclidean.py)
# ---------------------------------------------------------------------------


def _euclidean_cluster_block(
    cfg: EuclideanCfg, data: np.ndarray, perm: PermFn, logs: list
) -> tuple[np.ndarray, np.ndarray]:
    """euclidean.py:122-184 ``_cluster_block``. Returns (labels_full, centroids (d, k))."""
    n_rows, d = data.shape
    block_zero = row_norms(data) < F32(cfg.norm_threshold)
    if cfg.skip_zeros:
        non_zero = data[~block_zero]
    else:
        non_zero = data
        block_zero = np.zeros(n_rows, dtype=bool)
    if non_zero.shape[0] == 0:
        return np.zeros(n_rows, dtype=np.int64), np.zeros((d, cfg.K), dtype=F32)
    k_eff = min(cfg.K, non_zero.shape[0])
    train = non_zero
    if cfg.max_train_samples > 0 and non_zero.shape[0] > cfg.max_train_samples:
        train = non_zero[perm(non_zero.shape[0])[: cfg.max_train_samples]]
    cent, _, log = fit_euclidean(train, k_eff, cfg.max_iters, perm(train.shape[0]))
    logs.append(log)
    labels_nz = assign_l2(non_zero, cent.T)
    labels_full = np.zeros(n_rows, dtype=np.int64)
    labels_full[~block_zero] = labels_nz
    return labels_full, cent.T.copy()


def euclidean_fit(cfg: EuclideanCfg, w: np.ndarray, perm: PermFn) -> tuple[Codec, dict]:
    """euclidean.py:55-101 ``EuclideanCodebook.fit``."""
    raw = w.astype(F32)
    n_rows, in_dim = raw.shape
    bs = cfg.block_size
    n_blocks = in_dim // bs
    cov = n_blocks * bs
    rem = in_dim - cov
    logs: list[KmeansLog] = []
    if cfg.shared:
        pooled = raw[:, :cov].reshape(n_rows * n_blocks, bs)
        labels, cent = _euclidean_cluster_block(cfg, pooled, perm, logs)
        assignments = labels.reshape(n_rows, n_blocks).T.copy()
        centroids = cent[None]
    else:
        lab, cents = [], []
        for b in range(n_blocks):
            labels, cent = _euclidean_cluster_block(cfg, raw[:, b * bs : (b + 1) * bs], perm, logs)
            lab.append(labels)
            cents.append(cent)
        if len({c.shape for c in cents}) != 1:
            raise RuntimeError("stack expects each tensor to be equal size (euclidean.py:95)")
        assignments = np.stack(lab, 0)
        centroids = np.stack(cents, 0)
    remainder = bf16_round(raw[:, cov:]) if rem > 0 else None
    codec = Codec("euclidean", cfg, centroids=bf16_round(centroids), logs=logs)
    return codec, {"idxs": assignments, "remainder": remainder}


def euclidean_reconstruct(codec: Codec, cwr: dict) -> np.ndarray:
    """euclidean.py:103-120."""
    idxs = cwr["idxs"]
    n_blocks, n_rows = idxs.shape
    bs = codec.cfg.block_size
    cov = n_blocks * bs
    rem = cwr["remainder"].shape[1] if cwr["remainder"] is not None else 0
    recon = np.zeros((n_rows, cov + rem), dtype=F32)
    cbs = codec.centroids.astype(F32)
    for b in range(n_blocks):
        cb = cbs[0] if codec.cfg.shared else cbs[b]
        recon[:, b * bs : (b + 1) * bs] = cb.T[idxs[b]]
    if rem:
        recon[:, cov:] = cwr["remainder"].astype(F32)
    return recon


# ---------------------------------------------------------------------------
# SSVQ combinator (skcq/codebook/ssvq.py) and dispatch helpers
# ---------------------------------------------------------------------------


def ssvq_fold(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """ssvq.py:43-53: signs = sign(w) with 0 -> +1; folded = w * signs."""
    signs = np.sign(w.astype(F32))
    signs[signs == 0] = 1.0
    return (w.astype(F32) * signs).astype(F32), signs.astype(np.int8)


def fit(codec_spec: tuple, w: np.ndarray, sobol: SobolFn, perm: PermFn) -> tuple[Codec, dict]:
    """Fit a codec spec ``("spherical", cfg) | ("euclidean", cfg) | ("ssvq", inner_spec)``."""
    kind = codec_spec[0]
    if kind == "spherical":
        return spherical_fit(codec_spec[1], w, sobol, perm)
    if kind == "euclidean":
        return euclidean_fit(codec_spec[1], w, perm)
    if kind == "ssvq":
        folded, signs = ssvq_fold(w)
        inner, inner_cwr = fit(codec_spec[1], folded, sobol, perm)
        return Codec("ssvq", inner=inner), {"inner": inner_cwr, "signs": signs}
    raise ValueError(kind)


def reconstruct(codec: Codec, cwr: dict) -> np.ndarray:
    if codec.kind == "spherical":
        return spherical_reconstruct(codec, cwr)
    if codec.kind == "euclidean":
        return euclidean_reconstruct(codec, cwr)
    # ssvq.py:57-66: signs over min(recon width, signs width) columns.
    recon = reconstruct(codec.inner, cwr["inner"])
    cov = min(recon.shape[1], cwr["signs"].shape[1])
    recon[:, :cov] = recon[:, :cov] * cwr["signs"][:, :cov].astype(F32)
    return recon


def quantize_centroids(codec: Codec, bits: int) -> None:
    """spherical.py:306-315 / euclidean.py:186-195: one int scale per centroid index."""
    if codec.kind == "ssvq":
        quantize_centroids(codec.inner, bits)
        return
    if bits >= 16 or codec.centroids is None:
        return
    levels = F32(2 ** (bits - 1) - 1)
    cb = codec.centroids.astype(F32)
    flat = cb.reshape(-1, cb.shape[-1])
    cb_max = np.maximum(np.abs(flat).max(axis=0), F32(1e-10))
    q_scale = (cb_max / levels).astype(F32)
    q = np.clip(np.rint(flat / q_scale), -levels, levels).astype(F32)
    codec.centroids = bf16_round((q * q_scale).astype(F32)).reshape(cb.shape)


def quantize_scales(cwr: dict, codec: Codec, scale_dtype: str) -> None:
    """spherical.py:45-71 ``quantize_spherical_scales`` (bf16 and int<N> modes)."""
    scales = cwr["scales"].astype(F32)
    if scale_dtype == "bf16":
        cwr["scales"] = bf16_round(scales)
        codec.scale_dtype, codec.q_scale = "bf16", None
    elif scale_dtype.startswith("int"):
        bits = int(scale_dtype[3:])
        levels = F32(2 ** (bits - 1) - 1)
        abs_max = F32(np.abs(scales).max())
        codec.scale_dtype = scale_dtype
        if abs_max == 0:
            codec.q_scale = 0.0
            return
        q_scale = F32(abs_max / levels)
        q = np.clip(np.rint(scales / q_scale), -levels, levels)
        cwr["scales"] = q.astype(np.int8 if bits <= 8 else np.int16)
        codec.q_scale = float(q_scale)
    else:
        raise ValueError(scale_dtype)


# ---------------------------------------------------------------------------
# AQLM composite (skcq/codebook/aqlm.py)
# ---------------------------------------------------------------------------


def _unwrap_spherical(codec: Codec, cwr: dict):
    """aqlm.py:273-285 ``_unwrap_spherical_primary_from_cwr``."""
    if codec.kind == "ssvq" and codec.inner.kind == "spherical":
        return codec.inner, cwr["inner"], cwr["signs"]
    if codec.kind == "spherical":
        return codec, cwr, None
    return None, None, None


def refit_primary_scale(sph: Codec, sph_cwr: dict, signs, raw, zero_mask, recon_total) -> None:
    """aqlm.py:147-179 ``_refit_primary_scale`` (in place on ``sph_cwr['scales']``)."""
    bs = sph.cfg.block_size
    n_blocks = sph_cwr["idxs"].shape[0]
    for b in range(n_blocks):
        cols = slice(b * bs, (b + 1) * bs)
        cb = sph.centroids[0] if sph.cfg.shared else sph.centroids[b]
        d = cb.astype(F32).T[sph_cwr["idxs"][b]].copy()
        d[zero_mask] = 0.0
        pdir = d * signs[:, cols].astype(F32) if signs is not None else d
        scale_old = sph_cwr["scales"][:, b].astype(F32)
        other_b = recon_total[:, cols] - scale_old[:, None] * pdir
        target = raw[:, cols] - other_b
        dot = np.einsum("nd,nd->n", target, pdir, dtype=F32)
        nrm = row_norms(pdir)
        scale_new = (dot / (nrm * nrm + F32(1e-10))).astype(F32)
        scale_new[zero_mask] = 0.0
        sph_cwr["scales"][:, b] = scale_new


def aqlm_fit(
    primary_spec: tuple,
    residual_specs: list[tuple],
    w: np.ndarray,
    sobol: SobolFn,
    perm: PermFn,
    codebook_bits: int = 16,
    norm_threshold: float = 0.001,
) -> tuple[Codec, list[Codec], dict]:
    """aqlm.py:67-135 ``AQLMCodebook.fit``."""
    raw = w.astype(F32)
    zero_mask = row_norms(raw) < F32(norm_threshold)
    primary, primary_cwr = fit(primary_spec, raw, sobol, perm)
    recon = reconstruct(primary, primary_cwr)
    error = raw - recon
    residuals, res_cwrs = [], []
    for spec in residual_specs:
        codec, cwr = fit(spec, error, sobol, perm)
        residuals.append(codec)
        res_cwrs.append(cwr)
        recon = recon + reconstruct(codec, cwr)
        error = raw - recon
    if codebook_bits < 16:
        quantize_centroids(primary, codebook_bits)
        for r in residuals:
            quantize_centroids(r, codebook_bits)
    recon = reconstruct(primary, primary_cwr)
    for r, c in zip(residuals, res_cwrs, strict=True):
        recon = recon + reconstruct(r, c)
    sph, sph_cwr, signs = _unwrap_spherical(primary, primary_cwr)
    if sph is not None:
        refit_primary_scale(sph, sph_cwr, signs, raw, zero_mask, recon)
    return primary, residuals, {"primary": primary_cwr, "residuals": res_cwrs}


def aqlm_reconstruct(primary: Codec, residuals: list[Codec], cwr: dict) -> np.ndarray:
    """aqlm.py:137-141."""
    recon = reconstruct(primary, cwr["primary"])
    for r, c in zip(residuals, cwr["residuals"], strict=True):
        recon = recon + reconstruct(r, c)
    return recon
