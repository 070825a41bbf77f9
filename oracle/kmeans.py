"""Numpy restatement of SKCQ's Lloyd k-means (skcq/codebook/kmeans.py).

Test infrastructure only (see ``oracle/__init__.py``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

F32 = np.float32


def normalize_rows(x: np.ndarray, eps: float = 1e-12) -> np.ndarray:
    """``torch.nn.functional.normalize(x, dim=-1)``: x / max(||x||_2, eps)."""
    x = x.astype(F32, copy=False)
    n = np.sqrt(np.einsum("nd,nd->n", x, x, dtype=F32)).astype(F32)
    return (x / np.maximum(n, F32(eps))[:, None]).astype(F32)


def scores_cosine(data: np.ndarray, centroids_t: np.ndarray) -> np.ndarray:
    """The matrix ``chunk @ centroids`` maximised by kmeans.py:41-42."""
    return data.astype(F32) @ centroids_t.astype(F32)


def scores_l2(data: np.ndarray, centroids_t: np.ndarray) -> np.ndarray:
    """The matrix minimised by kmeans.py:59-65: ``-2 * (x @ C) + ||c||^2``."""
    c = centroids_t.astype(F32)
    cb_sq = np.square(c).sum(axis=0, dtype=F32)[None, :]
    d = data.astype(F32) @ c
    return (d * F32(-2.0) + cb_sq).astype(F32)


def assign_cosine(data: np.ndarray, centroids_t: np.ndarray) -> np.ndarray:
    """kmeans.py:25-43 ``assign_cosine``: argmax of dot products (first max wins)."""
    return scores_cosine(data, centroids_t).argmax(axis=-1).astype(np.int64)


def assign_l2(data: np.ndarray, centroids_t: np.ndarray) -> np.ndarray:
    """kmeans.py:46-66 ``assign_l2``: argmin of ``||c||^2 - 2 x.c`` (first min wins)."""
    return scores_l2(data, centroids_t).argmin(axis=-1).astype(np.int64)


def top2_margin(scores: np.ndarray, maximise: bool) -> np.ndarray:
    """Gap between the best and the second-best score of every row (>= 0)."""
    s = scores if maximise else -scores
    if s.shape[1] < 2:
        return np.full(s.shape[0], np.inf, dtype=F32)
    part = np.partition(s, -2, axis=1)[:, -2:]
    return (part[:, 1] - part[:, 0]).astype(F32)


@dataclass
class KmeansLog:
    """What ``KmeansExperiment`` reports through its events (events.py:19-35)."""

    k: int = 0
    n_points: int = 0
    iters: list[tuple[float, int]] = field(default_factory=list)  # (moved, n_empty)
    iters_run: int = 0
    final_moved: float = 0.0
    converged: bool = False
    # smallest relative top-2 gap seen in any assignment or reseed selection of
    # this run; below ~1e-6 the trajectory depends on rounding order (ties)
    # Exact ties (gap 0, e.g. two identical centroids) are counted separately:
    # the first index wins in every implementation when the tied values are
    # bit-identical, so they change labels but not reconstructions.
    min_margin: float = float("inf")
    exact_ties: int = 0

    def note(self, m: tuple[float, int]) -> None:
        self.min_margin = min(self.min_margin, float(m[0]))
        self.exact_ties += int(m[1])


def _gap_stats(gap: np.ndarray, den: np.ndarray) -> tuple[float, int]:
    pos = gap > 0
    rel = gap[pos] / den[pos]
    return (float(rel.min()) if rel.size else float("inf")), int((~pos).sum())


def rel_margin(scores: np.ndarray, maximise: bool) -> tuple[float, int]:
    """(min over rows of (best - second) / (|best| + |second|) for non-zero gaps,
    number of rows whose best two scores are exactly equal)."""
    s = scores if maximise else -scores
    if s.shape[1] < 2 or s.shape[0] == 0:
        return float("inf"), 0
    part = np.partition(s, -2, axis=1)[:, -2:]
    gap = (part[:, 1] - part[:, 0]).astype(np.float64)
    den = np.abs(part[:, 1]).astype(np.float64) + np.abs(part[:, 0]) + 1e-30
    return _gap_stats(gap, den)


def sort_gap(values: np.ndarray, order: np.ndarray, m: int) -> tuple[float, int]:
    """Relative gaps between consecutive selected keys and the first unselected one."""
    if m == 0 or len(order) < 2:
        return float("inf"), 0
    v = values[order[: m + 1]].astype(np.float64)
    return _gap_stats(np.abs(np.diff(v)), np.abs(v[1:]) + np.abs(v[:-1]) + 1e-30)


def _index_add(k: int, labels: np.ndarray, rows: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``index_add_`` of rows and of ones (kmeans.py:152-159), in row order."""
    d = rows.shape[1]
    sums = np.zeros((k, d), dtype=F32)
    np.add.at(sums, labels, rows.astype(F32))
    counts = np.bincount(labels, minlength=k).astype(F32)
    return sums, counts


def fit_cosine(
    data: np.ndarray,
    raw_data: np.ndarray | None,
    k: int,
    max_iters: int,
    init_centroids: np.ndarray,
) -> tuple[np.ndarray, np.ndarray, KmeansLog]:
    """kmeans.py:109-193 (``fit`` + ``_fit_cosine``).

    ``init_centroids`` is ``sobol_first_orthant(k_eff, d)`` (kmeans.py:69-74),
    shape ``(k_eff, d)``; ``k`` is clipped to ``min(k, n)`` as at kmeans.py:112.
    Returns ``(centroids (k_eff, d), labels (n,), log)``.
    """
    n, d = data.shape
    k_eff = min(k, n)
    raw = data if raw_data is None else raw_data
    log = KmeansLog(k=k_eff, n_points=n)
    unit = normalize_rows(data)
    cent = init_centroids.astype(F32).copy()
    assert cent.shape == (k_eff, d)
    final_moved = 0.0
    converged = False
    it = -1
    for it in range(max_iters):
        sc = scores_cosine(unit, cent.T)
        log.note(rel_margin(sc, True))
        labels = sc.argmax(axis=-1)
        sums, counts = _index_add(k_eff, labels, raw)
        empty = counts == 0
        n_empty = int(empty.sum())
        if n_empty > 0:
            # kmeans.py:163-172: worst-fit points (lowest similarity) fill the
            # empty clusters in ascending cluster order.
            sims = np.einsum("nd,nd->n", unit, cent[labels], dtype=F32)
            order = np.argsort(sims, kind="stable")
            log.note(sort_gap(sims, order, n_empty))
            worst = order[:n_empty]
            sums[empty] = unit[worst]
        new = normalize_rows(sums)
        moved = float(np.sqrt(np.square(new - cent, dtype=F32).sum(dtype=F32)))
        cent = new
        log.iters.append((moved, n_empty))
        if moved < 1e-6:
            converged = True
            final_moved = moved
            break
        final_moved = moved
    sc = scores_cosine(unit, cent.T)
    log.note(rel_margin(sc, True))
    labels = sc.argmax(axis=-1).astype(np.int64)
    log.iters_run = it + 1
    log.final_moved = final_moved
    log.converged = converged
    return cent, labels, log


def fit_euclidean(
    data: np.ndarray,
    k: int,
    max_iters: int,
    init_perm: np.ndarray,
) -> tuple[np.ndarray, np.ndarray, KmeansLog]:
    """kmeans.py:195-249 (``_fit_euclidean``).

    ``init_perm`` is ``torch.randperm(n)[:k_eff]`` (kmeans.py:201).
    """
    n, d = data.shape
    k_eff = min(k, n)
    log = KmeansLog(k=k_eff, n_points=n)
    data = data.astype(F32)
    cent = data[np.asarray(init_perm)[:k_eff]].copy()
    final_moved = 0.0
    converged = False
    it = -1
    for it in range(max_iters):
        sc = scores_l2(data, cent.T)
        log.note(rel_margin(sc, False))
        labels = sc.argmin(axis=-1)
        sums, counts = _index_add(k_eff, labels, data)
        empty = counts == 0
        n_empty = int(empty.sum())
        if n_empty > 0:
            # kmeans.py:221-230: farthest points, in descending distance order.
            diff = data - cent[labels]
            dists = np.square(diff, dtype=F32).sum(axis=-1, dtype=F32)
            order = np.argsort(-dists, kind="stable")
            log.note(sort_gap(dists, order, n_empty))
            worst = order[:n_empty]
            sums[empty] = data[worst]
        ne = ~empty
        sums[ne] = sums[ne] / counts[ne][:, None]
        new = sums
        moved = float(np.sqrt(np.square(new - cent, dtype=F32).sum(dtype=F32)))
        cent = new
        log.iters.append((moved, n_empty))
        if moved < 1e-6:
            converged = True
            final_moved = moved
            break
        final_moved = moved
    sc = scores_l2(data, cent.T)
    log.note(rel_margin(sc, False))
    labels = sc.argmin(axis=-1).astype(np.int64)
    log.iters_run = it + 1
    log.final_moved = final_moved
    log.converged = converged
    return cent, labels, log
