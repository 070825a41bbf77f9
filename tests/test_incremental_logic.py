"""The rules of the incremental Lloyd assignment, restated in numpy on the CPU
and checked against the full arg-max at every iteration (the GPU kernels
implement these rules; tests/test_gpu_incremental.py checks them there):

* centroids of clusters that kept their members keep their value, so their
  scores do not change;
* a point whose centroid did not move goes to the best moved centroid only if
  it scores higher, or the same with a lower index;
* a point whose centroid moved takes the best moved centroid when that scores
  above the point's previous score against its centroid; otherwise it is
  searched over all centroids;
* (euclidean) a point exactly on its unmoved centroid is not scored at all;
* (euclidean, Forgy start) a seed point takes its own centroid in the first
  assignment unless a centroid of identical value exists.

Scores come from one matrix per iteration, so the comparison is of the rules
alone, not of rounding."""

from __future__ import annotations

import numpy as np
import pytest


def _scores(x: np.ndarray, c: np.ndarray, cosine: bool) -> np.ndarray:
    if cosine:
        return x @ c.T
    return 2.0 * (x @ c.T) - (c * c).sum(1)[None, :]  # larger is better (= -(||c||^2 - 2 x.c))


def _first_max(s: np.ndarray) -> np.ndarray:
    return s.argmax(1)  # numpy: first maximum wins


def _incremental(x, c, c_old, lab_prev, moved, cosine):
    """The incremental assignment of x against c, given the previous labels,
    the previous centroids and the moved mask."""
    s = _scores(x, c, cosine)
    s_old = _scores(x, c_old, cosine)
    n = x.shape[0]
    lab = lab_prev.copy()
    mv = np.flatnonzero(moved)
    stats = {"skipped": 0, "to_moved": 0, "resolved": 0, "searched": 0}
    if mv.size == 0:
        return lab, stats
    # euclidean: points exactly on an unmoved centroid are not scored
    exact_self = (~moved[lab_prev]) & np.all(x == c[lab_prev], axis=1) if not cosine else np.zeros(n, bool)
    sm = s[:, mv]
    best_m = mv[_first_max(sm)]  # lowest index among equal moved scores
    v_best = s[np.arange(n), best_m]
    for i in range(n):
        a = lab_prev[i]
        if exact_self[i]:
            stats["skipped"] += 1
            continue
        if not moved[a]:
            if v_best[i] > s[i, a] or (v_best[i] == s[i, a] and best_m[i] < a):
                lab[i] = best_m[i]
                stats["to_moved"] += 1
        elif v_best[i] > s_old[i, a]:
            lab[i] = best_m[i]
            stats["resolved"] += 1
        else:
            lab[i] = _first_max(s[i:i + 1])[0]
            stats["searched"] += 1
    return lab, stats


def _run(n, K, d, iters, cosine, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_t(5, size=(n, d)) * 0.02).astype(np.float64)
    # a few exact duplicates, the case the tie rules are for
    x[n // 2: n // 2 + 20] = x[:20]
    if cosine:
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        c = np.abs(rng.standard_normal((K, d)))
        c /= np.linalg.norm(c, axis=1, keepdims=True)
        perm = None
    else:
        perm = rng.permutation(n)[:K]
        c = x[perm].copy()
    # first assignment
    full = _first_max(_scores(x, c, cosine))
    if perm is not None:
        lab = np.full(n, -1)
        _, first, counts = np.unique(c, axis=0, return_index=True, return_counts=True)
        unique_val = np.zeros(K, bool)
        unique_val[first[counts == 1]] = True
        lab[perm[unique_val]] = np.flatnonzero(unique_val)
        rest = lab < 0
        lab[rest] = _first_max(_scores(x[rest], c, cosine))
        # a seed whose own centroid is its arg-max unless a duplicate value exists
        assert np.array_equal(lab, full)
    lab = full
    members_prev = None
    total = {"skipped": 0, "to_moved": 0, "resolved": 0, "searched": 0}
    for _ in range(iters):
        members = [frozenset(np.flatnonzero(lab == k)) for k in range(K)]
        new = c.copy()
        for k in range(K):
            if members_prev is not None and members[k] == members_prev[k] and members[k]:
                continue  # same members as at the previous update: the same centroid
            if members[k]:
                m = x[list(members[k])].sum(0)
                new[k] = m / np.linalg.norm(m) if cosine else m / len(members[k])
        moved = np.any(new != c, axis=1)
        c_old, c = c, new
        members_prev = members
        inc, stats = _incremental(x, c, c_old, lab, moved, cosine)
        ref = _first_max(_scores(x, c, cosine))
        assert np.array_equal(inc, ref)
        for key, v in stats.items():
            total[key] += v
        lab = ref
    return total


@pytest.mark.parametrize("cosine", [False, True], ids=["l2", "cosine"])
def test_incremental_rules_equal_full_argmax(cosine):
    # l2: 1.5 points per centroid (the K = 65536 residual's density); cosine: 24
    if cosine:
        total = _run(n=3072, K=128, d=8, iters=12, cosine=True, seed=1)
    else:
        total = _run(n=1536, K=1024, d=4, iters=8, cosine=False, seed=2)
        assert total["skipped"] > 0
    # every rule was taken at least once
    assert total["to_moved"] > 0 and total["resolved"] > 0 and total["searched"] > 0, total
