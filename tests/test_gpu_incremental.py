"""Incremental Lloyd assignment (csrc/incremental.cu, _engine.IncrementalAssign).

A centroid whose cluster kept its members keeps its value, so a point
assigned to it can only move to a centroid that moved; the incremental pass
scores every point against the moved centroids only and re-assigns the points
whose centroid moved over all centroids. It must give exactly the labels of a
full assignment. Checked two ways on Student-t(5) block data at the benchmark
layer's densities (1.5 and 24 points per centroid, euclidean and spherical):

* every incremental assignment of a run equals a full pass on the same
  centroids and previous labels, apart from ties within the reference's
  rounding (whole runs cannot be compared bit for bit: the update's
  floating-point atomics add in a varying order);
* the final labels equal a fresh full assignment against the final centroids.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

CASES = [
    # (metric, nblk, n, bs, K, iters)
    (1, 6, 6144, 4, 4096, 12),     # l2, 1.5 points per centroid (the bs=4 K=65536 residual's density)
    (1, 4, 24576, 16, 1024, 15),   # l2, 24 points per centroid
    (0, 6, 24576, 8, 1024, 25),    # cosine primary, 24 points per centroid
    (0, 3, 3000, 12, 2048, 10),    # cosine, 1.5 points per centroid, bs 12
]


def _points(metric, nblk, n, bs, seed):
    from skcq_b200 import _engine

    g = torch.Generator().manual_seed(seed)
    z = torch.randn(n, nblk * bs, generator=g)
    chi2 = torch.randn(5, n, nblk * bs, generator=g).square().sum(0)
    w = z / torch.sqrt(chi2 / 5.0) * (0.02 / (5.0 / 3.0) ** 0.5)
    return _engine.gather_block_points(w.cuda(), bs, nblk, False, 0.0, False, metric)


def _run(metric, nblk, n, bs, K, iters, force, seed=3):
    from skcq_b200 import _engine
    from skcq_b200.codebook.kmeans import sobol_first_orthant

    pts = _points(metric, nblk, n, bs, seed)
    old = _engine.INCREMENTAL_FORCE
    _engine.INCREMENTAL_FORCE = force
    try:
        if metric == 0:
            run = _engine.lloyd(pts, K, iters,
                                init_cosine=lambda kk, dd: sobol_first_orthant(kk, dd, pts.X.device))
        else:
            g = torch.Generator().manual_seed(seed + 1)
            perms = [torch.randperm(nb, generator=g) for nb in pts.n_host]
            run = _engine.lloyd(pts, K, iters, init_perms=perms)
    finally:
        _engine.INCREMENTAL_FORCE = old
    return pts, run


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{'cos' if c[0] == 0 else 'l2'}_bs{c[3]}_K{c[4]}_n{c[2]}")
def test_incremental_assignment_equals_full(case):
    """Every incremental assignment of a run (one per iteration after the
    point where few clusters change) is compared, on the same centroids and
    previous labels, with a full tensor-core pass; points where the two differ
    must be ties within the reference's rounding (relative top-2 gap <= 1e-5
    under the exact fp32 formula)."""
    from skcq_b200 import _engine

    metric, nblk, n, bs, K, iters = case
    seen = {"calls": 0, "points": 0, "ties": 0}

    def check(pts, B, C, cnorm, k_pad, k_dev, active, labels):
        full = torch.zeros_like(labels)
        _engine.assign_call(pts, B, C, cnorm, k_pad, k_dev, active, full)
        torch.cuda.synchronize()
        act = torch.ones(pts.nblk, dtype=torch.bool) if active is None else active.bool().cpu()
        for b in range(pts.nblk):
            if not act[b]:
                continue
            nb = pts.n_host[b]
            diff = (full[b, :nb] != labels[b, :nb]).nonzero().flatten()
            seen["points"] += nb
            if diff.numel() == 0:
                continue
            x = pts.X[b, diff].double()
            ca, cf = C[b, labels[b, diff].long()].double(), C[b, full[b, diff].long()].double()
            if metric == 0:
                sa, sf = (x * ca).sum(1), (x * cf).sum(1)
            else:
                sa, sf = 2 * (x * ca).sum(1) - (ca * ca).sum(1), 2 * (x * cf).sum(1) - (cf * cf).sum(1)
            cn = torch.maximum(ca.norm(dim=1), cf.norm(dim=1))
            scale = (x.norm(dim=1) * cn + (cn * cn if metric == 1 else 0)).clamp_min(1e-30)
            assert ((sa - sf).abs() / scale <= 1e-5).all(), (b, diff.numel())
            seen["ties"] += diff.numel()
        seen["calls"] += 1

    _engine.INCREMENTAL_CHECK = check
    try:
        pts, run = _run(metric, nblk, n, bs, K, iters, force=True)  # incremental whenever lists exist
    finally:
        _engine.INCREMENTAL_CHECK = None
    assert seen["calls"] >= 2, seen
    assert seen["ties"] <= 1e-4 * seen["points"], seen
    # and the final labels are those of a fresh full assignment against the final centroids
    fresh = _engine.assign(pts, run)
    for b in range(pts.nblk):
        nb = pts.n_host[b]
        assert int((fresh[b, :nb] != run.labels[b, :nb]).sum()) <= max(1, int(1e-4 * nb)), b


def test_incremental_pass_is_taken():
    """The default threshold does choose incremental passes once few clusters
    change (the converging tail of a run)."""
    from skcq_b200 import _engine

    _engine.TIMER.reset()
    _engine.TIMER.enabled = True
    try:
        _run(1, 4, 6144, 4, 4096, 12, force=False)
        summ = _engine.TIMER.summary()
    finally:
        _engine.TIMER.enabled = False
    full_work = 2.0 * 4 * 6144 * 4096 * 4  # one full pass over the four problems
    assert summ["assign"]["work"] < 0.6 * full_work * summ["assign"]["launches"], summ["assign"]
