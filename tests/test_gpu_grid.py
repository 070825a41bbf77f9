"""The centroid-grid search for low-dimensional euclidean problems
(csrc/assign_grid.cu) gives exactly the labels of the exact full scan
(skcq_assign_exact: the reference formula's arg-max over all centroids, first
maximum; kmeans.py:46-66), through the engine's assignment (grid, then the
full search of the points the grid could not certify) and through the C ABI,
and certifies nearly every point."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from skcq_b200 import _lib

    _lib.load()


def _setup(nblk, n, bs, K, seed, forgy, dup=False, outliers=0):
    """Points of nblk blocks (gathered by the product's own path) and K
    centroids per problem: Forgy seeds (points) or random; dup makes exact
    duplicate centroids (ties the lower index wins); outliers puts a few points
    far outside the centroids (their nearest centroid lies beyond any cell
    neighbourhood)."""
    from skcq_b200 import _engine
    from skcq_b200._lib import call, ptr, stream

    g = torch.Generator().manual_seed(seed)
    chi2 = torch.randn(5, n, nblk * bs, generator=g).square_().sum(0)
    w = torch.randn(n, nblk * bs, generator=g) / torch.sqrt(chi2 / 5.0) * 0.02  # Student-t(5) entries
    if outliers:
        w[:outliers] *= 60.0
    pts = _engine.gather_block_points(w.cuda(), bs, nblk, False, 0.0, False, _engine.L2)
    k_pad = _engine.round_up(K, _engine.CENT_TILE)
    C = torch.zeros(nblk, k_pad, bs, device="cuda")
    if forgy:
        idx = torch.randperm(n, generator=g)[:K].cuda()
        C[:, :K] = pts.X[:, idx]
    else:
        C[:, :K] = (torch.randn(nblk, K, bs, generator=g) * 0.02).cuda()
    if dup:
        C[:, 1] = C[:, 0]
        C[:, K - 1] = C[:, 5]
        C[:, 7] = C[:, 3]
    k_dev = torch.full((nblk,), K, dtype=torch.int32, device="cuda")
    B = torch.empty(nblk, k_pad * pts.kp, device="cuda")
    cnorm = torch.empty(nblk, k_pad, device="cuda")
    call("skcq_pack_centroids", _engine.L2, ptr(C), nblk, k_pad, bs, ptr(k_dev), None, ptr(B), ptr(cnorm), stream())
    return pts, C, B, cnorm, k_pad, k_dev


def _exact(pts, C, cnorm, k_pad, k_dev):
    from skcq_b200 import _engine
    from skcq_b200._lib import call, ptr, stream

    lab = torch.full((pts.nblk, pts.n_pad), -5, dtype=torch.int32, device="cuda")
    call("skcq_assign_exact", _engine.L2, ptr(pts.X), ptr(C), ptr(cnorm), pts.nblk, pts.n_pad, k_pad, pts.bs,
         ptr(pts.n), ptr(k_dev), None, ptr(lab), stream())
    return lab


@pytest.mark.parametrize("bs,K,n,nblk,forgy,dup,outliers", [
    (4, 8192, 12288, 3, True, False, 0),
    (4, 65536, 98304, 2, True, True, 40),    # the layer's second residual: Forgy seeds, 98,304 points
    (4, 65536, 98304, 2, False, False, 0),
    (4, 20000, 30001, 2, False, True, 25),   # K not a power of the cell count
    (3, 10000, 20000, 2, False, True, 10),
    (2, 9000, 30000, 2, True, False, 10),
])
def test_grid_labels_equal_exact_scan(bs, K, n, nblk, forgy, dup, outliers):
    from skcq_b200 import _engine

    pts, C, B, cnorm, k_pad, k_dev = _setup(nblk, n, bs, K, seed=bs * 100 + K % 97, forgy=forgy, dup=dup,
                                            outliers=outliers)
    assert _engine.GRID and k_pad >= _engine.GRID_MIN_K
    labels = torch.full((nblk, pts.n_pad), -9, dtype=torch.int32, device="cuda")
    _engine.GRID_STATS.update(enabled=True, points=0.0, fallback=0.0)
    try:
        _engine.assign_call(pts, B, C, cnorm, k_pad, k_dev, None, labels)
        stats = dict(_engine.GRID_STATS)
    finally:
        _engine.GRID_STATS["enabled"] = False
    ref = _exact(pts, C, cnorm, k_pad, k_dev)
    torch.cuda.synchronize()
    # certified points carry the exact scan's label; the few searched by the
    # tensor-core pass may differ only inside its rounding (relative gap <= 1e-5)
    bad = (labels[:, :n] != ref[:, :n]).nonzero()
    assert len(bad) <= stats["fallback"], len(bad)
    for b, i in bad.tolist():
        x = pts.X[b, i].double()
        s = [float(2 * (x @ C[b, c].double()) - C[b, c].double() @ C[b, c].double())
             for c in (int(labels[b, i]), int(ref[b, i]))]
        assert abs(s[0] - s[1]) <= 1e-5 * (abs(s[0]) + abs(s[1])), (b, i, s)
    assert stats["points"] == nblk * n
    assert stats["fallback"] <= 0.15 * stats["points"], stats  # the grid does most of the work
    if outliers:
        assert stats["fallback"] >= outliers, stats  # the far points went to the full search


def test_grid_abi_certifies_flags_and_checks():
    """Through the C ABI: certified points carry the exact scan's label; an
    inactive problem is left untouched; a problem with a non-finite centroid
    certifies nothing; bad arguments are rejected."""
    from skcq_b200 import _engine, _lib
    from skcq_b200._lib import call, ptr, stream

    nblk, n, bs, K = 3, 20000, 4, 16384
    pts, C, B, cnorm, k_pad, k_dev = _setup(nblk, n, bs, K, seed=7, forgy=False)
    ref = _exact(pts, C, cnorm, k_pad, k_dev)
    C2 = C.clone()
    C2[2, 10, 1] = float("nan")
    cn2 = cnorm.clone()
    lib = _lib.load()
    G = _engine.grid_cells(bs, k_pad)
    nbytes = int(lib.skcq_assign_grid_scratch_bytes(nblk, pts.n_pad, k_pad, bs, G))
    assert nbytes > 0
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    unres = torch.full((nblk, pts.n_pad), 7, dtype=torch.uint8, device="cuda")
    labels = torch.full((nblk, pts.n_pad), -3, dtype=torch.int32, device="cuda")
    active = torch.tensor([1, 0, 1], dtype=torch.int32, device="cuda")
    call("skcq_assign_grid", ptr(pts.X), ptr(C2), ptr(cn2), nblk, pts.n_pad, k_pad, bs, ptr(pts.n), ptr(k_dev),
         ptr(active), G, 3, ptr(labels), ptr(unres), ptr(scratch), nbytes, stream())
    _lib.poll_device_error()
    torch.cuda.synchronize()
    u0 = unres[0, :n]
    assert set(u0.unique().tolist()) <= {0, 1}
    cert = u0 == 0
    assert cert.float().mean().item() > 0.85
    assert torch.equal(labels[0, :n][cert], ref[0, :n][cert])
    assert (labels[0, :n][~cert] == -3).all()
    assert (unres[1] == 7).all() and (labels[1] == -3).all()
    assert (unres[2, :n] == 1).all() and (labels[2] == -3).all()
    with pytest.raises(RuntimeError):
        call("skcq_assign_grid", ptr(pts.X), ptr(C), ptr(cnorm), nblk, pts.n_pad, k_pad, 5, ptr(pts.n), ptr(k_dev),
             None, G, 3, ptr(labels), ptr(unres), ptr(scratch), nbytes, stream())
    with pytest.raises(RuntimeError):
        call("skcq_assign_grid", ptr(pts.X), ptr(C), ptr(cnorm), nblk, pts.n_pad, k_pad, bs, ptr(pts.n), ptr(k_dev),
             None, G, 3, ptr(labels), ptr(unres), ptr(scratch), nbytes - 256, stream())
    with pytest.raises(RuntimeError):
        call("skcq_assign_grid", ptr(pts.X), ptr(C), ptr(cnorm), nblk, pts.n_pad, k_pad, bs, ptr(pts.n), ptr(k_dev),
             None, G, 1, ptr(labels), ptr(unres), ptr(scratch), nbytes, stream())
    assert lib.skcq_assign_grid_scratch_bytes(nblk, pts.n_pad, k_pad, bs, 1) == 0
