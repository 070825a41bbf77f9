"""Host-side choice between an incremental and a full k-means assignment
(skcq_b200/_engine.py plan_incremental): which form, which scan for the moved
centroids, and the padded sizes the kernels are launched with. No GPU."""

from __future__ import annotations

import numpy as np

from skcq_b200 import _engine

N, K = 98304, 4096


def _plan(m, p, bs=8, kp=24, keep=0.5, calibrated=False, ratio=1.0, force=False, nblk=8, k=K, n=N):
    return _engine.plan_incremental(np.full(nblk, m), np.full(nblk, p), np.full(nblk, n), np.full(nblk, k), bs, kp,
                                    keep, calibrated, ratio, force)


def test_few_moved_centroids_take_the_exact_scan():
    plan = _plan(m=60, p=1500)
    assert plan is not None
    m_pad, p_pad, work, est = plan
    assert m_pad == -128  # exact CUDA-core scan of lists padded to one tile
    assert p_pad == 1536 and p_pad % _engine.ROWS_PER_UNIT == 0
    assert work == 2.0 * 8 * 8 * (N * 60 + 1500 * K)
    assert est > 0


def test_many_moved_centroids_take_the_tensor_core_pass_or_a_full_one():
    plan = _plan(m=1200, p=20000)
    assert plan is not None and plan[0] == 1280  # tensor-core pass over 10 tiles of moved centroids
    assert _plan(m=4000, p=90000) is None  # nearly everything moved: a full pass


def test_nothing_moved():
    plan = _plan(m=0, p=0)
    assert plan is not None and plan[:3] == (0, 0, 0.0)


def test_measured_ratio_and_force():
    base = _plan(m=1500, p=30000, calibrated=True, ratio=1.0)
    assert base is not None
    assert _plan(m=1500, p=30000, calibrated=True, ratio=4.0) is None  # incremental passes measured slow
    assert _plan(m=4000, p=90000, force=True) is not None  # tests force the incremental form


def test_keep_share_scales_the_listed_points():
    # points on moved centroids that the moved-centroid pass resolves need no full search
    assert _plan(m=300, p=60000, keep=1.0) is None
    assert _plan(m=300, p=60000, keep=0.1) is not None


def test_large_codebooks_favour_incremental_passes():
    # K = 65536: one full pass is 512 tiles per point, so even 5 % moved centroids pay
    plan = _plan(m=3300, p=6000, bs=4, kp=16, k=65536)
    assert plan is not None and plan[0] > 0


def test_empty_selection():
    assert _engine.plan_incremental(np.zeros(0), np.zeros(0), np.zeros(0), np.zeros(0), 8, 24, 0.5, False,
                                    1.0) is None
