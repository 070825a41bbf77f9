"""The allocation-free reseed entry point, for callers that cannot allocate.

Hosts that own all device memory through their own allocator (and forbid
cudaMalloc), or plug-in interfaces that only receive a step's inputs and
outputs, cannot provide the scratch buffer skcq_reseed asks for.
skcq_reseed_noalloc serves them from a fixed array inside the library. This
file checks, through the C ABI, that it produces exactly what skcq_reseed
produces, on two calls in a row with different problem sets (the array is
shared between calls and must not carry anything over), and that oversized
problems are rejected. It is named to be collected last.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _problem(metric: int, nblk: int, n: int, bs: int, K: int, seed: int):
    """A problem set after assignment and update, with many empty clusters."""
    from skcq_b200 import _engine
    from skcq_b200._lib import call, ptr, stream

    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, nblk * bs, generator=g) * 0.05).cuda()
    pts = _engine.gather_block_points(w, bs, nblk, False, 0.0, False, metric)
    k_pad = _engine.round_up(K, _engine.CENT_TILE)
    C = torch.zeros(nblk, k_pad, bs, device="cuda")
    c = torch.randn(nblk, K, bs, generator=g) * 0.05
    if metric == _engine.COSINE:
        c = torch.nn.functional.normalize(c, dim=-1)
    C[:, :K] = c.cuda()
    cnorm = torch.empty(nblk, k_pad, device="cuda")
    run = _engine.KmeansRun(C=C, k_pad=k_pad, k_host=[K] * nblk, labels=None, iters_run=[], converged=[],
                            moved=None, n_empty=None, cnorm=cnorm)
    labels = _engine.assign(pts, run)
    k = torch.full((nblk,), K, dtype=torch.int32, device="cuda")
    sums = torch.zeros(nblk, k_pad, bs, device="cuda")
    counts = torch.zeros(nblk, k_pad, dtype=torch.int32, device="cuda")
    call("skcq_update", ptr(pts.R), ptr(labels), nblk, pts.n_pad, k_pad, bs, ptr(pts.n), ptr(k), None, ptr(sums),
         ptr(counts), None, stream())
    return pts, C, labels, k, k_pad, sums, counts


def _reseed_both(metric: int, nblk: int, n: int, bs: int, K: int, seed: int):
    from skcq_b200 import _lib
    from skcq_b200._lib import call, ptr, stream

    pts, C, labels, k, k_pad, sums, counts = _problem(metric, nblk, n, bs, K, seed)
    s_ref, s_new = sums.clone(), sums.clone()
    e_ref = torch.zeros(nblk, dtype=torch.int32, device="cuda")
    e_new = torch.full((nblk,), -7, dtype=torch.int32, device="cuda")
    scratch = torch.empty(int(_lib.load().skcq_reseed_scratch_bytes(nblk, k_pad)), dtype=torch.uint8, device="cuda")
    call("skcq_reseed", metric, ptr(pts.X), ptr(C), ptr(labels), nblk, pts.n_pad, k_pad, bs, ptr(pts.n), ptr(k),
         None, ptr(s_ref), ptr(counts), ptr(e_ref), ptr(scratch), stream())
    call("skcq_reseed_noalloc", metric, ptr(pts.X), ptr(C), ptr(labels), nblk, pts.n_pad, k_pad, bs, ptr(pts.n),
         ptr(k), None, ptr(s_new), ptr(counts), ptr(e_new), stream())
    _lib.poll_device_error()
    return s_ref.cpu(), s_new.cpu(), e_ref.cpu(), e_new.cpu()


def test_noalloc_reseed_matches_reseed_on_two_calls_in_a_row():
    # first call: cosine, 5 problems; second call: euclidean with different
    # shapes; third: K = 65536 (768 KiB of scratch per problem, so only 21
    # problems fit the static array at once and CTAs reuse their slot for
    # several problems), with more empty clusters than the shared-memory sort
    # holds, so the sort runs in the static array (n >= K, as in any fit)
    for metric, nblk, n, bs, K, seed in ((0, 5, 3000, 8, 2048, 1), (1, 3, 6000, 4, 4000, 2),
                                         (1, 32, 70000, 4, 65536, 3)):
        s_ref, s_new, e_ref, e_new = _reseed_both(metric, nblk, n, bs, K, seed)
        assert int(e_ref.min()) > 0, "the case must have empty clusters"
        if K == 65536:
            assert int(e_ref.min()) > 4096, "the case must reach the sort outside shared memory"
        assert torch.equal(e_ref, e_new)
        assert torch.equal(s_ref, s_new)  # same selection and order, bit for bit


def test_noalloc_reseed_rejects_problems_over_the_static_limit():
    from skcq_b200 import _lib
    from skcq_b200._lib import ptr, stream

    t = torch.zeros(16, device="cuda")
    i = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = _lib.load().skcq_reseed_noalloc(0, ptr(t), ptr(t), ptr(i), 1, 256, 1 << 22, 4, ptr(i), ptr(i), None,
                                         ptr(t), ptr(i), ptr(i), stream())
    assert rc == -1
    assert "static buffer" in _lib.last_error()
