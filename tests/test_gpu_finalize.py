"""skcq_finalize (kmeans.py:174-188 cosine, 231-244 euclidean): the vectorised
kernel taken for block sizes 4, 6, 8, 12 and 16 leaves every output with the
same bits as the scalar kernel (taken when the sum or centroid slice is not
16-byte aligned) on the same state: centroids, zeroed sums and counts, the
changed marks, moved, the empty-cluster history, iterations and convergence."""

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


def _offset(t: torch.Tensor) -> torch.Tensor:
    """A copy of t that starts 4 bytes past a 16-byte boundary."""
    buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
    v = buf[1:].view(t.shape)
    v.copy_(t)
    return v


@pytest.mark.parametrize("with_changed", [False, True])
@pytest.mark.parametrize("bs", [4, 6, 8, 12, 16])
@pytest.mark.parametrize("metric", [0, 1])
def test_finalize_vector_form_matches_scalar(metric, bs, with_changed):
    from skcq_b200._lib import call, ptr, stream

    nblk, k_pad, it, iters = 6, 1280, 2, 4
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(100 * bs + 10 * metric + int(with_changed))
    kvec = torch.tensor([1280, 1000, 777, 1, 1280, 300], dtype=torch.int32, device=dev)
    sums = torch.randn(nblk, k_pad, bs, generator=g, device=dev)
    C = torch.randn(nblk, k_pad, bs, generator=g, device=dev)
    counts = torch.randint(0, 4, (nblk, k_pad), generator=g, device=dev, dtype=torch.int32)
    # clusters whose recomputed value equals the old centroid bit for bit
    # (a single member / a reseeded point equal to it): not marked moved
    same = torch.rand(nblk, k_pad, generator=g, device=dev) < 0.2
    counts[same] = torch.where(counts[same] > 0, 1, 0).int()
    sums[same] = C[same] if metric == 1 else torch.nn.functional.normalize(sums[same], dim=-1)
    if metric == 0:
        C[same] = sums[same] / torch.clamp(sums[same].norm(dim=-1, keepdim=True), min=1e-12)
    changed = (torch.rand(nblk, k_pad, generator=g, device=dev) < 0.5).to(torch.uint8)
    changed[3] = 0
    counts[3, 0] = 2  # problem 3: its one cluster kept its members -> moved 0, converged
    active = torch.tensor([1, 1, 1, 1, 0, 1], dtype=torch.int32, device=dev)
    n_empty = torch.randint(0, 9, (nblk,), generator=g, device=dev, dtype=torch.int32)

    outs = []
    for aligned in (True, False):
        s = sums.clone() if aligned else _offset(sums)
        c = C.clone() if aligned else _offset(C)
        if aligned:
            assert s.data_ptr() % 16 == 0 and c.data_ptr() % 16 == 0
        else:
            assert s.data_ptr() % 16 != 0 and c.data_ptr() % 16 != 0
        st = {
            "sums": s, "C": c, "counts": counts.clone(), "active": active.clone(),
            "converged": torch.zeros(nblk, dtype=torch.int32, device=dev),
            "iters_run": torch.zeros(nblk, dtype=torch.int32, device=dev),
            "moved": torch.full((iters, nblk), -1.0, device=dev),
            "nempty": torch.full((iters, nblk), -1, dtype=torch.int32, device=dev),
            "changed": changed.clone() if with_changed else None,
        }
        call("skcq_finalize", metric, ptr(st["sums"]), ptr(st["counts"]), ptr(n_empty), nblk, k_pad, bs, ptr(kvec),
             ptr(st["active"]), ptr(st["converged"]), ptr(st["iters_run"]), ptr(st["moved"]), ptr(st["nempty"]),
             it, ptr(st["C"]), ptr(st["changed"]), stream())
        outs.append(st)
    torch.cuda.synchronize()
    a, b = outs
    for key in a:
        if a[key] is None:
            continue
        x, y = a[key].contiguous(), b[key].contiguous()
        if x.is_floating_point():
            x, y = x.view(torch.int32), y.view(torch.int32)
        assert torch.equal(x, y), key
    # the kept problem converged; the inactive one was not touched
    assert int(a["converged"][3]) == (1 if with_changed else int(a["moved"][it, 3] < 1e-6))
    assert float(a["moved"][it, 4]) == -1.0 and torch.equal(a["C"][4], C[4])
    live = (torch.arange(k_pad, device=dev)[None, :] < kvec[:, None]) & (active[:, None] != 0)
    assert int(a["counts"][live].abs().sum()) == 0 and float(a["sums"][live].abs().sum()) == 0.0
    assert torch.equal(a["counts"][~live], counts[~live])
