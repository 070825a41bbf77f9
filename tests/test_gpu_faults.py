"""Failure detection on the GPU without a GPU fault: a bounded device wait is
made to run out (a barrier nothing arrives on), the kernel returns, the host
reads the error status, and the CUDA context keeps working."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def test_bounded_wait_runs_out_and_the_context_stays_usable():
    from skcq_b200 import _lib
    from skcq_b200._lib import stream
    from skcq_b200.errors import DeviceTimeoutError, InfrastructureError

    lib = _lib.load()
    _lib.poll_device_error()  # start clean
    # about a millisecond of SM clocks: the wait gives up, records the code, returns
    assert lib.skcq_selftest_wait_timeout(2_000_000, stream()) == 0
    torch.cuda.synchronize()
    with pytest.raises(DeviceTimeoutError) as ei:
        _lib.poll_device_error()
    assert ei.value.code == 90 and isinstance(ei.value, InfrastructureError)
    _lib.poll_device_error()  # the poll cleared the word
    # the context still computes: a small assignment against the exact path
    from skcq_b200 import _engine

    g = torch.Generator().manual_seed(0)
    w = (torch.randn(1000, 8, generator=g) * 0.05).cuda()
    pts = _engine.gather_block_points(w, 4, 2, False, 0.0, False, _engine.L2)
    k_pad = _engine.round_up(64, _engine.CENT_TILE)
    C = torch.zeros(2, k_pad, 4, device="cuda")
    C[:, :64] = (torch.randn(2, 64, 4, generator=g) * 0.05).cuda()
    run = _engine.KmeansRun(C=C, k_pad=k_pad, k_host=[64, 64], labels=None, iters_run=[], converged=[],
                            moved=None, n_empty=None, cnorm=torch.empty(2, k_pad, device="cuda"))
    lab = _engine.assign(pts, run)
    torch.cuda.synchronize()
    _lib.poll_device_error()
    d = ((w.reshape(1000, 2, 1, 4).cpu() - C[:, :64].cpu()[None]) ** 2).sum(-1)  # (1000, 2, 64)
    ref = d.argmin(-1).T
    assert (lab[:, :1000].cpu() == ref).float().mean() > 0.99


def test_selftest_rejects_an_out_of_range_limit():
    from skcq_b200 import _lib
    from skcq_b200._lib import stream

    assert _lib.load().skcq_selftest_wait_timeout(0, stream()) == -1
    assert "limit" in _lib.last_error()
