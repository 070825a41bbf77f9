"""Row-sharded AQLM fit (skcq_b200/distributed.py) against the single-process
fit of the same matrix: two gloo ranks sharing one GPU (no kernel waits on
another rank, so this is safe on one device), then two NCCL ranks when two
GPUs are visible."""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _aqlm():
    from skcq_b200 import codebook as cb

    prim = cb.SSVQCodebook(cb.SphericalCodebook(cb.SphericalCodebookConfig(
        block_size=4, K=48, max_iters=15, norm_threshold=1e-9, skip_zeros=False)))
    res = [cb.EuclideanCodebook(cb.EuclideanCodebookConfig(block_size=4, K=32, max_iters=15, norm_threshold=1e-9,
                                                           skip_zeros=False))]
    return cb.AQLMCodebook(prim, res, cb.AQLMCodebookConfig(norm_threshold=1e-9))


def _worker(rank: int, world: int, port: int, backend: str, out_dir: str) -> None:
    import torch.distributed as dist

    from skcq_b200 import distributed as D
    from skcq_b200.codebook.events import KmeansDoneEvent, KmeansIterEvent

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank if backend == "nccl" else 0)
    torch.cuda.set_device(dev)
    dist.init_process_group(backend, rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(11)
        E, out_dim, in_dim = 12, 8, 16
        w = (torch.randn(E * out_dim, in_dim, generator=g) * 0.1).cuda()
        w[5, :4] = 0  # a zero block point
        torch.manual_seed(5)
        ref = _aqlm()
        ref_cwr = ref.fit(w)
        r0, r1 = D.expert_row_range(E, out_dim, world, rank)
        torch.manual_seed(5)
        sh = _aqlm()
        iters, done = [], []
        sh.on(KmeansIterEvent, iters.append)
        sh.on(KmeansDoneEvent, done.append)
        with D.row_sharded():
            cwr = sh.fit(w[r0:r1])
        ref_done = []
        torch.manual_seed(5)
        ref2 = _aqlm()
        ref2.on(KmeansDoneEvent, ref_done.append)
        ref2.fit(w)
        res = {
            "prim_cent": (sh.primary.inner.directions.float() - ref.primary.inner.directions.float()).abs().max().item(),
            "res_cent": (sh.residuals[0].centroids.float() - ref.residuals[0].centroids.float()).abs().max().item(),
            "idx0": (cwr.primary.inner.idxs == ref_cwr.primary.inner.idxs[:, r0:r1]).float().mean().item(),
            "idx1": (cwr.residuals[0].idxs == ref_cwr.residuals[0].idxs[:, r0:r1]).float().mean().item(),
            "signs": bool(torch.equal(cwr.primary.signs, ref_cwr.primary.signs[r0:r1])),
            "recon": ((sh.reconstruct(cwr) - ref.reconstruct(ref_cwr)[r0:r1]).norm()
                      / ref.reconstruct(ref_cwr)[r0:r1].norm()).item(),
            "iters": [d.iters_run for d in done] == [d.iters_run for d in ref_done],
            "reseeds": sum(e.n_empty for e in iters),
        }
        torch.save(res, os.path.join(out_dir, f"{backend}{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _check(out_dir, backend, world):
    for r in range(world):
        res = torch.load(os.path.join(out_dir, f"{backend}{r}.pt"))
        assert res["prim_cent"] < 1e-5 and res["res_cent"] < 1e-5, res
        assert res["idx0"] > 0.98 and res["idx1"] > 0.98, res
        assert res["signs"] and res["iters"], res
        assert res["recon"] < 1e-3, res
        assert res["reseeds"] > 0, "the case must exercise the cross-rank reseed"


def test_row_sharded_fit_matches_single_process_gloo(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), "gloo", str(tmp_path)), nprocs=2, join=True)
    _check(str(tmp_path), "gloo", 2)


def test_row_sharded_fit_matches_single_process_nccl(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_worker, args=(2, _free_port(), "nccl", str(tmp_path)), nprocs=2, join=True)
    _check(str(tmp_path), "nccl", 2)


def _worker_grid(rank: int, world: int, port: int, out_dir: str) -> None:
    """A euclidean bs=4 codebook with K = 8192, whose assignments take the
    centroid grid: the row-sharded fit against the single-process one."""
    import torch.distributed as dist

    from skcq_b200 import codebook as cb
    from skcq_b200 import distributed as D
    from skcq_b200.codebook.events import KmeansDoneEvent

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(21)
        E, out_dim, in_dim = 16, 1024, 8
        z = torch.randn(E * out_dim, in_dim, generator=g)
        chi2 = torch.randn(5, E * out_dim, in_dim, generator=g).square().sum(0)
        w = (z / torch.sqrt(chi2 / 5.0) * 0.02).cuda()

        def make():
            return cb.EuclideanCodebook(cb.EuclideanCodebookConfig(block_size=4, K=8192, max_iters=6,
                                                                   norm_threshold=1e-9, skip_zeros=False))

        torch.manual_seed(7)
        ref = make()
        ref_done = []
        ref.on(KmeansDoneEvent, ref_done.append)
        ref_cwr = ref.fit(w)
        r0, r1 = D.expert_row_range(E, out_dim, world, rank)
        torch.manual_seed(7)
        sh = make()
        done = []
        sh.on(KmeansDoneEvent, done.append)
        with D.row_sharded():
            cwr = sh.fit(w[r0:r1])
        res = {
            "cent": (sh.centroids.float() - ref.centroids.float()).abs().max().item(),
            "idx": (cwr.idxs == ref_cwr.idxs[:, r0:r1]).float().mean().item(),
            "iters": [d.iters_run for d in done] == [d.iters_run for d in ref_done],
        }
        torch.save(res, os.path.join(out_dir, f"grid{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_row_sharded_grid_fit_matches_single_process_gloo(tmp_path):
    """The centroid-grid assignment inside a row-sharded fit (each rank grids
    its own points against the shared centroids)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import torch.multiprocessing as mp

    mp.spawn(_worker_grid, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        res = torch.load(os.path.join(str(tmp_path), f"grid{r}.pt"))
        assert res["cent"] < 1e-5 and res["idx"] > 0.999 and res["iters"], res
