"""Expert-parallel CodebookExperts (skcq_b200/expert_parallel.py) against the
single-process forward on the same tokens: two gloo ranks sharing one GPU,
exchanging rows through CUDA IPC mappings of each other's buffers (no kernel
waits on another rank: the phases are separated by host barriers), fp32 small
batch (gather kernels) and bf16 large batch (tensor-core prefill on each
rank), the per-source row counts each rank received, an empty rank, an
invalid expert id and the capacity check."""

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


def _module(E, out_dim, in_dim, seed, dtype):
    from skcq_b200.codebook_experts import CodebookModule, _CodebookLayer

    g = torch.Generator().manual_seed(seed)
    layers = []
    for i, (bs, K) in enumerate([(8, 64), (4, 256)]):
        nb = in_dim // bs
        layers.append(_CodebookLayer(
            (torch.randn(nb, bs, K, generator=g) * 0.05).to(dtype), torch.randint(0, K, (E, nb, out_dim), generator=g),
            nb, bs, out_dim, K, scales=(torch.rand(E, nb, out_dim, generator=g) * 0.1).to(dtype) if i == 0 else None))
    return CodebookModule(torch.nn.ModuleList(layers), len(layers), out_dim).cuda()


def _worker(rank: int, world: int, port: int, out_dir: str, backend: str = "gloo", own_gpu: bool = False) -> None:
    import datetime

    import torch.distributed as dist

    from skcq_b200.codebook_experts import CodebookExperts
    from skcq_b200.expert_parallel import ExpertParallelExperts

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank if own_gpu else 0)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        res = {}
        E, H, I = 8, 64, 32
        for name, dtype, T, k in (("f32_small", torch.float32, 5, 2), ("bf16_large", torch.bfloat16, 2048, 2)):
            mods = [_module(E, I, H, 1, dtype), _module(E, I, H, 2, dtype), _module(E, H, I, 3, dtype)]
            full = CodebookExperts(*mods, E, torch.nn.functional.silu)
            ep = ExpertParallelExperts(*mods, E, torch.nn.functional.silu, max_tokens=2048, top_k=2)
            g = torch.Generator().manual_seed(100 + rank)  # each rank has its own tokens
            x = torch.randn(T, H, generator=g).to(dtype).cuda()
            topi = torch.rand(T, E, generator=g).argsort(-1)[:, :k].cuda()
            topw = torch.rand(T, k, generator=g).cuda()
            y_ep = ep(x, topi, topw).double()
            y_ref = full(x, topi, topw).double()
            cos = torch.nn.functional.cosine_similarity(y_ep.flatten(), y_ref.flatten(), dim=0).item()
            res[name] = ((y_ep - y_ref).abs().max().item() / y_ref.abs().max().item(), cos)
            # rows sent: one per (token, rank owning one of its experts), not one
            # per slot. The counts are read before the collective below, which
            # keeps the other rank's next dispatch from overwriting them first.
            o = ep._off[3]
            cnt = ep._bytes[o:o + 4 * world].view(torch.int32).cpu().tolist()
            owner = torch.tensor([0 if e < ep.bounds[1][0] else 1 for e in range(E)])
            sent = [int((owner[topi.cpu()] == d).any(1).sum()) for d in range(world)]
            got: list = [None] * world
            dist.all_gather_object(got, sent)
            res[name + "_counts"] = cnt == [got[s][rank] for s in range(world)]
            res[name + "_count_values"] = (cnt, [got[s][rank] for s in range(world)])
            res[name + "_dedup"] = sum(sent) < T * k or T * k == 0
            if name == "f32_small":
                ep.close()
        # a rank with no tokens still takes part in the collectives
        x0 = torch.randn(0 if rank == 1 else 3, 64, generator=torch.Generator().manual_seed(7)).cuda()
        t0 = torch.zeros(x0.shape[0], 2, dtype=torch.int64).cuda()
        t0[:, 1] = 5
        x0 = x0.to(torch.bfloat16)
        y0 = ep(x0, t0, torch.ones(x0.shape[0], 2).cuda())
        res["empty_ok"] = y0.shape == x0.shape and bool(torch.isfinite(y0).all())
        res["empty_detail"] = (tuple(y0.shape), tuple(x0.shape), y0.float().abs().max().item() if y0.numel() else 0.0)
        # an expert id outside [0, E) raises on the rank that passed it (after
        # the barriers, which every rank still takes)
        bad = torch.zeros(2, 2, dtype=torch.int64).cuda()
        bad[:, 1] = 1
        bad[0, 0] = 9 if rank == 0 else 0
        try:
            ep(torch.randn(2, 64).to(torch.bfloat16).cuda(), bad, torch.ones(2, 2).cuda())
            res["raised"] = False
        except RuntimeError:
            res["raised"] = True
        # more tokens than the buffers hold is refused on the host, before any collective
        try:
            ep(torch.randn(2049, 64).to(torch.bfloat16).cuda(), torch.zeros(2049, 2, dtype=torch.int64).cuda(),
               torch.ones(2049, 2).cuda())
            res["capacity_checked"] = False
        except ValueError:
            res["capacity_checked"] = True
        ep.close()
        torch.save(res, os.path.join(out_dir, f"ep{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _check(tmp_path) -> None:
    for r in range(2):
        res = torch.load(tmp_path / f"ep{r}.pt")
        assert res["f32_small"][0] < 1e-5 and res["f32_small"][1] > 0.999999, res
        assert res["bf16_large"][0] < 1e-2 and res["bf16_large"][1] > 0.9999, res
        assert res["f32_small_counts"] and res["bf16_large_counts"], (res["f32_small_count_values"],
                                                                      res["bf16_large_count_values"])
        assert res["bf16_large_dedup"], res
        assert res["empty_ok"] and res["capacity_checked"], (r, res["empty_ok"], res["empty_detail"],
                                                             res["capacity_checked"])
    # the id 9 of rank 0 is flagged by rank 0, which routed its other slot;
    # rank 1's inputs were valid
    assert torch.load(tmp_path / "ep0.pt")["raised"]
    assert not torch.load(tmp_path / "ep1.pt")["raised"]


def test_expert_parallel_matches_single_process(tmp_path):
    """Two gloo ranks sharing one GPU."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    _check(tmp_path)


@pytest.mark.parametrize("backend", ["gloo", "nccl"])
def test_expert_parallel_two_gpus(tmp_path, backend):
    """One rank per GPU: rows cross NVLink through the IPC mappings; the
    phases are ordered by a host barrier (gloo) or a one-element NCCL
    all-reduce on the stream (nccl)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), backend, True), nprocs=2, join=True)
    _check(tmp_path)
