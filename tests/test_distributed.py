"""Host logic of the row-sharded fit (skcq_b200/distributed.py) on CPU gloo
ranks: row ranges, global counts, Forgy ownership, the reseed candidate merge
and the flip-flag OR give the single-process answers."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from skcq_b200 import distributed as D


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        nblk, bs, k_pad = 3, 4, 8
        n_global = torch.tensor([10, 7, 0])
        # rank r holds points [r0, r1) of every problem (same split for all problems here)
        split = [torch.tensor([6, 3, 0]), torch.tensor([4, 4, 0])]
        X_glob = torch.randn(nblk, 10, bs, generator=g)
        n_loc = split[rank]
        lo = split[0] if rank == 1 else torch.zeros(3, dtype=torch.int64)
        n_pad = 16
        X = torch.zeros(nblk, n_pad, bs)
        for b in range(nblk):
            X[b, : n_loc[b]] = X_glob[b, lo[b] : lo[b] + n_loc[b]]
        with D.row_sharded() as sh:
            assert D.current() is sh and sh.world == world
            ng, gofs = D.global_counts(sh, n_loc.to(torch.int32))
            assert ng.tolist() == n_global.tolist() and gofs.tolist() == lo.tolist()
            # Forgy: perm over global indices, owners contribute, the sum is the gather
            perm = torch.zeros(nblk, k_pad, dtype=torch.int64)
            perm[0, :5] = torch.tensor([9, 0, 5, 6, 2])
            perm[1, :3] = torch.tensor([6, 1, 3])
            k = torch.tensor([5, 3, 0], dtype=torch.int32)
            C = D.owned_init(X, perm, k, gofs, n_loc.to(torch.int32))
            sh.all_reduce_sum_(C)
            ref = torch.zeros(nblk, k_pad, bs)
            ref[0, :5] = X_glob[0, perm[0, :5]]
            ref[1, :3] = X_glob[1, perm[1, :3]]
            assert torch.equal(C, ref)
            # reseed merge: keys = (score << 32 | global index) ^ 2^63; each rank sends its local worst m
            scores = torch.randint(0, 5, (nblk, 10), generator=g)  # many equal scores: ties by index
            gidx = torch.arange(10)[None, :].expand(nblk, 10)
            keys_glob = ((scores << 32) | gidx) ^ (-(1 << 63))
            counts = torch.ones(nblk, k_pad, dtype=torch.int32)
            counts[0, [1, 4, 6]] = 0
            counts[1, [0, 2]] = 0
            active = torch.tensor([1, 1, 0], dtype=torch.int32)
            k2 = torch.tensor([8, 5, 8], dtype=torch.int32)
            empty = D.empty_clusters(counts, k2, active)
            assert empty.sum(1).tolist() == [3, 2, 0]
            m = 3
            keys = torch.full((nblk, m), D.INT64_MAX, dtype=torch.int64)
            vecs = torch.zeros(nblk, m, bs)
            for b in range(2):
                loc = keys_glob[b, lo[b] : lo[b] + n_loc[b]]
                order = torch.argsort(loc)[: min(int(empty[b].sum()), int(n_loc[b]))]
                keys[b, : len(order)] = loc[order]
                vecs[b, : len(order)] = X[b, order]
            sums = torch.zeros(nblk, k_pad, bs)
            D.merge_reseed(sh.all_gather(keys), sh.all_gather(vecs), empty, sums)
            ref = torch.zeros(nblk, k_pad, bs)
            for b, cl in ((0, [1, 4, 6]), (1, [0, 2])):
                worst = torch.argsort(keys_glob[b, : n_global[b]])[: len(cl)]
                ref[b, cl] = X_glob[b, worst]
            assert torch.equal(sums, ref)
            flags = torch.tensor([1 << rank, 0, -(1 << 63) if rank == 1 else 0], dtype=torch.int64)
            assert D.or_over_ranks(sh, flags).tolist() == [3, 0, -(1 << 63)]
            # the incremental assignment's change marks: a cluster changed if it
            # changed on any rank
            changed = torch.zeros(nblk, k_pad, dtype=torch.uint8)
            changed[0, rank] = 1
            changed[2, 5] = 1
            sh.all_reduce_max_(changed)
            ref = torch.zeros(nblk, k_pad, dtype=torch.uint8)
            ref[0, :2] = 1
            ref[2, 5] = 1
            assert torch.equal(changed, ref)
        assert D.current() is None
        torch.save({"ok": True}, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_row_shard_host_logic_two_ranks(tmp_path):
    port = _free_port()
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert torch.load(tmp_path / f"r{r}.pt")["ok"]


@pytest.mark.parametrize("E,world", [(128, 8), (128, 3), (5, 2), (3, 4)])
def test_expert_row_range_partitions(E, world):
    ranges = [D.expert_row_range(E, 768, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == E * 768
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [(b - a) // 768 for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1 and all((b - a) % 768 == 0 for a, b in ranges)
