"""Expert-parallel CodebookExperts across ranks (one process per GPU).

Rank r of a ``world``-rank group holds experts [e0, e1) of every projection
(``expert_row_range`` split: whole experts, as even as possible) and the shared
per-block codebook tables. A forward on each rank's own tokens:

1. pairs (token, slot) are grouped by the rank that owns their expert, in
   pair order (p = kpos * T + token) within each destination;
2. one all-to-all of the per-rank pair counts, then one all-to-all of the
   pairs' hidden rows and expert ids (NCCL over NVLink; gloo through host
   copies);
3. each rank runs its experts on the rows it received with the local
   ``CodebookExperts`` forward, each row a top-1 route of weight 1 (the decode
   gather kernels or the tcgen05 prefill path, by batch size);
4. a second all-to-all returns the expert outputs, and the weighted combine
   adds each token's k outputs in ascending (expert, kpos) order -- the
   ``index_add_`` order of codebook_experts.py:467-480.

Every rank must call ``forward`` the same number of times (the all-to-alls are
collectives); a rank with no tokens passes a (0, H) batch.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist

from skcq_b200 import _lib
from skcq_b200._lib import call, ptr, stream
from skcq_b200.codebook_experts import _DTYPE, CodebookExperts, CodebookModule, _as_rows
from skcq_b200.distributed import expert_row_range


class ExpertParallelExperts(torch.nn.Module):
    """``CodebookExperts.forward`` semantics with experts placed across ranks.
    ``check_errors`` (default on) reads the device error word once at the end
    of each call, so an expert id outside [0, num_experts) raises."""

    check_errors: bool = True

    def __init__(self, gate: CodebookModule, up: CodebookModule, down: CodebookModule, num_experts: int,
                 act_fn: Callable[[torch.Tensor], torch.Tensor], group: dist.ProcessGroup | None = None) -> None:
        super().__init__()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.num_experts = num_experts
        self.host_staged = dist.get_backend(group) == "gloo"
        self.bounds = [expert_row_range(num_experts, 1, self.world, r) for r in range(self.world)]
        e0, e1 = self.bounds[self.rank]
        self.e0, self.e1 = e0, e1
        local = [m.slice_experts(e0, e1) if m.primary.assignments.shape[0] == num_experts else m
                 for m in (gate, up, down)]
        self.local = CodebookExperts(local[0], local[1], local[2], e1 - e0, act_fn)
        self.local.check_errors = False
        owner = torch.empty(num_experts, dtype=torch.int64)
        for r, (a, b) in enumerate(self.bounds):
            owner[a:b] = r
        self.register_buffer("owner", owner, persistent=False)

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int]) -> None:
        if self.host_staged:
            o, i = out.cpu(), inp.cpu()
            dist.all_to_all_single(o, i, out_splits, in_splits, group=self.group)
            out.copy_(o)
        else:
            dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                top_k_weights: torch.Tensor) -> torch.Tensor:
        dev = self.local.gate.primary.codebook.device
        if dev.type != "cuda":
            raise RuntimeError("ExpertParallelExperts needs its modules on a CUDA device")
        h = _as_rows(hidden_states.to(dev))
        T, H = h.shape
        k = top_k_index.shape[1]
        P = T * k
        topk = top_k_index.to(device=dev, dtype=torch.int64).contiguous()
        w = top_k_weights.to(dev)
        if w.dtype not in (torch.float32, torch.bfloat16):
            w = w.float()
        w = w.contiguous()
        # 1. pairs in pair order p = kpos * T + token, grouped by destination rank
        # (an id outside [0, E) is routed by its clamped value and then flagged
        # by the owning rank's route sort, raising at the end of the call)
        expert = topk.t().reshape(-1)
        if P:  # the sender flags its own out-of-range ids too (no host sync)
            chk = torch.empty(P, dtype=torch.int16, device=dev)
            call("skcq_pack_indices16", ptr(topk), P, self.num_experts, ptr(chk), stream())
        dest = self.owner.to(dev)[expert.clamp(0, self.num_experts - 1)]
        order = torch.sort(dest, stable=True).indices
        send_counts = torch.bincount(dest, minlength=self.world)
        # 2. counts, then rows and expert ids
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, [1] * self.world, [1] * self.world)
        s_split, r_split = send_counts.tolist(), recv_counts.tolist()
        n_recv = sum(r_split)
        tokens = order % T if T else order
        send_rows = h[tokens]
        send_ids = expert[order]
        recv_rows = torch.empty(n_recv, H, dtype=h.dtype, device=dev)
        recv_ids = torch.empty(n_recv, dtype=torch.int64, device=dev)
        self._a2a(recv_rows, send_rows, r_split, s_split)
        self._a2a(recv_ids, send_ids, r_split, s_split)
        # 3. the local experts, one top-1 route per received row
        if n_recv:
            ones = torch.ones(n_recv, 1, dtype=torch.float32, device=dev)
            y = self.local(recv_rows, (recv_ids - self.e0)[:, None], ones)
        else:
            y = torch.empty(0, H, dtype=h.dtype, device=dev)
        # 4. outputs back, then the weighted combine in (expert, kpos) order
        back = torch.empty(P, H, dtype=y.dtype, device=dev)
        self._a2a(back, y.contiguous(), s_split, r_split)
        y_pairs = torch.empty_like(back)
        y_pairs[order] = back
        out = torch.empty(T, H, dtype=h.dtype, device=dev)
        if P:
            row_of_pair = torch.arange(P, dtype=torch.int32, device=dev)
            call("skcq_combine", ptr(y_pairs), _DTYPE[y_pairs.dtype], 1, P, ptr(row_of_pair), ptr(topk), ptr(w),
                 _DTYPE[w.dtype], T, k, H, ptr(out), _DTYPE[out.dtype], stream())
        else:
            out.zero_()
        if self.check_errors:
            _lib.poll_device_error()
        return out.to(device=hidden_states.device, dtype=hidden_states.dtype)
