"""Expert-parallel CodebookExperts across the GPUs of one node (one process per GPU).

Rank r of a ``world``-rank group holds experts [e0, e1) of every projection
(``expert_row_range`` split: whole experts, as even as possible) and the shared
per-block codebook tables. Every rank allocates one exchange buffer and maps the
other ranks' buffers through CUDA IPC (``csrc/expert_parallel.cu``). A forward
on each rank's own tokens:

1. ``skcq_ep_dispatch`` stores each token's row once into every rank that owns
   one of its experts (not once per top-k slot), with per slot the expert's
   local id there and the routing weight, and publishes the per-source row
   counts -- routing stays on the device, with no host synchronisation;
2. a stream-ordered barrier: a one-element all-reduce over NCCL (with gloo, a
   device synchronise and a host barrier);
3. each rank runs its experts on the rows it received (the decode gather
   kernels or the tcgen05 prefill path, by the batch's size), and
   ``skcq_ep_return`` writes, per received row, the weighted sum over its local
   slots in ascending (expert, slot) order straight into the source rank's
   buffer -- the combine of codebook_experts.py:467-480 restricted to this
   rank's experts, fused with the return transfer;
4. a second barrier, then ``skcq_ep_gather`` adds each token's returned sums in
   ascending rank order (ascending expert ranges).

The result equals the single-process forward up to the order of the fp32
additions across ranks and, for bf16 outputs, one bf16 rounding of each rank's
partial sum (the reference's bf16 ``index_add_`` rounds after every expert).

Every rank must call ``forward`` the same number of times (the barriers are
collectives) with hidden states of the same dtype; a rank with no tokens passes
a (0, H) batch. ``max_tokens`` bounds the tokens any rank passes to one call
and ``top_k`` the slots per token; both size the exchange buffers. ``close()``
(collective) releases the buffers.
"""

from __future__ import annotations

import ctypes as C
from collections.abc import Callable

import torch
import torch.distributed as dist

from skcq_b200 import _lib
from skcq_b200._lib import call, ptr, stream
from skcq_b200.codebook_experts import _DTYPE, CodebookExperts, CodebookModule, _as_rows
from skcq_b200.distributed import expert_row_range

MAX_RANKS = 8  # SKCQ_EP_MAX_RANKS


class _DeviceBytes:
    """A device byte range exposed through ``__cuda_array_interface__`` (so
    torch can view the IPC-exported buffer without copying)."""

    def __init__(self, address: int, nbytes: int) -> None:
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (address, False),
                                         "strides": None, "version": 2}


class ExpertParallelExperts(torch.nn.Module):
    """``CodebookExperts.forward`` semantics with experts placed across ranks.
    ``check_errors`` (default on) reads the device error word once at the end
    of each call, so an expert id outside [0, num_experts) raises on the rank
    that passed it."""

    check_errors: bool = True
    # record CUDA events between the phases (dispatch + barrier, local
    # experts, return + barrier, gather) into ``last_phases``
    record_phases: bool = False

    def __init__(self, gate: CodebookModule, up: CodebookModule, down: CodebookModule, num_experts: int,
                 act_fn: Callable[[torch.Tensor], torch.Tensor], group: dist.ProcessGroup | None = None,
                 max_tokens: int = 4096, top_k: int = 8) -> None:
        super().__init__()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"expert parallelism spans at most {MAX_RANKS} ranks (one node), got {self.world}")
        if num_experts < self.world:
            raise ValueError(f"{num_experts} experts cannot be split over {self.world} ranks")
        dev = gate.primary.codebook.device
        if dev.type != "cuda":
            raise RuntimeError("ExpertParallelExperts needs its modules on a CUDA device")
        self._dev = dev
        self.num_experts = num_experts
        self.nccl = dist.get_backend(group) == "nccl"
        self.bounds = [expert_row_range(num_experts, 1, self.world, r) for r in range(self.world)]
        e0, e1 = self.bounds[self.rank]
        self.e0, self.e1 = e0, e1
        local = [m.slice_experts(e0, e1) if m.primary.assignments.shape[0] == num_experts else m
                 for m in (gate, up, down)]
        self.local = CodebookExperts(local[0], local[1], local[2], e1 - e0, act_fn)
        self.local.check_errors = False
        self.capacity = int(max_tokens)
        self.top_k_cap = int(top_k)
        self.hidden = down.out_dim
        offs = (C.c_int64 * 6)()
        call("skcq_ep_layout", self.world, self.capacity, self.top_k_cap, self.hidden, offs)
        self._off = list(offs)
        handle = C.create_string_buffer(64)
        base = C.c_void_p()
        with torch.cuda.device(dev):
            call("skcq_ep_alloc", C.c_size_t(self._off[5]), C.byref(base), handle)
        self._base = base.value
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        peers, self._opened = [], []
        with torch.cuda.device(dev):
            for r, raw in enumerate(handles):
                if r == self.rank:
                    peers.append(self._base)
                    continue
                p = C.c_void_p()
                call("skcq_ep_open", C.create_string_buffer(raw, 64), C.byref(p))
                peers.append(p.value)
                self._opened.append(p.value)
        self._peers = (C.c_void_p * self.world)(*peers)
        self._bounds_arr = (C.c_int32 * (self.world + 1))(*([b[0] for b in self.bounds] + [num_experts]))
        self._bytes = torch.as_tensor(_DeviceBytes(self._base, self._off[5]), device=dev)
        self._flag = torch.zeros(1, dtype=torch.int32, device=dev)

    def _rows(self, dtype: torch.dtype) -> torch.Tensor:
        """The received token rows, (world * capacity, hidden) of ``dtype``."""
        n = self.world * self.capacity * self.hidden * (2 if dtype == torch.bfloat16 else 4)
        o = self._off[0]
        return self._bytes[o:o + n].view(dtype).view(self.world * self.capacity, self.hidden)

    def _barrier(self) -> None:
        if self.nccl:
            dist.all_reduce(self._flag, group=self.group)
        else:
            torch.cuda.synchronize(self._dev)
            dist.barrier(group=self.group)

    def close(self) -> None:
        """Collective: unmap the other ranks' buffers, then free this rank's."""
        if self._base is None:
            return
        torch.cuda.synchronize(self._dev)
        dist.barrier(group=self.group)
        with torch.cuda.device(self._dev):
            for p in self._opened:
                call("skcq_ep_close", p)
        self._opened = []
        dist.barrier(group=self.group)
        self._bytes = None
        with torch.cuda.device(self._dev):
            call("skcq_ep_free", self._base)
        self._base = None

    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                top_k_weights: torch.Tensor) -> torch.Tensor:
        if self._base is None:
            raise RuntimeError("ExpertParallelExperts used after close()")
        dev = self._dev
        h = _as_rows(hidden_states.to(dev))
        T, H = h.shape
        k = top_k_index.shape[1]
        if H != self.hidden:
            raise ValueError(f"hidden size {H}, the modules have {self.hidden}")
        if T > self.capacity or k > self.top_k_cap:
            raise ValueError(f"{T} tokens x top-{k} exceed the exchange buffers ({self.capacity} x {self.top_k_cap})")
        topk = top_k_index.to(device=dev, dtype=torch.int64).contiguous()
        w = top_k_weights.to(dev)
        if w.dtype not in (torch.float32, torch.bfloat16):
            w = w.float()
        w = w.contiguous()
        W, Cap, E = self.world, self.capacity, self.num_experts
        n_chunks = max(1, -(-T // 1024))
        scratch = torch.empty(8 * n_chunks + T * W, dtype=torch.int32, device=dev)
        pos = scratch[8 * n_chunks:]
        live = T > 0
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)] if self.record_phases else None
        if ev:
            ev[0].record()
        # 1. rows and slots to their experts' ranks
        call("skcq_ep_dispatch", ptr(h) if live else None, _DTYPE[h.dtype], h.stride(0) if live else H,
             ptr(topk) if live else None, ptr(w) if live else None, _DTYPE[w.dtype], T, k, E, self._bounds_arr,
             self._peers, W, self.rank, Cap, self.top_k_cap, H, ptr(scratch), ptr(pos) if live else None, stream())
        self._barrier()
        if ev:
            ev[1].record()
        # 2. this rank's experts on the rows it received
        Tl = W * Cap
        topk_l = torch.empty(Tl, k, dtype=torch.int64, device=dev)
        w_l = torch.empty(Tl, k, dtype=torch.float32, device=dev)
        call("skcq_ep_unpack", self._base, W, Cap, k, self.top_k_cap, H, ptr(topk_l), ptr(w_l), stream())
        d, n_split, inv = self.local.pair_outputs(self._rows(h.dtype), topk_l, skip_negative=True,
                                                  pairs_hint=max(T, 1) * k)
        if ev:
            ev[2].record()
        # 3. per received row, the weighted sum over local slots, into its source
        call("skcq_ep_return", ptr(d), _DTYPE[d.dtype], n_split, Tl * k, ptr(inv), ptr(topk_l), ptr(w_l), self._base,
             self._peers, self._bounds_arr, E, W, self.rank, Cap, k, self.top_k_cap, H, _DTYPE[h.dtype], stream())
        self._barrier()
        if ev:
            ev[3].record()
        # 4. each token's returned sums, ascending rank order
        out = torch.empty(T, H, dtype=h.dtype, device=dev)
        call("skcq_ep_gather", self._base, ptr(pos) if live else None, T, W, Cap, self.top_k_cap, H, _DTYPE[h.dtype],
             ptr(out) if live else None, _DTYPE[out.dtype], stream())
        if ev:
            ev[4].record()
            self.last_phases = ev
        if self.check_errors:
            _lib.poll_device_error()
        return out.to(device=hidden_states.device, dtype=hidden_states.dtype)
