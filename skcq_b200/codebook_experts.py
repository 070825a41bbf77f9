"""Codebook-quantized MoE experts on B200 (interface of skcq/codebook_experts.py).

``CodebookModule`` keeps the reference's parameters, buffers, state-dict keys and
meta (so saved modules load in either implementation); its forward runs the
grouped gather-dequant kernel of ``csrc/forward.cu`` over all codebook layers
at once. ``CodebookExperts.forward`` routes (token, slot) pairs to experts on
the device (no per-expert host synchronisation), runs gate, up, SwiGLU and down
for every expert in four launches, and combines the weighted outputs in the
reference's expert order.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any, Literal

import torch
import torch.nn as nn
import torch.nn.functional as F  # noqa: N812

from skcq_b200 import _lib
from skcq_b200._lib import call, ptr, stream

ForwardMode = Literal["matmul_gather", "gather_matmul"]

_DTYPE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2, torch.int8: 3, torch.int16: 4}


def _choose_forward_mode(k: int, out_dim: int) -> ForwardMode:
    """codebook_experts.py:26-27 (kept for API parity; both modes compute the
    same values and the kernel does not need to choose)."""
    return "gather_matmul" if k > out_dim else "matmul_gather"


class _CodebookLayer(nn.Module):
    """One codebook's buffers (codebook_experts.py:77-130): ``codebook``
    (n_blocks | 1, bs, K), ``assignments`` (E, n_blocks, out) int64, optional
    ``scales`` (E, n_blocks, out), ``remainder`` (E, out, rem), optional
    ``signs`` (E, out, cov) int8."""

    codebook: nn.Parameter
    assignments: torch.Tensor
    scales: nn.Parameter | None
    remainder: torch.Tensor
    signs: torch.Tensor | None

    def __init__(
        self,
        codebook: torch.Tensor,
        assignments: torch.Tensor,
        n_blocks: int,
        block_size: int,
        out_dim: int,
        k: int,
        remainder: torch.Tensor | None = None,
        signs: torch.Tensor | None = None,
        scales: torch.Tensor | None = None,
        scale_q_scale: torch.Tensor | None = None,
    ) -> None:
        super().__init__()
        self.n_blocks = n_blocks
        self.block_size = block_size
        self.out_dim = out_dim
        self.k = k
        self.has_scale = scales is not None
        num_experts = assignments.shape[0]
        self.codebook = nn.Parameter(codebook)
        self.register_buffer("assignments", assignments)
        if scales is not None:
            if scales.is_floating_point():
                self.scales = nn.Parameter(scales)
            else:
                self.register_buffer("scales", scales)
        else:
            self.scales = None
        if scale_q_scale is not None:
            self.register_buffer("scale_q_scale", scale_q_scale)
        if remainder is None:
            remainder = torch.zeros(num_experts, out_dim, 0, dtype=codebook.dtype, device=codebook.device)
        self.rem = remainder.shape[-1]
        self.register_buffer("remainder", remainder)
        self.sign_cov = signs.shape[-1] if signs is not None else 0
        self.register_buffer("signs", signs)
        self.forward_mode: ForwardMode = _choose_forward_mode(k, out_dim)
        self._packed: tuple | None = None

    # -- device layout -------------------------------------------------------

    @staticmethod
    def _key(t: torch.Tensor | None) -> tuple | None:
        if t is None:
            return None
        return (t.data_ptr(), t._version, t.dtype, tuple(t.shape), str(t.device))

    def _layout(self, dev: torch.device) -> dict[str, Any]:
        """Device tensors of the forward layout (csrc/forward.cu): transposed
        centroid table, uint16 indices, sign bitmasks, scales and remainder on
        ``dev``. Rebuilt when any source tensor changes (in place or by
        ``.to()``); index and sign validation happens here, once."""
        key = (str(dev), *(self._key(t) for t in (self.codebook, self.assignments, self.scales, self.remainder,
                                                  self.signs)))
        cache = self._packed
        if cache is not None and cache[0] == key:
            return cache[1]
        nb, bs = self.n_blocks, self.block_size
        if self.codebook.shape[0] != nb:
            raise RuntimeError(
                "gather(): index size must not exceed the input size (a shared codebook cannot drive the "
                "per-expert forward, codebook_experts.py:49)"
            )
        if self.signs is not None and self.signs.shape[-1] != nb * bs:
            raise RuntimeError(
                f"shape '[{self.out_dim}, {nb}, {bs}]' is invalid for signs covering {self.signs.shape[-1]} columns "
                "(codebook_experts.py:54)"
            )
        if bs > 32:
            raise RuntimeError(f"block size {bs} exceeds the forward kernel's 32")
        cb = self.codebook.detach().to(dev)
        if cb.dtype not in (torch.float32, torch.bfloat16):
            cb = cb.float()
        cb = cb.contiguous()
        K = cb.shape[-1]
        if K > 65536:
            raise RuntimeError(f"codebook size {K} exceeds the 16-bit index format")
        table = torch.empty(nb, K, bs, dtype=cb.dtype, device=dev)
        call("skcq_transpose_codebook", ptr(cb), _DTYPE[cb.dtype], nb, bs, K, ptr(table), stream())
        a = self.assignments.to(device=dev, dtype=torch.int64).contiguous()
        idx16 = torch.empty(a.shape, dtype=torch.int16, device=dev)
        call("skcq_pack_indices16", ptr(a), a.numel(), K, ptr(idx16), stream())
        mask = None
        if self.signs is not None:
            sg = self.signs.to(device=dev, dtype=torch.int8).contiguous()
            E, out, ld = sg.shape
            mask = torch.empty(E, nb, out, dtype=torch.int32, device=dev)
            call("skcq_pack_sign_masks", ptr(sg), E, out, ld, nb, bs, ptr(mask), stream())
        scales = None
        if self.has_scale and self.scales is not None:
            scales = self.scales.detach().to(dev)
            if scales.dtype not in _DTYPE:
                scales = scales.float()
            scales = scales.contiguous()
        rem = None
        if self.rem > 0:
            rem = self.remainder.detach().to(dev)
            if rem.dtype not in (torch.float32, torch.bfloat16):
                rem = rem.float()
            rem = rem.contiguous()
        _lib.poll_device_error()  # an index outside [0, K) or a sign other than +-1 raises here
        lay = {"table": table, "idx16": idx16, "mask": mask, "scales": scales, "rem": rem, "K": K}
        self._packed = (key, lay)
        return lay

    def descriptor(self, dev: torch.device, primary: bool) -> FwdLayer:
        """``skcq_fwd_layer`` over this layer's device layout. Only the primary
        layer's scales enter the forward (codebook_experts.py:327-331)."""
        lay = self._layout(dev)
        d = FwdLayer()
        d.n_blocks, d.bs, d.K = self.n_blocks, self.block_size, lay["K"]
        d.table, d.table_dtype = ptr(lay["table"]), _DTYPE[lay["table"].dtype]
        d.idx16 = ptr(lay["idx16"])
        s = lay["scales"]
        if primary and s is not None:
            d.scales, d.scale_dtype = ptr(s), _DTYPE[s.dtype]
            d.q_scale = float(self.scale_q_scale) if not s.is_floating_point() else 1.0
        if lay["rem"] is not None:
            d.remainder, d.rem_dtype, d.rem = ptr(lay["rem"]), _DTYPE[lay["rem"].dtype], self.rem
        if lay["mask"] is not None:
            d.sign_mask = ptr(lay["mask"])
        return d


class FwdLayer(_lib.C.Structure):
    """``skcq_fwd_layer`` (include/skcq_b200.h)."""

    _fields_ = [
        ("n_blocks", _lib.I), ("bs", _lib.I), ("K", _lib.I),
        ("table", _lib.P), ("table_dtype", _lib.I),
        ("idx16", _lib.P),
        ("scales", _lib.P), ("scale_dtype", _lib.I), ("q_scale", _lib.F),
        ("remainder", _lib.P), ("rem_dtype", _lib.I), ("rem", _lib.I),
        ("sign_mask", _lib.P),
        ("lut", _lib.P), ("lut_tokens", _lib.I),
    ]


def _cuda_of(*tensors: torch.Tensor) -> torch.device:
    for t in tensors:
        if t is not None and t.is_cuda:
            return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("skcq_b200 needs a CUDA device (B200, sm_100a); none is available")
    return torch.device("cuda", torch.cuda.current_device())


def _as_rows(x: torch.Tensor) -> torch.Tensor:
    """f32 or bf16 rows with unit column stride (the dtypes the kernels read)."""
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    if x.dim() != 2 or x.stride(-1) != 1:
        x = x.reshape(-1, x.shape[-1]).contiguous()
    return x


# CTAs the split-K decode aims for (8 per SM on 148 SMs)
_TARGET_CTAS = 8 * 148
_MAX_SPLITS = 64


def _choose_splits(max_active: int, out_dim: int, min_blocks: int, rows: int) -> int:
    """Block-range splits so that small batches still fill the GPU; one split
    once there are enough (segment, output tile) items or many rows."""
    tiles = -(-out_dim // 128)
    items = max(1, max_active * tiles)
    s = -(-_TARGET_CTAS // items)
    s = min(s, _MAX_SPLITS, max(1, min_blocks))
    # the [splits][rows][out] f32 partial buffer stays below 256 MiB
    s = min(s, max(1, (256 << 20) // max(1, rows * out_dim * 4)))
    return max(1, s)


class CodebookModule(nn.Module):
    """Composite codebook layers of one projection (codebook_experts.py:153-339)."""

    def __init__(self, layers: nn.ModuleList, n_codebooks: int, out_dim: int) -> None:
        super().__init__()
        self.layers = layers
        self.n_codebooks = n_codebooks
        self.out_dim = out_dim
        self.n_blocks = layers[0].n_blocks
        self.block_size = layers[0].block_size

    @property
    def primary(self) -> _CodebookLayer:
        return self.layers[0]

    @property
    def additives(self) -> list[_CodebookLayer]:
        return list(self.layers[1:])

    @classmethod
    def from_cwr(cls, aqlm, cwr, out_dim: int) -> CodebookModule:
        """codebook_experts.py:183-234."""
        n_rows = _cwr_n_rows(cwr)
        num_experts = n_rows // out_dim
        pairs = [(aqlm.primary, cwr.primary), *zip(aqlm.residuals, cwr.residuals, strict=True)]
        layer_list: list[_CodebookLayer] = []
        for cb, layer_cwr in pairs:
            centroids, a3, s3, r3, g3 = _extract_and_reshape(cb, layer_cwr, num_experts, out_dim)
            n_blocks = a3.shape[1]
            block_size = getattr(cb, "block_size", centroids.shape[1])
            k = centroids.shape[-1]
            q = None
            if s3 is not None and not s3.is_floating_point():
                inner = cb.inner if hasattr(cb, "inner") else cb
                sq = getattr(inner, "scale_quant", None)
                if sq is not None and sq.q_scale is not None:
                    q = sq.q_scale
            layer_list.append(_CodebookLayer(centroids, a3, n_blocks, block_size, out_dim, k, remainder=r3,
                                             signs=g3, scales=s3, scale_q_scale=q))
        return cls(nn.ModuleList(layer_list), len(pairs), out_dim)

    @classmethod
    def empty(cls, n_blocks: int, block_size: int, out_dim: int, k_list: list[int], num_experts: int,
              n_blocks_list: list[int] | None = None, block_size_list: list[int] | None = None,
              rem_list: list[int] | None = None, sign_cov_list: list[int] | None = None,
              has_scale_list: list[bool] | None = None) -> CodebookModule:
        """Zero-filled module sized for ``load_state_dict`` (codebook_experts.py:236-282)."""
        n_cb = len(k_list)
        nbl = n_blocks_list or [n_blocks] * n_cb
        bsl = block_size_list or [block_size] * n_cb
        reml = rem_list or [0] * n_cb
        scl = sign_cov_list or [0] * n_cb
        hsl = has_scale_list or [True] + [False] * (n_cb - 1)
        layers = []
        for c in range(n_cb):
            layers.append(_CodebookLayer(
                torch.zeros(nbl[c], bsl[c], k_list[c], dtype=torch.bfloat16),
                torch.zeros(num_experts, nbl[c], out_dim, dtype=torch.long),
                nbl[c], bsl[c], out_dim, k_list[c],
                remainder=torch.zeros(num_experts, out_dim, reml[c], dtype=torch.bfloat16),
                signs=torch.zeros(num_experts, out_dim, scl[c], dtype=torch.int8) if scl[c] > 0 else None,
                scales=torch.zeros(num_experts, nbl[c], out_dim, dtype=torch.bfloat16) if hsl[c] else None,
            ))
        return cls(nn.ModuleList(layers), n_cb, out_dim)

    @classmethod
    def load(cls, path: Any) -> CodebookModule:
        """codebook_experts.py:284-301."""
        data = torch.load(path, weights_only=True)
        meta = data["meta"]
        module = cls.empty(
            n_blocks=meta["n_blocks"], block_size=meta["block_size"], out_dim=meta["out_dim"],
            k_list=meta["k_list"], num_experts=meta["num_experts"], n_blocks_list=meta.get("n_blocks_list"),
            block_size_list=meta.get("block_size_list"), rem_list=meta.get("rem_list"),
            sign_cov_list=meta.get("sign_cov_list"), has_scale_list=meta.get("has_scale_list"),
        )
        module.load_state_dict(data["state_dict"])
        return module

    def slice_experts(self, e0: int, e1: int) -> CodebookModule:
        """A module for experts [e0, e1) only: per-expert buffers (assignments,
        scales, remainder, signs) sliced, per-block codebooks shared. Used for
        expert-parallel placement."""
        layers = []
        for lay in self.layers:
            q = getattr(lay, "scale_q_scale", None)
            layers.append(_CodebookLayer(
                lay.codebook.detach(), lay.assignments[e0:e1], lay.n_blocks, lay.block_size, lay.out_dim, lay.k,
                remainder=lay.remainder[e0:e1],
                signs=lay.signs[e0:e1] if lay.signs is not None else None,
                scales=lay.scales.detach()[e0:e1] if lay.has_scale and lay.scales is not None else None,
                scale_q_scale=q,
            ))
        return CodebookModule(nn.ModuleList(layers), self.n_codebooks, self.out_dim)

    def _all_layers(self) -> list[_CodebookLayer]:
        return list(self.layers)

    def state_dict_with_meta(self) -> dict[str, Any]:
        """codebook_experts.py:306-323 (same keys and meta)."""
        cbs = self._all_layers()
        return {
            "state_dict": self.state_dict(),
            "meta": {
                "n_blocks": self.n_blocks, "block_size": self.block_size, "out_dim": self.out_dim,
                "n_codebooks": self.n_codebooks, "k_list": [cb.k for cb in cbs],
                "n_blocks_list": [cb.n_blocks for cb in cbs], "block_size_list": [cb.block_size for cb in cbs],
                "rem_list": [cb.rem for cb in cbs], "sign_cov_list": [cb.sign_cov for cb in cbs],
                "has_scale_list": [cb.has_scale for cb in cbs], "num_experts": self.primary.assignments.shape[0],
            },
        }

    @property
    def min_blocks(self) -> int:
        return min(layer.n_blocks for layer in self.layers)

    def run_segments(self, x: torch.Tensor, seg: torch.Tensor, seg_expert: torch.Tensor | None,
                     n_seg: int, *, row_token: torch.Tensor | None = None, T: int = 0,
                     active: torch.Tensor | None = None, max_active: int | None = None,
                     n_rows: int | None = None, n_split: int | None = None,
                     rows_hint: int | None = None,
                     lut_layers: list[bool] | None = None) -> tuple[torch.Tensor, int]:
        """Grouped forward over expert segments of rows (device tensors).

        Row r of segment s (expert ``seg_expert[s]``, or s) reads
        ``x[row_token[r] % T]`` (``x[r]`` without a token map). Layers flagged
        in ``lut_layers`` (and without signs) read their block dots from a
        per-row lookup table built here (codebook_experts.py:57-60); the
        result is the same. Returns the ``(n_split, n_rows, out_dim)`` f32
        partial sums and ``n_split``; their sum over the first axis is the
        module output."""
        x = _as_rows(x)
        dev = x.device
        P = int(n_rows if n_rows is not None else (row_token.numel() if row_token is not None else x.shape[0]))
        max_active = n_seg if max_active is None else max_active
        S = n_split or _choose_splits(max_active, self.out_dim, self.min_blocks, P)
        descs = [layer.descriptor(dev, primary=(i == 0)) for i, layer in enumerate(self.layers)]
        luts = []
        if lut_layers is not None:
            # the reference's matmul_gather mode for these layers: per-row tables
            # of block dots over x's rows, read by the forward instead of
            # gathering centroids (identical results)
            n_tok = T if row_token is not None else x.shape[0]
            for d, use in zip(descs, lut_layers, strict=False):
                if not use or d.sign_mask:
                    continue
                lut = torch.empty(d.n_blocks * d.K * n_tok, dtype=torch.float32, device=dev)
                call("skcq_lut_build", _lib.C.addressof(d), ptr(x), _DTYPE[x.dtype], x.stride(0), n_tok, ptr(lut),
                     stream())
                d.lut, d.lut_tokens = ptr(lut), n_tok
                luts.append(lut)
        arr = (FwdLayer * len(descs))(*descs)
        part = torch.empty(S, P, self.out_dim, dtype=torch.float32, device=dev)
        hint = rows_hint if rows_hint is not None else -(-P // max(1, max_active))
        call("skcq_codebook_forward", _lib.C.cast(arr, _lib.C.c_void_p), len(descs), ptr(x), _DTYPE[x.dtype],
             x.stride(0), ptr(row_token), T, ptr(seg), ptr(seg_expert), ptr(active), n_seg, max_active,
             x.shape[1], self.out_dim, S, hint, ptr(part), P, stream())
        return part, S

    def dequant_into(self, W: torch.Tensor, active: torch.Tensor | None, max_slots: int, in_dim: int,
                     half: int = -1) -> None:
        """Decode the active experts' dense weights into ``W`` (the tcgen05
        operand image of skcq_prefill_dequant)."""
        dev = W.device
        descs = [layer.descriptor(dev, primary=(i == 0)) for i, layer in enumerate(self.layers)]
        arr = (FwdLayer * len(descs))(*descs)
        call("skcq_prefill_dequant", _lib.C.cast(arr, _lib.C.c_void_p), len(descs), ptr(active), max_slots,
             self.out_dim, in_dim, half, ptr(W), stream())

    def prefill(self, A: torch.Tensor, tiles: torch.Tensor, max_tiles: int, active: torch.Tensor | None,
                max_slots: int, n_rows: int, in_dim: int, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """Tensor-core forward of packed rows ``A`` (skcq_prefill_pack layout):
        decode the active experts' weights once, then one grouped GEMM
        (fp32 accumulation). Returns (n_rows, out_dim) in ``out_dtype``
        (f32 or bf16)."""
        dev = A.device
        KC, NT = -(-in_dim // 64), -(-self.out_dim // 256)
        W = torch.empty(max_slots * NT * KC * 16384, dtype=torch.bfloat16, device=dev)
        self.dequant_into(W, active, max_slots, in_dim)
        y = torch.empty(n_rows, self.out_dim, dtype=out_dtype, device=dev)
        call("skcq_prefill_gemm", ptr(A), ptr(W), ptr(tiles), max_tiles, in_dim, self.out_dim, ptr(y),
             _DTYPE[out_dtype], y.stride(0), stream())
        return y

    def forward(self, hidden_states: torch.Tensor, expert_idx: int) -> torch.Tensor:
        """codebook_experts.py:325-339 for one expert; output in the input dtype
        on the input's device."""
        E = self.primary.assignments.shape[0]
        e = int(expert_idx)
        if not -E <= e < E:
            raise IndexError(f"index {e} is out of bounds for dimension 0 with size {E}")
        e %= E
        dev = _cuda_of(hidden_states, self.primary.codebook)
        h = _as_rows(hidden_states.to(dev))
        T = h.shape[0]
        meta = torch.tensor([0, T, e], dtype=torch.int32).to(dev, non_blocking=True)
        part, S = self.run_segments(h, meta[:2], meta[2:], 1)
        y = torch.empty(T, self.out_dim, dtype=h.dtype, device=dev)
        call("skcq_sum_splits", ptr(part), S, T, self.out_dim, ptr(y), _DTYPE[y.dtype], y.stride(0), stream())
        return y.to(device=hidden_states.device, dtype=hidden_states.dtype)


def _cwr_n_rows(cwr) -> int:
    """codebook_experts.py:347-356 (duck-typed over AQLM / SSVQ / leaf payloads)."""
    if hasattr(cwr, "primary"):
        return _cwr_n_rows(cwr.primary)
    inner = cwr.inner if hasattr(cwr, "inner") else cwr
    if hasattr(inner, "idxs"):
        return inner.idxs.shape[1]
    raise TypeError(f"Unknown CWR type: {type(inner)}")


def _extract_and_reshape(cb, cwr, num_experts: int, out_dim: int):
    """codebook_experts.py:359-419: per-expert views of one codebook's payload."""
    if hasattr(cwr, "inner") and hasattr(cwr, "signs"):
        inner_cwr, signs_flat = cwr.inner, cwr.signs
    else:
        inner_cwr, signs_flat = cwr, None
    centroids = cb.centroids_tensor
    idxs = inner_cwr.idxs
    scales_flat = getattr(inner_cwr, "scales", None)
    remainder_flat = inner_cwr.remainder
    n_blocks = idxs.shape[0]
    a3 = idxs.reshape(n_blocks, num_experts, out_dim).permute(1, 0, 2).contiguous()
    s3 = (scales_flat.reshape(num_experts, out_dim, n_blocks).permute(0, 2, 1).contiguous()
          if scales_flat is not None else None)
    r3 = (remainder_flat.reshape(num_experts, out_dim, remainder_flat.shape[1]).contiguous()
          if remainder_flat is not None else None)
    g3 = (signs_flat.reshape(num_experts, out_dim, signs_flat.shape[1]).to(torch.int8).contiguous()
          if signs_flat is not None else None)
    return centroids, a3, s3, r3, g3


class _SwiGLU(nn.Module):
    def __init__(self, act_fn: Callable[[torch.Tensor], torch.Tensor]) -> None:
        super().__init__()
        self.act_fn = act_fn

    def forward(self, gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
        return self.act_fn(gate) * up


def _is_silu(fn) -> bool:
    return fn is F.silu or isinstance(fn, nn.SiLU)


class CodebookExperts(nn.Module):
    """Drop-in replacement for a Qwen-style MoE experts block
    (codebook_experts.py:436-482).

    Routing, gate/up, SwiGLU, down and the weighted combine run on the device
    without host synchronisation; ``check_errors`` (default on) reads the
    device error word once at the end so that an expert id outside
    ``[0, num_experts)`` raises like the reference's ``one_hot``."""

    check_errors: bool = True
    # bf16 batches with at least this many (token, slot) rows per expert on
    # average take the tensor-core prefill path
    prefill_min_rows: int = 32
    # Decode lookup tables (the reference's matmul_gather mode): "off" (the
    # default: on B200 the gather path measured faster at every batch of 1 to
    # 64 tokens but 2 on the benchmark layer); "on" for every sign-free layer
    # of the three projections whose table stays below lut_max_bytes; "auto"
    # for those whose table build (one block dot per token and centroid) also
    # does less work than the gathers it replaces (one per routed row and
    # output). All three give the same bits.
    decode_lut: str = "off"
    lut_max_bytes: int = 64 << 20

    def __init__(self, gate: CodebookModule, up: CodebookModule, down: CodebookModule, num_experts: int,
                 act_fn: Callable[[torch.Tensor], torch.Tensor]) -> None:
        super().__init__()
        self.num_experts = num_experts
        self.gate = gate
        self.up = up
        self.intermediate = _SwiGLU(act_fn)
        self.down = down

    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                top_k_weights: torch.Tensor) -> torch.Tensor:
        dev = _cuda_of(hidden_states, self.gate.primary.codebook)
        h = _as_rows(hidden_states.to(dev))
        T, H = h.shape
        k = top_k_index.shape[1]
        topk = top_k_index.to(device=dev, dtype=torch.int64).contiguous()
        w = top_k_weights.to(dev)
        if w.dtype not in (torch.float32, torch.bfloat16):
            w = w.float()
        w = w.contiguous()
        d, Sd, inv = self.pair_outputs(h, topk)
        out = torch.empty(T, H, dtype=h.dtype, device=dev)
        call("skcq_combine", ptr(d), _DTYPE[d.dtype], Sd, T * k, ptr(inv), ptr(topk), ptr(w), _DTYPE[w.dtype], T, k,
             H, ptr(out), _DTYPE[out.dtype], stream())
        if self.check_errors:
            _lib.poll_device_error()
        return out.to(device=hidden_states.device, dtype=hidden_states.dtype)

    def pair_outputs(self, h: torch.Tensor, topk: torch.Tensor, skip_negative: bool = False,
                     pairs_hint: int | None = None) -> tuple[torch.Tensor, int, torch.Tensor]:
        """Expert outputs of every routed (token, slot) pair of ``h`` (T, H) and
        ``topk`` (T, k) int64 on the modules' device: returns ``(d, n_split,
        row_of_pair)`` with pair p = kpos * T + token's output the sum over
        splits of ``d[s][row_of_pair[p]]`` (``d`` is (n_split, P, H) f32 on the
        gather path, (P, H) bf16 with n_split 1 on the tensor-core path).
        ``skip_negative``: slots with a negative id are not routed here.
        ``pairs_hint``: the expected number of routed pairs (defaults to T * k),
        which picks the path."""
        dev = h.device
        T = h.shape[0]
        k = topk.shape[1]
        E = self.num_experts
        P = T * k
        route = torch.empty(2 * max(P, 1) + 2 * (E + 1), dtype=torch.int32, device=dev)
        perm = route[:max(P, 1)]
        inv = route[max(P, 1):2 * max(P, 1)]
        seg = route[2 * max(P, 1):2 * max(P, 1) + E + 1]
        active = route[2 * max(P, 1) + E + 1:]
        scratch_bytes = int(_lib.load().skcq_route_sort_scratch_bytes(T, k, E))
        scratch = torch.empty(scratch_bytes, dtype=torch.uint8, device=dev) if scratch_bytes else None
        call("skcq_route_sort", ptr(topk), T, k, E, ptr(perm), ptr(seg), ptr(inv), ptr(active), ptr(scratch),
             scratch_bytes, int(skip_negative), stream())
        max_active = min(E, P)
        I = self.gate.out_dim
        if self._use_prefill(h, P if pairs_hint is None else pairs_hint, max_active):
            return self._prefill_pairs(h, perm, seg, active, T, P, max_active), 1, inv
        S = _choose_splits(max_active, I, min(self.gate.min_blocks, self.up.min_blocks), P)
        # rows per expert: at most T when a token's k experts are distinct
        seg_kw = {"active": active, "max_active": max_active, "n_rows": P, "rows_hint": min(T, 8)}
        g, _ = self.gate.run_segments(h, seg, None, E, row_token=perm, T=T, n_split=S,
                                      lut_layers=self._lut_layers(self.gate, T, P), **seg_kw)
        u, _ = self.up.run_segments(h, seg, None, E, row_token=perm, T=T, n_split=S,
                                    lut_layers=self._lut_layers(self.up, T, P), **seg_kw)
        inter = torch.empty(P, I, dtype=torch.float32, device=dev)
        if _is_silu(self.intermediate.act_fn):
            call("skcq_swiglu", ptr(g), ptr(u), S, P * I, ptr(inter), stream())
        else:
            gs, us = g.sum(0), u.sum(0)
            inter.copy_(self.intermediate(gs, us))
        d, Sd = self.down.run_segments(inter, seg, None, E, lut_layers=self._lut_layers(self.down, P, P), **seg_kw)
        return d, Sd, inv

    def _lut_layers(self, mod: CodebookModule, n_tok: int, P: int) -> list[bool] | None:
        """Which layers of ``mod`` read a lookup table: x has ``n_tok`` rows and
        ``P`` routed rows are computed."""
        if self.decode_lut == "off":
            return None
        use = []
        for lay in mod.layers:
            table = lay.n_blocks * lay.k * n_tok * 4
            ok = lay.signs is None and table <= self.lut_max_bytes and lay.block_size in (4, 6, 8, 12, 16)
            if self.decode_lut == "auto":
                ok = ok and n_tok * lay.k < P * mod.out_dim
            use.append(ok)
        return use if any(use) else None

    def _use_prefill(self, h: torch.Tensor, P: int, max_active: int) -> bool:
        mods = (self.gate, self.up, self.down)
        return (h.dtype == torch.bfloat16 and P >= self.prefill_min_rows * max(1, max_active)
                and all(la.codebook.dtype == torch.bfloat16 for m in mods for la in m.layers))

    def _prefill_pairs(self, h, perm, seg, active, T, P, max_active) -> torch.Tensor:
        """Tensor-core path: plan 128-row tiles per expert, pack the routed
        rows once for gate and up, decode each projection's active experts and
        run the grouped tcgen05 GEMM; SwiGLU is fused into packing the down
        projection's rows. Returns the (P, H) bf16 pair outputs."""
        dev = h.device
        H = h.shape[1]
        I = self.gate.out_dim
        max_tiles = -(-P // 128) + max_active
        tiles = torch.empty(1 + 3 * max_tiles, dtype=torch.int32, device=dev)
        call("skcq_prefill_plan", ptr(seg), self.num_experts, max_tiles, ptr(tiles), stream())
        A = torch.empty(max_tiles * (-(-H // 64)) * 8192, dtype=torch.bfloat16, device=dev)
        call("skcq_prefill_pack", 0, ptr(h), _DTYPE[h.dtype], h.stride(0), ptr(perm), T, None, 0, H, ptr(tiles),
             max_tiles, ptr(A), stream())
        A2 = torch.empty(max_tiles * (-(-I // 64)) * 8192, dtype=torch.bfloat16, device=dev)
        if _is_silu(self.intermediate.act_fn) and self.up.out_dim == I:
            # gate and up share one weight image; the GEMM epilogue applies SwiGLU
            # and writes the down projection's packed rows
            Wgu = torch.empty(max_active * (-(-I // 128)) * (-(-H // 64)) * 16384, dtype=torch.bfloat16, device=dev)
            self.gate.dequant_into(Wgu, active, max_active, H, half=0)
            self.up.dequant_into(Wgu, active, max_active, H, half=1)
            call("skcq_prefill_gemm_swiglu", ptr(A), ptr(Wgu), ptr(tiles), max_tiles, H, I, ptr(A2), stream())
            del Wgu
        else:
            g = self.gate.prefill(A, tiles, max_tiles, active, max_active, P, H)
            u = self.up.prefill(A, tiles, max_tiles, active, max_active, P, H)
            inter = self.intermediate(g, u).float().contiguous()
            del g, u
            call("skcq_prefill_pack", 0, ptr(inter), _DTYPE[torch.float32], inter.stride(0), None, 0, None, 0, I,
                 ptr(tiles), max_tiles, ptr(A2), stream())
        del A
        # bf16 down outputs, as the reference's bf16 module produces them
        return self.down.prefill(A2, tiles, max_tiles, active, max_active, P, I, out_dtype=torch.bfloat16)


class GraphedExperts:
    """CUDA-graph replay of ``CodebookExperts.forward`` for one batch shape.

    Decode steps are launch-bound (route, three layers per projection, SwiGLU,
    combine); capturing them once and replaying removes the per-launch host
    cost. Inputs are copied into static buffers, the graph is replayed and the
    static output tensor is returned (overwritten by the next call). Device-side
    checks (an expert id out of range) are recorded and can be read with
    ``skcq_b200._lib.poll_device_error()``.
    """

    def __init__(self, experts: CodebookExperts, n_tokens: int, top_k: int, dtype: torch.dtype = torch.bfloat16,
                 weights_dtype: torch.dtype = torch.float32, device: torch.device | None = None) -> None:
        dev = device or _cuda_of(experts.gate.primary.codebook)
        H = experts.down.out_dim
        self.experts = experts
        self.x = torch.zeros(n_tokens, H, dtype=dtype, device=dev)
        self.topi = torch.arange(top_k, device=dev).remainder(experts.num_experts).expand(n_tokens, top_k).contiguous()
        self.topw = torch.full((n_tokens, top_k), 1.0 / top_k, dtype=weights_dtype, device=dev)
        check = experts.check_errors
        experts.check_errors = False
        try:
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                for _ in range(2):  # builds device layouts and configures kernels outside the capture
                    experts(self.x, self.topi, self.topw)
            torch.cuda.current_stream(dev).wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, capture_error_mode="relaxed"):
                self.out = experts(self.x, self.topi, self.topw)
        finally:
            experts.check_errors = check

    def __call__(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                 top_k_weights: torch.Tensor) -> torch.Tensor:
        self.x.copy_(hidden_states, non_blocking=True)
        self.topi.copy_(top_k_index, non_blocking=True)
        self.topw.copy_(top_k_weights, non_blocking=True)
        self.graph.replay()
        return self.out
