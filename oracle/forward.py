"""Numpy restatement of the codebook-expert forward (skcq/codebook_experts.py).

Test infrastructure only (see ``oracle/__init__.py``). A layer is a dict with
the buffers of ``_CodebookLayer`` (codebook_experts.py:77-150):
``codebook (n_blocks, bs, K)``, ``assignments (E, n_blocks, out)``,
``scales (E, n_blocks, out)`` or None (float, already dequantised),
``remainder (E, out, rem)``, ``signs (E, out, cov)`` or None,
``block_size``, ``forward_mode``.
"""

from __future__ import annotations

import numpy as np

from oracle.codecs import Codec
from oracle.kmeans import F32


def choose_forward_mode(k: int, out_dim: int) -> str:
    """codebook_experts.py:26-27."""
    return "gather_matmul" if k > out_dim else "matmul_gather"


def codebook_pass(layer: dict, hidden: np.ndarray, e: int) -> np.ndarray:
    """codebook_experts.py:30-61 ``_codebook_pass`` -> (n_blocks, T, out)."""
    cb = layer["codebook"].astype(F32)
    assign = layer["assignments"][e]  # (n_blocks, out)
    n_blocks = assign.shape[0]
    bs = layer["block_size"]
    cov = n_blocks * bs
    hb = hidden[:, :cov].astype(F32).reshape(-1, n_blocks, bs).transpose(1, 0, 2)
    signs = layer.get("signs")
    mode = "gather_matmul" if signs is not None else layer["forward_mode"]
    if cb.shape[0] != n_blocks:
        raise RuntimeError("gather: index size exceeds input size (shared codebook, codebook_experts.py:49)")
    if mode == "gather_matmul":
        g = np.take_along_axis(cb, assign[:, None, :].repeat(bs, axis=1), axis=2)
        if signs is not None:
            out_dim = assign.shape[1]
            s = signs[e]
            if s.shape[1] != cov:
                raise RuntimeError("signs reshape: in_dim not divisible by block_size (codebook_experts.py:54)")
            g = g * s.reshape(out_dim, n_blocks, bs).transpose(1, 2, 0).astype(F32)
        return np.matmul(hb, g)
    logits = np.matmul(hb, cb)  # (n_blocks, T, K)
    t = hidden.shape[0]
    return np.take_along_axis(logits, np.broadcast_to(assign[:, None, :], (n_blocks, t, assign.shape[1])), axis=2)


def remainder_pass(layer: dict, hidden: np.ndarray, e: int) -> np.ndarray:
    """codebook_experts.py:64-74."""
    n_blocks = layer["assignments"].shape[1]
    cov = n_blocks * layer["block_size"]
    rem_w = layer["remainder"][e].astype(F32)  # (out, rem)
    x_rem = hidden[:, cov : cov + rem_w.shape[1]].astype(F32)
    return x_rem @ rem_w.T


def module_forward(layers: list[dict], hidden: np.ndarray, e: int) -> np.ndarray:
    """codebook_experts.py:325-339 ``CodebookModule.forward``."""
    p = layers[0]
    prim = codebook_pass(p, hidden, e)
    if p.get("scales") is not None:
        out = (prim * p["scales"][e][:, None, :].astype(F32)).sum(axis=0, dtype=F32)
    else:
        out = prim.sum(axis=0, dtype=F32)
    out = out + remainder_pass(p, hidden, e)
    for layer in layers[1:]:
        out = out + codebook_pass(layer, hidden, e).sum(axis=0, dtype=F32)
        out = out + remainder_pass(layer, hidden, e)
    return out.astype(F32)


def layers_from_fit(codecs: list[Codec], cwrs: list[dict], out_dim: int) -> list[dict]:
    """codebook_experts.py:183-234 ``from_cwr`` + :359-419 ``_extract_and_reshape``."""
    layers = []
    for codec, cwr in zip(codecs, cwrs, strict=True):
        signs = None
        inner_codec, inner = codec, cwr
        if codec.kind == "ssvq":
            inner_codec, inner, signs = codec.inner, cwr["inner"], cwr["signs"]
        idxs = inner["idxs"]
        n_blocks, n_rows = idxs.shape
        e = n_rows // out_dim
        scales = None
        if inner.get("scales") is not None:
            s = inner["scales"]
            if inner_codec.scale_dtype.startswith("int"):
                s = s.astype(F32) * F32(inner_codec.q_scale)
            scales = s.astype(F32).reshape(e, out_dim, n_blocks).transpose(0, 2, 1).copy()
        rem = inner["remainder"]
        k = inner_codec.centroids.shape[-1]
        layers.append(
            {
                "codebook": inner_codec.centroids.astype(F32),
                "assignments": idxs.reshape(n_blocks, e, out_dim).transpose(1, 0, 2).copy(),
                "scales": scales,
                "remainder": (rem.reshape(e, out_dim, rem.shape[1]) if rem is not None else np.zeros((e, out_dim, 0), F32)),
                "signs": signs.reshape(e, out_dim, signs.shape[1]) if signs is not None else None,
                "block_size": inner_codec.cfg.block_size,
                "forward_mode": choose_forward_mode(k, out_dim),
            }
        )
    return layers


def silu(x: np.ndarray) -> np.ndarray:
    return (x / (F32(1.0) + np.exp(-x.astype(F32)))).astype(F32)


def experts_forward(gate, up, down, num_experts, hidden, top_k_index, top_k_weights) -> np.ndarray:
    """codebook_experts.py:454-481 ``CodebookExperts.forward`` with SiLU SwiGLU."""
    final = np.zeros_like(hidden, dtype=F32)
    for e in range(num_experts):
        pos, tok = np.nonzero((top_k_index == e).T)  # (top_k, T) row-major order
        if tok.size == 0:
            continue
        x = hidden[tok].astype(F32)
        inter = silu(module_forward(gate, x, e)) * module_forward(up, x, e)
        y = module_forward(down, inter, e) * top_k_weights[tok, pos][:, None].astype(F32)
        np.add.at(final, tok, y)
    return final
