"""Integer and fp8 baselines of the sweep (interface of skcq/vq/runner.py:86-188).

Affine (asymmetric) round-to-nearest quantisation of a weight matrix per
tensor, per channel (row) or per block of ``block_size`` consecutive columns,
each returning ``(reconstruction, bits per weight)`` with the reference's bit
accounting: ``bits`` per weight plus one fp16 minimum and one fp16 scale
(32 bits) per group, and the remainder columns of the per-block form kept as
bf16 (16 bits). The arithmetic is the reference's, element for element; the
per-block form is vectorised over blocks instead of a Python loop, so it runs
as a handful of device ops on the input's device.
"""

from __future__ import annotations

from collections.abc import Callable
from functools import partial

import torch


def _quant_affine(W: torch.Tensor, bits: int) -> torch.Tensor:  # noqa: N803
    """runner.py:101-111."""
    n_levels = 2**bits - 1
    w_min = W.min()
    w_max = W.max()
    scale = (w_max - w_min) / n_levels
    if scale == 0:
        return W.clone()
    q = torch.round((W - w_min) / scale).clamp(0, n_levels)
    return q * scale + w_min


def quant_intN_per_tensor(W: torch.Tensor, bits: int) -> tuple[torch.Tensor, float]:  # noqa: N802, N803
    """runner.py:114-122."""
    n_rows, in_dim = W.shape
    recon = _quant_affine(W, bits)
    return recon, (bits * n_rows * in_dim + 32) / (n_rows * in_dim)


def _affine_rows(W: torch.Tensor, bits: int) -> torch.Tensor:  # noqa: N803
    n_levels = 2**bits - 1
    w_min = W.amin(dim=-1, keepdim=True)
    w_max = W.amax(dim=-1, keepdim=True)
    scale = ((w_max - w_min) / n_levels).clamp(min=1e-10)
    q = torch.round((W - w_min) / scale).clamp(0, n_levels)
    return q * scale + w_min


def quant_intN_per_channel(W: torch.Tensor, bits: int) -> tuple[torch.Tensor, float]:  # noqa: N802, N803
    """runner.py:125-138."""
    n_rows, in_dim = W.shape
    recon = _affine_rows(W, bits)
    return recon, (bits * n_rows * in_dim + 32 * n_rows) / (n_rows * in_dim)


def quant_intN_per_block(W: torch.Tensor, bits: int, block_size: int) -> tuple[torch.Tensor, float]:  # noqa: N802, N803
    """runner.py:141-160: one min + scale per (row, block); remainder columns bf16."""
    n_rows, in_dim = W.shape
    n_blocks = in_dim // block_size
    quant_dim = n_blocks * block_size
    remainder_dim = in_dim - quant_dim
    recon = torch.empty_like(W)
    if n_blocks:
        blocks = W[:, :quant_dim].reshape(n_rows, n_blocks, block_size)
        recon[:, :quant_dim] = _affine_rows(blocks, bits).reshape(n_rows, quant_dim)
    if remainder_dim > 0:
        recon[:, quant_dim:] = W[:, quant_dim:]
    total = bits * n_rows * quant_dim + 32 * n_blocks * n_rows + 16 * n_rows * remainder_dim
    return recon, total / (n_rows * in_dim)


def quant_fp8_e4m3(W: torch.Tensor) -> tuple[torch.Tensor, float]:  # noqa: N803
    return W.to(torch.float8_e4m3fn).to(W.dtype), 8.0


def quant_fp8_e5m2(W: torch.Tensor) -> tuple[torch.Tensor, float]:  # noqa: N803
    return W.to(torch.float8_e5m2).to(W.dtype), 8.0


def integer_schemes(block_size: int) -> list[tuple[str, Callable[[torch.Tensor], tuple[torch.Tensor, float]]]]:
    """(name, quant_fn) pairs in the reference's order (runner.py:171-188)."""
    schemes: list[tuple[str, Callable[[torch.Tensor], tuple[torch.Tensor, float]]]] = []
    for bits in [2, 3, 4, 8]:
        schemes.append((f"int{bits}_per_tensor", partial(quant_intN_per_tensor, bits=bits)))
        schemes.append((f"int{bits}_per_channel", partial(quant_intN_per_channel, bits=bits)))
        schemes.append((f"int{bits}_per_block{block_size}", partial(quant_intN_per_block, bits=bits,
                                                                       block_size=block_size)))
    schemes.append(("fp8_e4m3", quant_fp8_e4m3))
    schemes.append(("fp8_e5m2", quant_fp8_e5m2))
    return schemes
