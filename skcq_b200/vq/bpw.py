"""Bits-per-weight accounting of a k-means codebook composite (the formula of
skcq/vq/bpw.py:34-96, used to report results in the reference's units).

Per codebook c (block size bs_c, K_c centroids, n_blocks_c = in_dim // bs_c):
centroid storage ``n_cb * K_c * bs_c * codebook_bits`` (n_cb = 1 when shared),
indices ``n_rows * n_blocks_c * ceil(log2 K_c)`` (1 bit when K_c <= 1), raw
bf16 remainder ``16 * n_rows * (in_dim - n_blocks_c * bs_c)``, one sign bit
per covered element when sign-split; plus, for a cosine primary only,
``n_rows * n_blocks * scale_bits`` of scales.
"""

from __future__ import annotations

import math


def bits_per_weight_kmeans(
    n_rows: int,
    in_dim: int,
    n_blocks: int,
    block_size: int,
    n_codebooks: int,
    k_per_codebook: list[int],
    shared_codebook: bool = False,
    sign_split: bool = False,
    scale_bits_per_elem: int = 16,
    bs_per_codebook: list[int] | None = None,
    codebook_bits: int = 16,
    residual_sign_split: bool | list[bool] | None = None,
    primary_metric: str = "cosine",
) -> float:
    bss = bs_per_codebook if bs_per_codebook is not None else [block_size] * n_codebooks
    if residual_sign_split is None:
        res_ss = [False] * (n_codebooks - 1)
    elif isinstance(residual_sign_split, bool):
        res_ss = [residual_sign_split] * (n_codebooks - 1)
    else:
        res_ss = list(residual_sign_split)[: n_codebooks - 1]
        res_ss += [False] * (n_codebooks - 1 - len(res_ss))
    sign_flags = [sign_split, *res_ss]
    total = 0
    for c, (bs_c, k_c) in enumerate(zip(bss, k_per_codebook, strict=True)):
        nb_c = in_dim // bs_c
        cov_c = nb_c * bs_c
        total += (1 if shared_codebook else nb_c) * k_c * bs_c * codebook_bits
        total += n_rows * nb_c * (1 if k_c <= 1 else math.ceil(math.log2(k_c)))
        total += n_rows * (in_dim - cov_c) * 16
        if sign_flags[c]:
            total += n_rows * cov_c
    if primary_metric == "cosine":
        total += n_rows * n_blocks * scale_bits_per_elem
    return total / (n_rows * in_dim)
