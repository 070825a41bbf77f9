"""Compressed-weight payloads (the field layout of skcq/codebook/cwr.py).

These dataclasses are the drop-in boundary's data format: the same names,
fields, shapes and dtypes as the reference, so payloads move between the two
implementations unchanged. ``n_rows`` is the CWR's own row count (a CWR may
hold a subset of the rows a codebook was trained on).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class CompressedWeightsRepresentation:
    """Base of every per-row compressed payload returned by ``fit``."""


@dataclass
class EuclideanCWR(CompressedWeightsRepresentation):
    """Euclidean codec payload: ``idxs (n_blocks, n_rows) int64``,
    ``remainder (n_rows, rem) bf16`` or None."""

    idxs: torch.Tensor
    remainder: torch.Tensor | None


@dataclass
class SphericalCWR(CompressedWeightsRepresentation):
    """Spherical codec payload: ``idxs (n_blocks, n_rows) int64``, per-(row,
    block) ``scales (n_rows, n_blocks)`` (f32 after fit; bf16/fp16/fp8/int
    after ``quantize_spherical_scales``), ``remainder (n_rows, rem) bf16``."""

    idxs: torch.Tensor
    scales: torch.Tensor
    remainder: torch.Tensor | None


@dataclass
class SSVQCWR[CWR: CompressedWeightsRepresentation](CompressedWeightsRepresentation):
    """Sign-split wrapper: ``signs (n_rows, in_dim) int8`` of +-1 over the
    inner payload."""

    inner: CWR
    signs: torch.Tensor


@dataclass
class AQLMCWR(CompressedWeightsRepresentation):
    """Composite payload: the primary's and each residual's CWR."""

    primary: CompressedWeightsRepresentation
    residuals: list[CompressedWeightsRepresentation]


def cwr_to(cwr: CompressedWeightsRepresentation, device: torch.device) -> CompressedWeightsRepresentation:
    """Move every tensor of a (possibly nested) payload to ``device``."""

    def mv(t):
        if not isinstance(t, torch.Tensor):
            return t
        if device.type == "cpu" and t.is_cuda:
            from skcq_b200._engine import to_host

            return to_host(t)
        return t.to(device)

    if isinstance(cwr, AQLMCWR):
        return AQLMCWR(cwr_to(cwr.primary, device), [cwr_to(r, device) for r in cwr.residuals])
    if isinstance(cwr, SSVQCWR):
        return SSVQCWR(cwr_to(cwr.inner, device), mv(cwr.signs))
    if isinstance(cwr, SphericalCWR):
        return SphericalCWR(mv(cwr.idxs), mv(cwr.scales), mv(cwr.remainder))
    if isinstance(cwr, EuclideanCWR):
        return EuclideanCWR(mv(cwr.idxs), mv(cwr.remainder))
    raise TypeError(f"Unknown CWR type: {type(cwr)}")
