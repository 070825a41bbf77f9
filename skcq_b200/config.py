"""Experiment configuration and AQLM assembly (interface of skcq/config.py).

Same pydantic models, field names, defaults and YAML round trip as the
reference, and the same ``build_aqlm_codebook`` assembly rules
(config.py:137-197): a spherical primary of block size ``in_dim // n_blocks``
(never sign-split), euclidean residuals with ``skip_zeros=False`` and optional
SSVQ wrapping, and ``codebook_bits=16``. The codebooks it returns are this
package's B200 implementations, so ``build_aqlm_codebook(...).fit(rows)`` runs
on the GPU.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
import yaml
from pydantic import BaseModel, Field

from skcq_b200.codebook.aqlm import AQLMCodebook, AQLMCodebookConfig
from skcq_b200.codebook.base import WeightsCodebookBase
from skcq_b200.codebook.euclidean import EuclideanCodebook, EuclideanCodebookConfig
from skcq_b200.codebook.spherical import SphericalCodebook, SphericalCodebookConfig
from skcq_b200.codebook.ssvq import SSVQCodebook

__all__ = ["CodebookParams", "LayerOverride", "ExperimentConfig", "build_aqlm_codebook", "CodecSpec",
           "assemble_aqlm"]


class CodebookParams(BaseModel):
    """config.py:19-67."""

    k_gate: int = Field(default=4096, description="Codebook size for gate projection")
    k_up: int = Field(default=4096, description="Codebook size for up projection")
    k_down: int = Field(default=4096, description="Codebook size for down projection")
    n_blocks_gate_up: int = Field(default=1, description="Number of sub-blocks for gate/up input dim (PQ)")
    n_blocks_down: int = Field(default=1, description="Number of sub-blocks for down input dim (PQ)")
    n_codebooks: int = Field(default=2, description="Number of codebooks (1 = no residual, 2 = primary + 1 residual)")
    max_iters: int = Field(default=100, description="Max k-means iterations")
    norm_threshold: float = Field(
        default=0.001, description="Rows with norm below this are treated as zeros, skipped from clustering"
    )
    skip_zeros: bool = Field(default=True, description="Whether to exclude near-zero rows from codebook building")
    residual_k: int | list[int] | None = Field(
        default=None, description="K for residual codebooks (c>=1): one for all, a per-codebook list, or the primary K"
    )
    residual_block_sizes: int | list[int] | None = Field(
        default=None,
        description="Block size for residual codebooks (c>=1); leftover columns are stored raw (bf16)",
    )
    residual_sign_split: bool | list[bool] | None = Field(
        default=None, description="SSVQ sign-split for residual codebooks (c>=1)"
    )
    chunk_budget_mb: int = Field(
        default=2048, description="Accepted for compatibility; the B200 kernels do not chunk by memory budget"
    )


class LayerOverride(BaseModel):
    """config.py:70-83: every field optional; set fields override the defaults."""

    k_gate: int | None = None
    k_up: int | None = None
    k_down: int | None = None
    n_blocks_gate_up: int | None = None
    n_blocks_down: int | None = None
    n_codebooks: int | None = None
    max_iters: int | None = None
    norm_threshold: float | None = None
    skip_zeros: bool | None = None
    residual_k: int | list[int] | None = None
    residual_block_sizes: int | list[int] | None = None
    residual_sign_split: bool | list[bool] | None = None
    chunk_budget_mb: int | None = None


class ExperimentConfig(BaseModel):
    """config.py:86-113."""

    model_id: str = Field(default="Qwen/Qwen3.6-35B-A3B")
    defaults: CodebookParams = Field(default_factory=CodebookParams)
    layer_overrides: dict[int, LayerOverride] = Field(default_factory=dict)
    eval_samples: int = Field(default=1000, description="Number of C4 validation samples for perplexity")
    output_dir: Path = Field(default=Path("codebooks"))

    def params_for_layer(self, layer_idx: int) -> CodebookParams:
        if layer_idx not in self.layer_overrides:
            return self.defaults
        override = self.layer_overrides[layer_idx]
        return self.defaults.model_copy(update={k: v for k, v in override.model_dump().items() if v is not None})

    @classmethod
    def from_yaml(cls, path: str | Path) -> ExperimentConfig:
        with open(path) as f:
            data: dict[str, Any] = yaml.safe_load(f)
        return cls(**data)

    def to_yaml(self, path: str | Path) -> None:
        with open(path, "w") as f:
            yaml.dump(self.model_dump(mode="json"), f, default_flow_style=False, sort_keys=False)


def _per_codebook(value, primary, n_codebooks: int) -> list:
    """Primary value for c = 0; residual c >= 1 from a scalar, a list indexed
    c - 1, or the primary value when None (config.py:116-134)."""
    if value is None:
        return [primary] * n_codebooks
    if isinstance(value, list):
        return [primary if c == 0 else value[c - 1] for c in range(n_codebooks)]
    return [primary if c == 0 else value for c in range(n_codebooks)]


def _resolve_residual_ss(residual_ss: bool | list[bool] | None, n_codebooks: int) -> list[bool]:
    if residual_ss is None:
        return [False] * n_codebooks
    if isinstance(residual_ss, bool):
        return [residual_ss] * n_codebooks
    return list(residual_ss[:n_codebooks]) + [False] * (n_codebooks - len(residual_ss))


@dataclass(frozen=True)
class CodecSpec:
    """One codebook of a composite: its metric ("cosine" = spherical directions
    with per-row scales, "euclidean" = plain centroids), block size, K, SSVQ
    sign split, and the options of its k-means fit."""

    metric: str
    block_size: int
    K: int
    sign_split: bool = False
    skip_zeros: bool = True
    shared: bool = False
    max_train_samples: int = 0


def make_codec(spec: CodecSpec, *, max_iters: int, norm_threshold: float, chunk_budget_mb: int,
               device: torch.device | None) -> WeightsCodebookBase:
    """The B200 codec a spec describes, SSVQ-wrapped when it is sign-split."""
    cls, cfg_cls = ((SphericalCodebook, SphericalCodebookConfig) if spec.metric == "cosine"
                    else (EuclideanCodebook, EuclideanCodebookConfig))
    codec: WeightsCodebookBase = cls(cfg_cls(
        block_size=spec.block_size, K=spec.K, shared=spec.shared, max_iters=max_iters,
        norm_threshold=norm_threshold, skip_zeros=spec.skip_zeros, chunk_budget_mb=chunk_budget_mb, device=device,
        max_train_samples=spec.max_train_samples,
    ))
    return SSVQCodebook(codec) if spec.sign_split else codec


def assemble_aqlm(specs: list[CodecSpec], *, max_iters: int, norm_threshold: float, codebook_bits: int,
                  out_dim: int | None, num_experts: int | None, device: torch.device | None = None,
                  chunk_budget_mb: int = 2048) -> AQLMCodebook:
    """A composite from its codebook specs, primary first."""
    codecs = [make_codec(sp, max_iters=max_iters, norm_threshold=norm_threshold, chunk_budget_mb=chunk_budget_mb,
                         device=device) for sp in specs]
    return AQLMCodebook(
        primary=codecs[0],
        residuals=codecs[1:],
        config=AQLMCodebookConfig(codebook_bits=codebook_bits, norm_threshold=norm_threshold, device=device,
                                  out_dim=out_dim, num_experts=num_experts),
    )


def build_aqlm_codebook(
    params: CodebookParams,
    k: int,
    n_blocks: int,
    n_codebooks: int,
    in_dim: int,
    out_dim: int,
    num_experts: int = 0,
    device: torch.device | None = None,
    name: str = "",
) -> AQLMCodebook:
    """One projection's AQLM codebook (config.py:137-197): a spherical primary
    of block size in_dim // n_blocks (never sign-split), euclidean residuals
    fitted with skip_zeros=False, 16-bit centroids."""
    primary_bs = in_dim // n_blocks if n_blocks > 0 else in_dim
    bs_list = _per_codebook(params.residual_block_sizes, primary_bs, n_codebooks)
    k_list = _per_codebook(params.residual_k, k, n_codebooks)
    ss_list = _resolve_residual_ss(params.residual_sign_split, n_codebooks)
    specs = [CodecSpec("cosine", primary_bs, k, skip_zeros=params.skip_zeros)]
    specs += [CodecSpec("euclidean", bs_list[c], k_list[c], sign_split=ss_list[c], skip_zeros=False)
              for c in range(1, n_codebooks)]
    return assemble_aqlm(specs, max_iters=params.max_iters, norm_threshold=params.norm_threshold, codebook_bits=16,
                         out_dim=out_dim, num_experts=num_experts or None, device=device,
                         chunk_budget_mb=params.chunk_budget_mb)
