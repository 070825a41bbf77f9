"""Model build driver (interface of skcq/quantize.py:17-106).

``extract_and_build_codebooks`` slices each MoE layer's fused
``gate_up_proj`` / ``down_proj`` into expert-major rows exactly as the
reference does (quantize.py:56-61) and fits one AQLM codebook per projection
on the GPU. ``cuda_worker`` keeps the reference's offload hook: any object
with a ``build_codebook(rows, params=, k=, n_blocks=, n_codebooks=,
num_experts=, out_dim=, name=)`` method is used instead of the local fit.
The multi-GPU farm (``skcq_b200.farm``) distributes the same jobs.
"""

from __future__ import annotations

import logging
from collections.abc import Mapping

import torch

from skcq_b200.codebook.aqlm import AQLMCodebook
from skcq_b200.codebook.cwr import AQLMCWR
from skcq_b200.config import CodebookParams, LayerOverride, build_aqlm_codebook

logger = logging.getLogger(__name__)


def get_text_model(model: torch.nn.Module) -> torch.nn.Module:
    """The text decoder of a CausalLM or ConditionalGeneration model (eval_model.py:11-15)."""
    if hasattr(model, "model") and hasattr(model.model, "language_model"):
        return model.model.language_model
    return model.model


def layer_params(params: CodebookParams, layer_overrides: Mapping[int, LayerOverride] | None,
                 layer_idx: int) -> CodebookParams:
    if layer_overrides and layer_idx in layer_overrides:
        return params.model_copy(
            update={k: v for k, v in layer_overrides[layer_idx].model_dump().items() if v is not None}
        )
    return params


def projection_rows(experts: torch.nn.Module, intermediate_size: int,
                    hidden_size: int) -> list[tuple[str, torch.Tensor, int]]:
    """[(name, expert-major rows, out_dim)] for gate, up and down (quantize.py:56-61)."""
    gate_up = experts.gate_up_proj.data
    down = experts.down_proj.data
    return [
        ("gate", gate_up[:, :intermediate_size, :].reshape(-1, hidden_size), intermediate_size),
        ("up", gate_up[:, intermediate_size:, :].reshape(-1, hidden_size), intermediate_size),
        ("down", down.reshape(-1, intermediate_size), hidden_size),
    ]


def extract_and_build_codebooks(
    model: torch.nn.Module,
    params: CodebookParams | None = None,
    layer_overrides: Mapping[int, LayerOverride] | None = None,
    device: torch.device | None = None,
    progress: bool = True,
    cuda_worker=None,
) -> list[dict[str, tuple[AQLMCodebook, AQLMCWR]]]:
    """quantize.py:17-106."""
    if params is None:
        params = CodebookParams()
    config = model.config
    if hasattr(config, "text_config"):
        config = config.text_config
    intermediate_size: int = config.moe_intermediate_size
    hidden_size: int = config.hidden_size
    num_experts: int = config.num_experts
    results: list[dict[str, tuple[AQLMCodebook, AQLMCWR]]] = []
    layers = get_text_model(model).layers
    for layer_idx, layer in enumerate(layers):
        if progress:
            logger.info("Processing layer %d/%d", layer_idx, len(layers))
        lp = layer_params(params, layer_overrides, layer_idx)
        ks = {"gate": (lp.k_gate, lp.n_blocks_gate_up), "up": (lp.k_up, lp.n_blocks_gate_up),
              "down": (lp.k_down, lp.n_blocks_down)}
        layer_result: dict[str, tuple[AQLMCodebook, AQLMCWR]] = {}
        for name, rows, out_dim in projection_rows(layer.mlp.experts, intermediate_size, hidden_size):
            k, n_blocks = ks[name]
            cb_name = f"L{layer_idx}.{name}"
            if cuda_worker is not None:
                layer_result[name] = cuda_worker.build_codebook(
                    rows, params=lp, k=k, n_blocks=n_blocks, n_codebooks=lp.n_codebooks, num_experts=num_experts,
                    out_dim=out_dim, name=cb_name,
                )
            else:
                aqlm = build_aqlm_codebook(lp, k=k, n_blocks=n_blocks, n_codebooks=lp.n_codebooks,
                                           in_dim=rows.shape[1], out_dim=out_dim, device=device, name=cb_name)
                layer_result[name] = (aqlm, aqlm.fit(rows))
        results.append(layer_result)
    return results
