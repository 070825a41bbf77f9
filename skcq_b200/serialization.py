"""On-disk codebooks (interface of build.py:30-106 in the reference).

``save_codebooks`` / ``load_codebooks`` write and read the reference's layout:
``<dir>/layer_<i>/{gate,up,down}.pt``, each file
``CodebookModule.state_dict_with_meta()``, so directories written by either
implementation load in the other. ``modules_from_results`` and
``replace_experts`` are the reference's helpers for turning build results into
modules and installing them in a Hugging Face MoE model.

``save_packed`` / ``load_packed`` store one module compactly: assignments as
16-bit indices (the reference keeps int64), SSVQ signs as one bit each (the
reference keeps int8), everything else as is. ``load_packed`` restores the
reference's keys, dtypes and values exactly.
"""

from __future__ import annotations

import logging
from pathlib import Path
from typing import Any

import torch

from skcq_b200.codebook_experts import CodebookExperts, CodebookModule
from skcq_b200.quantize import get_text_model

logger = logging.getLogger(__name__)

PROJECTIONS = ("gate", "up", "down")
PACKED_FORMAT = "skcq_b200.packed.v1"


def modules_from_results(codebook_results: list[dict[str, tuple[Any, Any]]]) -> list[dict[str, CodebookModule]]:
    """(AQLMCodebook, AQLMCWR) pairs -> CodebookModules (build.py:30-43)."""
    modules: list[dict[str, CodebookModule]] = []
    for layer_result in codebook_results:
        layer_modules: dict[str, CodebookModule] = {}
        for name in PROJECTIONS:
            aqlm, cwr = layer_result[name]
            if aqlm.config is None or aqlm.config.out_dim is None:
                raise ValueError(f"{name}: AQLMCodebookConfig.out_dim is required to build a module")
            layer_modules[name] = CodebookModule.from_cwr(aqlm, cwr, out_dim=aqlm.config.out_dim)
        modules.append(layer_modules)
    return modules


def replace_experts(model: torch.nn.Module, codebook_modules: list[dict[str, CodebookModule]],
                    num_experts: int) -> None:
    """Install CodebookExperts in place of every layer's ``mlp.experts``
    (build.py:46-72); the experts' ``act_fn`` is kept."""
    text_model = get_text_model(model)
    num_layers = len(text_model.layers)
    for layer_idx, layer in enumerate(text_model.layers):
        mlp = layer.mlp
        experts = CodebookExperts(
            gate=codebook_modules[layer_idx]["gate"], up=codebook_modules[layer_idx]["up"],
            down=codebook_modules[layer_idx]["down"], num_experts=num_experts, act_fn=mlp.experts.act_fn,
        )
        mlp.experts = experts.to(next(mlp.experts.parameters()).device)
        if (layer_idx + 1) % 5 == 0 or layer_idx + 1 == num_layers:
            logger.info("Replacing experts: %d/%d layers", layer_idx + 1, num_layers)


def save_codebooks(codebook_results: list[dict[str, tuple[Any, Any]]], output_dir: Path | str) -> None:
    """``<output_dir>/layer_<i>/<proj>.pt`` = state_dict_with_meta (build.py:75-91)."""
    output_dir = Path(output_dir)
    output_dir.mkdir(parents=True, exist_ok=True)
    for layer_idx, layer_modules in enumerate(modules_from_results(codebook_results)):
        layer_dir = output_dir / f"layer_{layer_idx}"
        layer_dir.mkdir(exist_ok=True)
        for name in PROJECTIONS:
            torch.save(layer_modules[name].state_dict_with_meta(), layer_dir / f"{name}.pt")


def load_codebooks(codebook_dir: Path | str, num_layers: int) -> list[dict[str, CodebookModule]]:
    """Modules saved by ``save_codebooks`` (build.py:94-106)."""
    codebook_dir = Path(codebook_dir)
    return [{name: CodebookModule.load(codebook_dir / f"layer_{i}" / f"{name}.pt") for name in PROJECTIONS}
            for i in range(num_layers)]


def _pack_signs(signs: torch.Tensor) -> torch.Tensor:
    """int8 +-1 (..., n) -> uint8 (..., ceil(n / 8)), bit j of byte i = column 8i + j negative."""
    if not bool(((signs == 1) | (signs == -1)).all()):
        raise ValueError("packed signs hold +-1 only")
    neg = (signs < 0).to(torch.uint8)
    n = neg.shape[-1]
    pad = (-n) % 8
    if pad:
        neg = torch.nn.functional.pad(neg, (0, pad))
    neg = neg.reshape(*neg.shape[:-1], -1, 8)
    weights = torch.tensor([1 << j for j in range(8)], dtype=torch.uint8, device=neg.device)
    return (neg * weights).sum(-1, dtype=torch.uint8)


def _unpack_signs(packed: torch.Tensor, n: int) -> torch.Tensor:
    bits = torch.tensor([1 << j for j in range(8)], dtype=torch.uint8, device=packed.device)
    neg = (packed.unsqueeze(-1) & bits) != 0
    neg = neg.reshape(*packed.shape[:-1], -1)[..., :n]
    return torch.where(neg, -1, 1).to(torch.int8)


def save_packed(module: CodebookModule, path: Path | str) -> None:
    """One module with 16-bit indices and 1-bit signs (see module docstring)."""
    data = module.state_dict_with_meta()
    sd = data["state_dict"]
    packed: dict[str, torch.Tensor] = {}
    shapes: dict[str, list[int]] = {}
    for key, value in sd.items():
        t = value.detach().cpu()
        if key.endswith(".assignments"):
            if t.numel() and (int(t.min()) < 0 or int(t.max()) > 65535):
                raise ValueError(f"{key}: indices outside [0, 65535] cannot be packed to 16 bits")
            packed[key] = t.to(torch.int32).to(torch.int16)  # two's-complement wrap of 32768..65535
        elif key.endswith(".signs") and t.numel():
            packed[key] = _pack_signs(t)
            shapes[key] = list(t.shape)
        else:
            packed[key] = t
    torch.save({"format": PACKED_FORMAT, "meta": data["meta"], "tensors": packed, "sign_shapes": shapes}, path)


def load_packed(path: Path | str) -> CodebookModule:
    """A module saved by ``save_packed``, with the reference's keys and dtypes."""
    data = torch.load(path, weights_only=True)
    if data.get("format") != PACKED_FORMAT:
        raise ValueError(f"{path}: not a {PACKED_FORMAT} file")
    sd: dict[str, torch.Tensor] = {}
    for key, t in data["tensors"].items():
        if key.endswith(".assignments"):
            sd[key] = t.to(torch.int64) & 0xFFFF
        elif key in data["sign_shapes"]:
            shape = data["sign_shapes"][key]
            sd[key] = _unpack_signs(t, shape[-1]).reshape(shape)
        else:
            sd[key] = t
    meta = data["meta"]
    module = CodebookModule.empty(
        n_blocks=meta["n_blocks"], block_size=meta["block_size"], out_dim=meta["out_dim"], k_list=meta["k_list"],
        num_experts=meta["num_experts"], n_blocks_list=meta.get("n_blocks_list"),
        block_size_list=meta.get("block_size_list"), rem_list=meta.get("rem_list"),
        sign_cov_list=meta.get("sign_cov_list"), has_scale_list=meta.get("has_scale_list"),
    )
    # match floating dtypes to the saved ones before loading (empty() is bf16)
    for name, p in list(module.named_parameters()) + list(module.named_buffers()):
        if name in sd and p is not None and p.is_floating_point() and sd[name].is_floating_point():
            p.data = p.data.to(sd[name].dtype)
    module.load_state_dict(sd)
    return module
