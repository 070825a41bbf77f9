"""Weight ingest for the codebook build (interface of worker.py:62-134).

``build_layer_shard_map`` reads ``model.safetensors.index.json`` into
{layer: {"gate_up": shard file, "down": shard file}}; ``extract_rows`` reads
one layer's fused expert weights and slices them into the expert-major rows of
gate, up and down exactly as the reference (quantize.py:56-61, worker.py:98-134).
Two additions for the B200 build: ``device`` reads the tensors straight onto a
GPU (safetensors' own device placement, no host copy of the full layer kept),
and ``experts`` reads only a range of experts (the slice a row-sharded rank
fits) through safetensors' lazy slicing.

``farm_layers`` is the layer-level job farm on one node: rank r of a
``world``-rank group fits layers r, r + world, ... (each a full AQLM build of
gate, up and down, via ``build_aqlm_codebook``), with no communication.
"""

from __future__ import annotations

import json
import logging
from pathlib import Path

import torch
from safetensors import safe_open

from skcq_b200.config import CodebookParams, LayerOverride, build_aqlm_codebook
from skcq_b200.errors import InfrastructureError
from skcq_b200.quantize import layer_params

logger = logging.getLogger(__name__)

LayerShardMap = dict[int, dict[str, str]]
ProjectionRows = dict[str, torch.Tensor]

_PREFIX = "model.language_model.layers."


def _layer_of(key: str) -> int | None:
    """Layer index of a key like 'model.language_model.layers.5.mlp...' (worker.py:89-95)."""
    parts = key.split(".")
    for i, p in enumerate(parts):
        if p == "layers" and i + 1 < len(parts) and parts[i + 1].lstrip("-").isdigit():
            return int(parts[i + 1])
    return None


def build_layer_shard_map(model_dir: Path | str) -> LayerShardMap:
    """{layer: {gate_up: shard, down: shard}} from the safetensors index (worker.py:62-86)."""
    index_path = Path(model_dir) / "model.safetensors.index.json"
    if not index_path.exists():
        raise FileNotFoundError(f"No safetensors index at {index_path}")
    with open(index_path) as f:
        weight_map: dict[str, str] = json.load(f)["weight_map"]
    shards: LayerShardMap = {}
    for key, shard in weight_map.items():
        if not key.startswith(_PREFIX):
            continue
        if ".mlp.experts.gate_up_proj" in key:
            kind = "gate_up"
        elif ".mlp.experts.down_proj" in key:
            kind = "down"
        else:
            continue
        layer = _layer_of(key)
        if layer is not None:
            shards.setdefault(layer, {})[kind] = shard
    return shards


def _read(path: Path, key: str, device: str, experts: tuple[int, int] | None) -> torch.Tensor:
    with safe_open(path, framework="pt", device=device) as f:
        if experts is None:
            return f.get_tensor(key)
        return f.get_slice(key)[experts[0]:experts[1]]


def extract_rows(model_dir: Path | str, layer_idx: int, layer_shards: LayerShardMap, num_experts: int,
                 hidden_size: int, intermediate_size: int, device: str | torch.device = "cpu",
                 experts: tuple[int, int] | None = None) -> ProjectionRows:
    """{"gate": (E*I, H), "up": (E*I, H), "down": (E*H, I)} rows of one layer
    (worker.py:98-134); with ``experts = (e0, e1)`` only those experts' rows."""
    model_dir = Path(model_dir)
    dev = str(device)
    shards = layer_shards[layer_idx]
    e0, e1 = experts if experts is not None else (0, num_experts)
    if not 0 <= e0 <= e1 <= num_experts:
        raise ValueError(f"expert range {experts} outside [0, {num_experts}]")
    gate_up = _read(model_dir / shards["gate_up"], f"{_PREFIX}{layer_idx}.mlp.experts.gate_up_proj", dev, experts)
    down = _read(model_dir / shards["down"], f"{_PREFIX}{layer_idx}.mlp.experts.down_proj", dev, experts)
    if gate_up.shape != (e1 - e0, 2 * intermediate_size, hidden_size):
        raise ValueError(f"gate_up_proj of layer {layer_idx} has shape {tuple(gate_up.shape)}")
    if down.shape != (e1 - e0, hidden_size, intermediate_size):
        raise ValueError(f"down_proj of layer {layer_idx} has shape {tuple(down.shape)}")
    return {
        "gate": gate_up[:, :intermediate_size, :].reshape(-1, hidden_size),
        "up": gate_up[:, intermediate_size:, :].reshape(-1, hidden_size),
        "down": down.reshape(-1, intermediate_size),
    }


def farm_assignment(num_layers: int, world: int, rank: int) -> list[int]:
    """Layers fitted by ``rank``: round-robin over the group."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a group of {world}")
    return list(range(rank, num_layers, world))


def farm_layers(model_dir: Path | str, params: CodebookParams, num_layers: int, num_experts: int,
                hidden_size: int, intermediate_size: int, *, rank: int = 0, world: int = 1,
                layer_overrides: dict[int, LayerOverride] | None = None, device: str | torch.device = "cuda",
                retries: int = 2) -> dict[int, dict[str, tuple]]:
    """Fit this rank's layers: {layer: {proj: (AQLMCodebook, AQLMCWR)}}.

    Rows are read straight onto ``device``; each projection is fitted as in
    quantize.py:63-101 (k and n_blocks per projection, per-layer overrides).
    A (layer, projection) job that fails with an ``InfrastructureError`` (a
    device wait that ran out) is fitted again from a fresh codebook, up to
    ``retries`` more times, as the reference's workers report such a job back
    for another attempt (worker.py:256-258); after that the error propagates
    with the job in its context. Bugs (``RuntimeError``, ``ValueError``) are
    never retried."""
    shards = build_layer_shard_map(model_dir)
    out: dict[int, dict[str, tuple]] = {}
    for layer in farm_assignment(num_layers, world, rank):
        lp = layer_params(params, layer_overrides, layer)
        rows = extract_rows(model_dir, layer, shards, num_experts, hidden_size, intermediate_size, device=device)
        ks = {"gate": (lp.k_gate, lp.n_blocks_gate_up, intermediate_size),
              "up": (lp.k_up, lp.n_blocks_gate_up, intermediate_size),
              "down": (lp.k_down, lp.n_blocks_down, hidden_size)}
        result = {}
        for name in ("gate", "up", "down"):
            k, n_blocks, out_dim = ks[name]
            w = rows[name]
            for attempt in range(retries + 1):
                aqlm = build_aqlm_codebook(lp, k=k, n_blocks=n_blocks, n_codebooks=lp.n_codebooks,
                                           in_dim=w.shape[1], out_dim=out_dim, num_experts=num_experts,
                                           name=f"L{layer}.{name}")
                try:
                    result[name] = (aqlm, aqlm.fit(w))
                    break
                except InfrastructureError as e:
                    if attempt == retries:
                        raise InfrastructureError(f"layer {layer} {name}: {e}",
                                                  context={"layer": layer, "projection": name,
                                                           "attempts": attempt + 1, **e.context}) from e
                    logger.warning("layer %d %s: %s; fitting again (attempt %d of %d)", layer, name, e,
                                   attempt + 2, retries + 1)
        out[layer] = result
        del rows
    return out
