"""Model-level quality metrics for a codebook-quantized MoE (interface of
skcq/metrics.py:19-251 in the reference).

* ``install_routing_capture`` hooks every layer's ``mlp.experts`` and records
  the (top-k expert ids, top-k weights) each call receives; ``routing_agreement``
  compares two captures: the fraction of tokens whose routed expert *set* is
  unchanged, the mean cosine of the per-token routing weights (aligned by
  expert id) and the mean Jensen-Shannon divergence of those weights.
* ``capture_reference_logits`` / ``kld_against_reference``: mean
  KL(reference || model) of the next-token distributions over a token chunk.
* ``token_log_likelihoods``: log p(token_t | context) per position.

The arithmetic follows the reference step for step (same clamps, epsilons,
chunking boundaries and token counts), so numbers from either implementation
compare; the reductions run on the model's device and synchronise with the
host once per call instead of once per chunk.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F  # noqa: N812

from skcq_b200.quantize import get_text_model

logger = logging.getLogger(__name__)

_EPS = 1e-12


@dataclass
class RoutingCapture:
    """Routing decisions seen by the experts modules, one entry per call
    (metrics.py:18-44): ``top_k_index`` / ``top_k_weights`` are (tokens, top_k)
    CPU tensors, ``layer_index`` the layer that made the call (a layer may
    appear several times). A call without weights stores an empty tensor."""

    layer_index: list[int] = field(default_factory=list)
    top_k_index: list[torch.Tensor] = field(default_factory=list)
    top_k_weights: list[torch.Tensor] = field(default_factory=list)

    def reset(self) -> None:
        self.layer_index.clear()
        self.top_k_index.clear()
        self.top_k_weights.clear()

    def num_calls(self) -> int:
        return len(self.layer_index)

    def per_layer_index_tensors(self) -> dict[int, list[torch.Tensor]]:
        out: dict[int, list[torch.Tensor]] = {}
        for layer, idx in zip(self.layer_index, self.top_k_index, strict=True):
            out.setdefault(layer, []).append(idx)
        return out

    def per_layer_weight_tensors(self) -> dict[int, list[torch.Tensor]]:
        out: dict[int, list[torch.Tensor]] = {}
        for layer, w in zip(self.layer_index, self.top_k_weights, strict=True):
            out.setdefault(layer, []).append(w)
        return out


def install_routing_capture(model: torch.nn.Module) -> tuple[RoutingCapture, list]:
    """Forward pre-hooks on every layer's ``mlp.experts`` (metrics.py:47-80).

    Both the original experts module and ``CodebookExperts`` take
    ``(hidden_states, top_k_index, top_k_weights)`` positionally; calls whose
    second argument is not a tensor are ignored."""
    capture = RoutingCapture()
    handles = []
    for layer_idx, layer in enumerate(get_text_model(model).layers):

        def hook(_module, args, _layer=layer_idx):
            if len(args) < 2 or not isinstance(args[1], torch.Tensor):
                return
            capture.layer_index.append(_layer)
            capture.top_k_index.append(args[1].detach().cpu())
            w = args[2] if len(args) >= 3 and isinstance(args[2], torch.Tensor) else None
            capture.top_k_weights.append(w.detach().cpu() if w is not None else torch.empty(0))

        handles.append(layer.mlp.experts.register_forward_pre_hook(hook))
    return capture, handles


def remove_hooks(handles: list) -> None:
    for h in handles:
        h.remove()


def _weights_by_expert_id(weights: list[torch.Tensor], idx: torch.Tensor) -> torch.Tensor | None:
    """One layer's weights, each row reordered by ascending expert id
    (metrics.py:161-179): None when the calls carry no weights or the row
    counts disagree."""
    if not weights or weights[0].numel() == 0:
        return None
    w = torch.cat(weights, dim=0)
    if w.shape[0] != idx.shape[0]:
        return None
    return w.gather(-1, idx.argsort(dim=-1, stable=True))


def _js_divergence(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Row-wise symmetric Jensen-Shannon divergence of non-negative weights,
    each row renormalised to sum 1 (metrics.py:182-193)."""
    a = a.clamp_min(0)
    b = b.clamp_min(0)
    a = a / a.sum(-1, keepdim=True).clamp_min(_EPS)
    b = b / b.sum(-1, keepdim=True).clamp_min(_EPS)
    m = 0.5 * (a + b)
    lm = (m + _EPS).log()
    kl_am = (a * ((a + _EPS).log() - lm)).sum(-1)
    kl_bm = (b * ((b + _EPS).log() - lm)).sum(-1)
    return 0.5 * (kl_am + kl_bm)


def routing_agreement(base: RoutingCapture, quant: RoutingCapture) -> dict[str, object]:
    """Compare two captures layer by layer (metrics.py:88-158).

    For every layer present in both with the same (tokens, top_k): tokens whose
    sorted expert ids match, the cosine of the expert-id-aligned weights and
    their Jensen-Shannon divergence. Layers whose shapes differ are skipped
    with a warning."""
    b_idx, q_idx = base.per_layer_index_tensors(), quant.per_layer_index_tensors()
    b_w, q_w = base.per_layer_weight_tensors(), quant.per_layer_weight_tensors()
    layers = sorted(set(b_idx) & set(q_idx))
    tokens = same_set = 0
    cos_sum = jsd_sum = 0.0
    cos_n = jsd_n = 0
    per_layer: list[dict[str, object]] = []
    for layer in layers:
        bi = torch.cat(b_idx[layer], dim=0)
        qi = torch.cat(q_idx[layer], dim=0)
        if bi.shape != qi.shape:
            logger.warning("routing layer %d: shape mismatch %s vs %s, skipping", layer, tuple(bi.shape),
                           tuple(qi.shape))
            continue
        n = bi.shape[0]
        tokens += n
        match = (bi.sort(dim=-1).values == qi.sort(dim=-1).values).all(dim=-1)
        same_set += int(match.sum())
        bw = _weights_by_expert_id(b_w[layer], bi)
        qw = _weights_by_expert_id(q_w[layer], qi)
        if bw is not None and qw is not None and bw.shape == qw.shape:
            cos = F.cosine_similarity(bw, qw, dim=-1)
            cos_sum += float(cos.sum())
            cos_n += cos.numel()
            jsd = _js_divergence(bw, qw)
            jsd_sum += float(jsd.sum())
            jsd_n += jsd.numel()
        per_layer.append({"layer": layer, "tokens": n, "set_agreement": float(match.float().mean()) if n else 0.0})
    return {
        "common_layers": len(layers),
        "total_tokens": tokens,
        "set_agreement": same_set / tokens if tokens else 0.0,
        "weight_cosine": cos_sum / cos_n if cos_n else 0.0,
        "routing_jsd": jsd_sum / jsd_n if jsd_n else 0.0,
        "per_layer": per_layer,
    }


@torch.no_grad()
def capture_reference_logits(model: torch.nn.Module, input_ids: torch.Tensor, max_length: int = 2048) -> torch.Tensor:
    """fp32 next-token logits of the first ``max_length`` positions, shape
    (min(max_length, seq_len) - 1, vocab), on the model's device
    (metrics.py:196-207)."""
    logits = model(input_ids[:, :max_length]).logits
    return logits[:, :-1].float().squeeze(0)


@torch.no_grad()
def kld_against_reference(model: torch.nn.Module, input_ids: torch.Tensor, reference_logits: torch.Tensor,
                          token_chunk: int = 256) -> float:
    """Mean over tokens of KL(reference || model) on the chunk the reference
    logits were taken from (metrics.py:210-237), ``token_chunk`` positions of
    log-softmax at a time; one host synchronisation."""
    logits = model(input_ids[:, : reference_logits.shape[0] + 1]).logits[:, :-1].float().squeeze(0)
    n = min(reference_logits.shape[0], logits.shape[0])
    ref = reference_logits[:n].to(logits.device)
    total = torch.zeros((), dtype=torch.float64, device=logits.device)
    for i in range(0, n, token_chunk):
        j = min(i + token_chunk, n)
        log_p = F.log_softmax(ref[i:j], dim=-1)
        log_q = F.log_softmax(logits[i:j], dim=-1)
        total += (log_p.exp() * (log_p - log_q)).sum(-1).sum(dtype=torch.float64)
    return float(total) / n


@torch.no_grad()
def token_log_likelihoods(model: torch.nn.Module, input_ids: torch.Tensor) -> torch.Tensor:
    """log p(token_t | tokens_<t) for t = 1 .. seq_len - 1, on the CPU
    (metrics.py:240-251)."""
    logits = model(input_ids).logits[:, :-1].float()
    lp = F.log_softmax(logits, dim=-1).gather(-1, input_ids[:, 1:].unsqueeze(-1)).squeeze(-1)
    return lp.squeeze(0).cpu()
