"""Quality of a codebook-quantized MoE against its dense original (the flow of
eval_quantized.py:86-179 in the reference, as a library call).

``evaluate_quantized`` takes the dense model, measures its perplexity, its
reference next-token logits over the first ``kld_tokens`` tokens and its
routing decisions there, installs the codebook experts in place
(``serialization.replace_experts`` by default), measures the same on the
quantized model and returns the reference's summary keys. The reference
caches the dense baseline from another process; here both sides run in one.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from skcq_b200.eval_model import compute_perplexity
from skcq_b200.metrics import (capture_reference_logits, install_routing_capture, kld_against_reference,
                               remove_hooks, routing_agreement)


def _routing(model: torch.nn.Module, input_ids: torch.Tensor):
    capture, handles = install_routing_capture(model)
    try:
        with torch.no_grad():
            model(input_ids)
    finally:
        remove_hooks(handles)
    return capture


def evaluate_quantized(model: torch.nn.Module, tokenizer: object, text: str, codebook_modules: list,
                       num_experts: int, *, kld_tokens: int = 2048, max_length: int = 2048, stride: int = 512,
                       replace: Callable | None = None) -> dict[str, object]:
    """Dense baseline, expert replacement, quantized metrics; ``model`` is
    modified in place (its experts become the codebook experts)."""
    if replace is None:
        from skcq_b200.serialization import replace_experts as replace
    input_ids = tokenizer(text, return_tensors="pt").input_ids.to(model.device)
    base_ppl = compute_perplexity(model, tokenizer, text, max_length=max_length, stride=stride)
    ref_logits = capture_reference_logits(model, input_ids, max_length=kld_tokens)
    base_routing = _routing(model, input_ids[:, :kld_tokens])

    replace(model, codebook_modules, num_experts)
    quant_ppl = compute_perplexity(model, tokenizer, text, max_length=max_length, stride=stride)
    kld = kld_against_reference(model, input_ids, ref_logits)
    quant_routing = _routing(model, input_ids[:, :kld_tokens])
    return {
        "baseline_ppl": base_ppl,
        "quantized_ppl": quant_ppl,
        "ppl_ratio": quant_ppl / base_ppl if base_ppl else None,
        "ppl_delta": quant_ppl - base_ppl,
        "kld_base_to_quant": kld,
        "kld_tokens": kld_tokens,
        "routing": routing_agreement(base_routing, quant_routing),
    }
