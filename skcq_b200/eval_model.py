"""Model loading and perplexity for the quality evaluation (interface of
skcq/eval_model.py:11-150 in the reference).

``compute_perplexity`` is the reference's sliding-window perplexity: windows of
``max_length`` tokens starting every ``stride`` tokens, every window after the
first scoring only its last ``stride`` targets, cross-entropy summed over the
scored targets of all windows and exponentiated once. Here the per-window
sums stay on the device (one host synchronisation at the end). ``load_model``
reads a Hugging Face checkpoint (a local directory here: there is no network);
``get_calibration_text`` streams C4 through the ``datasets`` package when it is
installed, or reads a local text file.
"""

from __future__ import annotations

import logging
import math
from pathlib import Path

import torch
import torch.nn.functional as F  # noqa: N812

from skcq_b200.quantize import get_text_model

logger = logging.getLogger(__name__)

__all__ = ["compute_perplexity", "get_calibration_text", "get_text_model", "load_model"]


def load_model(model_id: str, device: str = "auto") -> tuple[torch.nn.Module, object]:
    """(model in bf16, tokenizer) from ``model_id`` (eval_model.py:18-51); with
    ``device="auto"`` and a GPU present the weights load on the CPU and move to
    the GPU afterwards."""
    from transformers import AutoModelForCausalLM, AutoTokenizer

    tokenizer = AutoTokenizer.from_pretrained(model_id, trust_remote_code=True)
    on_gpu = device == "auto" and torch.cuda.is_available()
    model = AutoModelForCausalLM.from_pretrained(model_id, device_map="cpu" if on_gpu else device,
                                                 dtype=torch.bfloat16, trust_remote_code=True)
    model.eval()
    if on_gpu:
        model = model.to(device="cuda")
    return model, tokenizer


@torch.no_grad()
def compute_perplexity(model: torch.nn.Module, tokenizer: object, text: str, max_length: int = 2048,
                       stride: int = 512, token_chunk: int = 256) -> float:
    """Sliding-window perplexity of ``text`` (eval_model.py:54-129)."""
    input_ids = tokenizer(text, return_tensors="pt").input_ids.to(model.device)
    seq_len = input_ids.size(1)
    nll = torch.zeros((), dtype=torch.float64, device=input_ids.device)
    count = torch.zeros((), dtype=torch.int64, device=input_ids.device)
    for begin in range(0, seq_len, stride):
        end = min(begin + max_length, seq_len)
        chunk = input_ids[:, begin:end]
        targets = chunk.clone()
        if begin > 0:
            targets[:, :-stride] = -100  # earlier windows scored these
        logits = model(chunk).logits[..., :-1, :]
        labels = targets[..., 1:]
        for i in range(0, logits.size(1), token_chunk):
            j = min(i + token_chunk, logits.size(1))
            lab = labels[:, i:j].reshape(-1)
            nll += F.cross_entropy(logits[:, i:j].float().reshape(-1, logits.size(-1)), lab, ignore_index=-100,
                                   reduction="sum").double()
            count += (lab != -100).sum()
        if end >= seq_len:
            break
    return math.exp(float(nll) / int(count))


def get_calibration_text(num_samples: int = 1000, path: str | Path | None = None) -> str:
    """``num_samples`` C4 validation documents joined by newlines
    (eval_model.py:132-150), or the first ``num_samples`` lines of the text
    file at ``path``."""
    if path is not None:
        with open(path, encoding="utf-8") as f:
            return "\n".join(line.rstrip("\n") for _, line in zip(range(num_samples), f))
    try:
        from datasets import load_dataset  # type: ignore[import-untyped]
    except ImportError as e:
        raise RuntimeError("get_calibration_text needs the `datasets` package (C4) or a local text file path") from e
    ds = load_dataset("allenai/c4", "en", split="validation", streaming=True)
    texts = [s["text"] for _, s in zip(range(num_samples), ds)]
    return "\n".join(texts)
