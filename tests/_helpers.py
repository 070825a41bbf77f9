"""Shared helpers for the test-suite (fixtures loading, init replay, comparisons)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def sub(d: dict, prefix: str) -> dict:
    return {k[len(prefix):]: v for k, v in d.items() if k.startswith(prefix)}


def sobol_np(k: int, d: int) -> np.ndarray:
    """The reference's initial directions (skcq/codebook/kmeans.py:69-74)."""
    sob = torch.quasirandom.SobolEngine(dimension=d, scramble=True, seed=42)
    pts = sob.draw(k).clamp(min=1e-6)
    return torch.nn.functional.normalize(pts, dim=-1).numpy()


class PermReplay:
    """Replays recorded ``torch.randperm`` draws in order."""

    def __init__(self, lens: np.ndarray, flat: np.ndarray) -> None:
        self.perms = np.split(flat.astype(np.int64), np.cumsum(lens)[:-1]) if len(lens) else []
        self.i = 0

    @classmethod
    def from_case(cls, d: dict) -> PermReplay:
        return cls(d["perm_lens"], d["perm_flat"])

    def __call__(self, n: int) -> np.ndarray:
        p = self.perms[self.i]
        self.i += 1
        assert len(p) == n, f"recorded permutation has length {len(p)}, asked {n}"
        return p

    def torch_patch(self):
        """A drop-in for ``torch.randperm`` returning the recorded draws."""

        def randperm(n, *a, device=None, **kw):
            return torch.from_numpy(self(int(n))).to(device if device is not None else "cpu")

        return randperm


def bf16_from_bits(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.int32).astype(np.uint32) << 16).view(np.float32)


def label_agreement(a: np.ndarray, b: np.ndarray, margin: np.ndarray, tol: float) -> tuple[int, int]:
    """(#disagreements where margin > tol, #rows with margin > tol)."""
    m = margin > tol
    return int((a[m] != b[m]).sum()), int(m.sum())


def rel_err(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


class TinyLM(torch.nn.Module):
    """A small deterministic causal language model for the eval metrics: token
    embeddings, a running mean over the prefix (so every position depends on its
    context) and an output projection. ``model(ids).logits`` has the shape of a
    Hugging Face causal LM's output; weights come from ``seed``."""

    def __init__(self, vocab: int = 97, dim: int = 24, seed: int = 0, noise: float = 0.0) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.emb = torch.nn.Parameter(torch.randn(vocab, dim, generator=g))
        self.out = torch.nn.Parameter(torch.randn(dim, vocab, generator=g) * 0.5)
        if noise:
            with torch.no_grad():
                self.out.add_(torch.randn(dim, vocab, generator=g) * noise)

    @property
    def device(self) -> torch.device:
        return self.emb.device

    def forward(self, ids: torch.Tensor):
        h = self.emb[ids]
        steps = torch.arange(1, ids.shape[1] + 1, device=ids.device, dtype=h.dtype).view(1, -1, 1)
        h = h.cumsum(dim=1) / steps
        return type("Out", (), {"logits": h @ self.out})()


class CharTokenizer:
    """``tokenizer(text, return_tensors="pt").input_ids``: one id per character."""

    def __init__(self, vocab: int = 97) -> None:
        self.vocab = vocab

    def __call__(self, text: str, return_tensors: str = "pt"):
        ids = torch.tensor([[ord(c) % self.vocab for c in text]], dtype=torch.long)
        return type("Enc", (), {"input_ids": ids})()


def routing_calls(seed: int, calls: list[tuple[int, int]], top_k: int = 4, experts: int = 16,
                  weights: bool = True) -> list[tuple[int, torch.Tensor, torch.Tensor]]:
    """Synthetic routing decisions: one (layer, top-k ids, top-k weights) per MoE call."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for layer, tokens in calls:
        ids = torch.stack([torch.randperm(experts, generator=g)[:top_k] for _ in range(tokens)])
        w = torch.softmax(torch.randn(tokens, top_k, generator=g), dim=-1) if weights else torch.empty(0)
        out.append((layer, ids, w))
    return out


def perturb_routing(calls, seed: int, experts: int = 16):
    """A 'quantized' copy of ``calls``: some rows get one expert replaced, some rows
    are reordered (same set), every weight is jittered."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for layer, ids, w in calls:
        ids = ids.clone()
        n, k = ids.shape
        for r in range(n):
            u = float(torch.rand(1, generator=g))
            if u < 0.2:
                pool = [e for e in range(experts) if e not in ids[r].tolist()]
                ids[r, int(torch.randint(k, (1,), generator=g))] = pool[int(torch.randint(len(pool), (1,), generator=g))]
            elif u < 0.5:
                ids[r] = ids[r, torch.randperm(k, generator=g)]
        if w.numel():
            w = (w * (1 + 0.1 * torch.randn(w.shape, generator=g))).clamp_min(0)
        out.append((layer, ids, w))
    return out


class DenseExperts(torch.nn.Module):
    """Fused-weight MoE experts in the Hugging Face layout (gate_up_proj (E, 2I, H),
    down_proj (E, H, I), act_fn) with the experts-module call signature
    ``(hidden (T, H), top_k_index (T, k), top_k_weights (T, k)) -> (T, H)``."""

    def __init__(self, E: int, H: int, I: int, g: torch.Generator, scale: float = 0.2) -> None:
        super().__init__()
        self.gate_up_proj = torch.nn.Parameter(torch.randn(E, 2 * I, H, generator=g) * scale)
        self.down_proj = torch.nn.Parameter(torch.randn(E, H, I, generator=g) * scale)
        self.act_fn = torch.nn.functional.silu
        self.I = I

    def forward(self, hidden, top_k_index, top_k_weights):
        out = torch.zeros_like(hidden)
        for e in range(self.gate_up_proj.shape[0]):
            tok, slot = torch.where(top_k_index == e)
            if tok.numel() == 0:
                continue
            gu = hidden[tok] @ self.gate_up_proj[e].T
            h = self.act_fn(gu[:, : self.I]) * gu[:, self.I:]
            out.index_add_(0, tok, (h @ self.down_proj[e].T) * top_k_weights[tok, slot, None])
        return out


class TinyMoE(torch.nn.Module):
    """A small causal MoE language model in the Hugging Face module layout
    (``model.model.layers[i].mlp.{gate, experts}``): embeddings, per layer a
    softmax top-k router and fused experts added to the residual stream, and an
    output projection; the running prefix mean keeps positions context-dependent."""

    def __init__(self, vocab: int = 97, H: int = 32, I: int = 16, E: int = 4, layers: int = 2, top_k: int = 2,
                 seed: int = 0) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.emb = torch.nn.Parameter(torch.randn(vocab, H, generator=g))
        self.out = torch.nn.Parameter(torch.randn(H, vocab, generator=g) * 0.3)
        self.top_k = top_k
        self.model = torch.nn.Module()
        self.model.layers = torch.nn.ModuleList()
        for _ in range(layers):
            layer = torch.nn.Module()
            layer.mlp = torch.nn.Module()
            layer.mlp.gate = torch.nn.Linear(H, E, bias=False)
            with torch.no_grad():
                layer.mlp.gate.weight.copy_(torch.randn(E, H, generator=g))
            layer.mlp.experts = DenseExperts(E, H, I, g)
            self.model.layers.append(layer)

    @property
    def device(self) -> torch.device:
        return self.emb.device

    def forward(self, ids: torch.Tensor):
        h = self.emb[ids]
        steps = torch.arange(1, ids.shape[1] + 1, device=ids.device, dtype=h.dtype).view(1, -1, 1)
        h = h.cumsum(dim=1) / steps
        for layer in self.model.layers:
            x = h.reshape(-1, h.shape[-1])
            probs = torch.softmax(layer.mlp.gate(x.to(layer.mlp.gate.weight.dtype)).float(), dim=-1)
            w, i = probs.topk(self.top_k, dim=-1)
            w = w / w.sum(-1, keepdim=True)
            h = h + layer.mlp.experts(x, i, w.to(x.dtype)).reshape(h.shape).to(h.dtype)
        return type("Out", (), {"logits": h @ self.out})()
