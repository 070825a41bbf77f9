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
