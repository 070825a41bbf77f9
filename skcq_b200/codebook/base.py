"""Codec plug-in interface (the contract of skcq/codebook/base.py)."""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Literal

import torch

from skcq_b200.codebook.cwr import CompressedWeightsRepresentation
from skcq_b200.codebook.events import Experiment

DistanceMetric = Literal["cosine", "euclidean"]


class WeightsCodebookBase[CWR: CompressedWeightsRepresentation](Experiment, ABC):
    """A codec: ``fit(w)`` learns centroids from ``w (n_rows, in_dim)`` and
    returns the per-row payload; ``reconstruct(cwr)`` decodes a payload (of any
    row count) to ``(n_rows_cwr, in_dim)`` float32; ``quantize_centroids`` fake
    quantises the learned centroids; ``centroids_tensor`` is
    ``(n_blocks | 1, bs, K)``."""

    @abstractmethod
    def fit(self, w: torch.Tensor) -> CWR: ...

    @abstractmethod
    def reconstruct(self, cwr: CWR) -> torch.Tensor: ...

    def quantize_centroids(self, bits: int) -> None:  # noqa: B027 - optional hook
        """Default: nothing to quantise."""

    @property
    def centroids_tensor(self) -> torch.Tensor:
        raise NotImplementedError
