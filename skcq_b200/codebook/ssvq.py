"""Sign-split combinator on B200 (interface of skcq/codebook/ssvq.py).

``fit`` folds the weights to |w| (sign 0 counts as +1), fits the inner codec
on the folded matrix and keeps int8 +-1 signs over the full input width;
``reconstruct`` re-applies them to the inner reconstruction.
"""

from __future__ import annotations

import logging

import torch

from skcq_b200 import _engine
from skcq_b200.codebook.base import WeightsCodebookBase
from skcq_b200.codebook.cwr import SSVQCWR
from skcq_b200.codebook.events import Experiment, KmeansDoneEvent, KmeansIterEvent, KmeansStartEvent

logger = logging.getLogger(__name__)


class SSVQCodebook(WeightsCodebookBase[SSVQCWR], Experiment):
    """Wraps any codec of this package with per-element signs."""

    def __init__(self, inner: WeightsCodebookBase) -> None:
        Experiment.__init__(self)
        self.inner = inner
        for ev in (KmeansStartEvent, KmeansIterEvent, KmeansDoneEvent):
            self._forward_from(inner, ev)

    def fit(self, w: torch.Tensor) -> SSVQCWR:
        """ssvq.py:41-55: one vectorised fold kernel, then the inner fit."""
        out_dev = w.device
        dev = _engine.cuda_device(None, w)
        folded, signs = _engine.ssvq_fold(w.to(dev))
        inner_cwr = self.inner.fit(folded if w.is_cuda else folded.to(out_dev))
        return SSVQCWR(inner=inner_cwr, signs=signs.to(out_dev))

    def views(self, cwr: SSVQCWR, dev: torch.device) -> list[_engine.CodecView]:
        v = self.inner.views(cwr.inner, dev)
        assert len(v) == 1
        signs = cwr.signs.to(device=dev, dtype=torch.int8)
        if signs.stride(-1) != 1:
            signs = signs.contiguous()
        width = v[0].n_blocks * v[0].bs + (v[0].rem.shape[1] if v[0].rem is not None else 0)
        v[0].signs = signs
        v[0].sign_cols = min(width, signs.shape[1])  # ssvq.py:62-65
        return v

    def reconstruct(self, cwr: SSVQCWR) -> torch.Tensor:
        """ssvq.py:57-66."""
        inner_cwr = cwr.inner
        out_dev = inner_cwr.idxs.device
        dev = _engine.cuda_device(None, inner_cwr.idxs)
        v = self.views(cwr, dev)
        n_rows = inner_cwr.idxs.shape[1]
        in_dim = v[0].n_blocks * v[0].bs + (v[0].rem.shape[1] if v[0].rem is not None else 0)
        return _engine.reconstruct(v, n_rows, in_dim).to(out_dev)

    def quantize_centroids(self, bits: int) -> None:
        self.inner.quantize_centroids(bits)

    @property
    def centroids_tensor(self) -> torch.Tensor:
        return self.inner.centroids_tensor
