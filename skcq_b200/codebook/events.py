"""Event bus of the codebook build (interface of skcq/codebook/events.py).

The same event types, fields and ``Experiment.on / _emit / _forward_from``
contract as the reference, so listeners written against it (progress bars,
sweep reporters) work unchanged. The batched device engine runs all blocks
of a codebook together and emits each block's events afterwards, in block
order, with the payloads the per-block reference loop would have produced.
"""

from __future__ import annotations

from collections import defaultdict
from collections.abc import Callable
from dataclasses import dataclass
from typing import TypeVar

from tqdm import tqdm

T = TypeVar("T")


@dataclass
class KmeansStartEvent:
    """One k-means run starts (events.py:19-27)."""

    name: str
    metric: str
    k: int
    max_iters: int
    n_points: int
    block_idx: int = 0
    n_blocks: int = 1


@dataclass
class KmeansIterEvent:
    """One Lloyd iteration finished (events.py:30-35)."""

    iter: int
    max_iters: int
    moved: float
    n_empty: int


@dataclass
class KmeansDoneEvent:
    """A k-means run finished (events.py:38-42)."""

    iters_run: int
    final_moved: float
    converged: bool


@dataclass
class CodebookStartEvent:
    """A composite fit starts (events.py:50-55)."""

    n_codebooks: int
    primary_block_size: int
    primary_k: int
    metric: str


@dataclass
class CodebookIterEvent:
    """A child k-means iteration, tagged with its codebook (events.py:58-68)."""

    codebook_idx: int
    n_codebooks: int
    block_idx: int
    n_blocks: int
    iter: int
    max_iters: int
    moved: float
    n_empty: int
    metric: str


@dataclass
class CodebookDoneEvent:
    """One codebook of a composite is fitted (events.py:71-74)."""

    codebook_idx: int
    n_codebooks: int


class Experiment:
    """Listener registry: ``on(EventType, callback)``; ``_emit`` calls the
    callbacks registered for the event's exact type, in registration order."""

    def __init__(self) -> None:
        self._listeners: dict[type, list[Callable[..., None]]] = defaultdict(list)

    def on(self, event_type: type[T], callback: Callable[[T], None]) -> None:
        self._listeners[event_type].append(callback)

    def _emit(self, event: object) -> None:
        for cb in list(self._listeners.get(type(event), ())):
            cb(event)

    def _forward_from(self, child: Experiment, event_type: type[T]) -> None:
        child.on(event_type, self._emit)


class TqdmListener:
    """Progress on stderr (events.py:109-151): one bar ticking per block for
    per-block codebooks, one bar ticking per iteration for a shared codebook."""

    def __init__(self) -> None:
        self._pbar: tqdm | None = None
        self._n_blocks = 1
        self._block_mode = False

    def on_start(self, e: KmeansStartEvent) -> None:
        if e.n_blocks > 1:
            if self._pbar is not None:
                return
            self._block_mode, self._n_blocks = True, e.n_blocks
            self._pbar = tqdm(total=e.n_blocks, desc=e.name.split(" blk=")[0], leave=True)
        else:
            self._block_mode = False
            self._pbar = tqdm(total=e.max_iters, desc=e.name, leave=True)

    def on_iter(self, e: KmeansIterEvent) -> None:
        if self._pbar is not None and not self._block_mode:
            self._pbar.update(1)
            self._pbar.set_postfix(moved=f"{e.moved:.6f}", empty=e.n_empty)

    def on_done(self, e: KmeansDoneEvent) -> None:
        if self._pbar is None:
            return
        if self._block_mode:
            self._pbar.update(1)
            self._pbar.set_postfix(iters=e.iters_run, conv=int(e.converged), moved=f"{e.final_moved:.6f}")
            if self._pbar.n >= self._n_blocks:
                self._pbar.close()
                self._pbar = None
        else:
            self._pbar.close()
            self._pbar = None
