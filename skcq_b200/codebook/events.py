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
    callbacks registered for the event's exact type, in registration order.
    A callback may come with ``when``, a predicate checked at emit time (the
    forwarding and wrapping callbacks between nested experiments use it, so
    that events nobody listens to further up cost nothing); ``listens(type)``
    tells an emitter whether building an event is worth it."""

    def __init__(self) -> None:
        self._listeners: dict[type, list[tuple[Callable[..., None], Callable[[], bool] | None]]] = defaultdict(list)

    def on(self, event_type: type[T], callback: Callable[[T], None],
           when: Callable[[], bool] | None = None) -> None:
        self._listeners[event_type].append((callback, when))

    def listens(self, event_type: type) -> bool:
        return any(when is None or when() for _, when in self._listeners.get(event_type, ()))

    def _emit(self, event: object) -> None:
        for cb, when in list(self._listeners.get(type(event), ())):
            if when is None or when():
                cb(event)

    def _forward_from(self, child: Experiment, event_type: type[T]) -> None:
        child.on(event_type, self._emit, when=lambda: self.listens(event_type))


class TqdmListener:
    """Console progress of k-means fits on stderr.

    One bar per fit, measured in block-iterations: a per-block fit of
    ``n_blocks`` problems gets ``n_blocks * max_iters`` units and advances by
    each block's ``iters_run`` when it finishes (a block that converges early
    skips its remaining units); a single (shared) problem advances by one unit
    per Lloyd iteration. The postfix shows how many blocks converged, or the
    last movement and empty-cluster count of a single problem. Register
    ``on_start`` / ``on_iter`` / ``on_done`` for the three k-means events.
    """

    def __init__(self) -> None:
        self._bar: tqdm | None = None
        self._blocks_left = 0
        self._blocks_total = 0
        self._converged = 0
        self._units_per_block = 0

    def _finish(self) -> None:
        if self._bar is not None:
            self._bar.close()
        self._bar = None

    def on_start(self, e: KmeansStartEvent) -> None:
        if self._bar is not None and self._blocks_left > 0 and e.n_blocks == self._blocks_total:
            return  # the next block of the fit whose bar is open
        self._finish()
        self._blocks_total = self._blocks_left = max(e.n_blocks, 1)
        self._converged = 0
        self._units_per_block = e.max_iters
        title = e.name.partition(" blk=")[0]
        self._bar = tqdm(total=self._blocks_total * e.max_iters, desc=title, unit="blk-it", leave=True)

    def on_iter(self, e: KmeansIterEvent) -> None:
        if self._bar is None or self._blocks_total > 1:
            return
        self._bar.update(1)
        self._bar.set_postfix_str(f"moved {e.moved:.3g}, {e.n_empty} empty", refresh=False)

    def on_done(self, e: KmeansDoneEvent) -> None:
        if self._bar is None:
            return
        self._converged += int(e.converged)
        if self._blocks_total > 1:
            # unused iterations of an early-converged block are skipped over
            self._bar.update(self._units_per_block)
            self._bar.set_postfix_str(f"{self._converged}/{self._blocks_total} converged", refresh=False)
        self._blocks_left -= 1
        if self._blocks_left <= 0:
            self._finish()
