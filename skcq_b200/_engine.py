"""Device engine: batched k-means problem sets and codec kernels.

Owns the HBM layouts of the batched path and drives the C ABI
(``include/skcq_b200.h``). One *problem set* is ``nblk`` independent k-means
problems of dimension ``bs`` (one per column block of a weight matrix, or one
pooled problem for a shared codebook). All problems advance together, one
kernel per step for the whole set; a problem that converges freezes
(``active = 0``) exactly where the reference's per-block loop would stop.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass, field

import numpy as np
import torch

from skcq_b200 import _lib
from skcq_b200._lib import call, ptr, stream

COSINE = 0
L2 = 1
ROWS_PER_UNIT = 256  # SKCQ_ROWS_PER_UNIT
CENT_TILE = 128  # SKCQ_CENT_TILE


class KernelTimer:
    """Optional CUDA-event timing of engine kernels on the launching stream
    (used by the benchmark for the roofline; off by default)."""

    def __init__(self) -> None:
        self.enabled = False
        self.records: list[tuple[str, torch.cuda.Event, torch.cuda.Event, float, float, float]] = []

    def reset(self) -> None:
        self.records = []

    def run(self, name: str, fn, work: float = 0.0, padded: float = 0.0, nbytes: float = 0.0) -> None:
        if not self.enabled:
            fn()
            return
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        self.records.append((name, s, e, work, padded, nbytes))

    def summary(self) -> dict[str, dict[str, float]]:
        torch.cuda.synchronize()
        out: dict[str, dict[str, float]] = {}
        for name, s, e, work, padded, nbytes in self.records:
            d = out.setdefault(name, {"launches": 0, "ms": 0.0, "work": 0.0, "padded": 0.0, "bytes": 0.0})
            d["launches"] += 1
            d["ms"] += s.elapsed_time(e)
            d["work"] += work
            d["padded"] += padded
            d["bytes"] += nbytes
        return out


TIMER = KernelTimer()


def round_up(x: int, m: int) -> int:
    return (max(x, 1) + m - 1) // m * m


def to_device_f32(t: torch.Tensor, dev: torch.device) -> torch.Tensor:
    """``t`` as contiguous f32 on ``dev``. A host tensor is copied in its own
    dtype (without blocking the host when it is pinned) and converted on the
    device: converting a bf16 matrix on the host first costs about 14x the copy."""
    if t.device != dev:
        t = t.to(device=dev, non_blocking=t.device.type == "cpu" and t.is_pinned())
    return t.to(torch.float32).contiguous()


_STAGE_BYTES = 64 << 20


def to_host(src: torch.Tensor) -> torch.Tensor:
    """Device tensor -> pageable host tensor (what ``.cpu()`` returns), through
    two pinned staging buffers: a copy straight into pageable memory runs at a
    fraction of the bandwidth of a pinned one, and the staged chunks overlap
    the device-to-host copy of one with the host copy of the other."""
    dst = torch.empty(src.shape, dtype=src.dtype)
    n = src.numel() * src.element_size()
    if n == 0:
        return dst
    with torch.cuda.device(src.device):  # the copies and their events on the source's stream
        _stage_to_host(src, dst, n)
    return dst


def _stage_to_host(src: torch.Tensor, dst: torch.Tensor, n: int) -> None:
    s = src.contiguous().reshape(-1).view(torch.uint8)
    d = dst.reshape(-1).view(torch.uint8)
    stage = [torch.empty(min(n, _STAGE_BYTES), dtype=torch.uint8, pin_memory=True) for _ in range(2)]
    done = [torch.cuda.Event(), torch.cuda.Event()]
    prev = None
    for i, o in enumerate(range(0, n, _STAGE_BYTES)):
        e = min(n, o + _STAGE_BYTES)
        buf = stage[i % 2][: e - o]
        buf.copy_(s[o:e], non_blocking=True)  # the host copy out of this buffer two chunks ago has finished
        done[i % 2].record()
        if prev is not None:
            po, pe, pbuf, pev = prev
            pev.synchronize()
            d[po:pe].copy_(pbuf)
        prev = (o, e, buf, done[i % 2])
    po, pe, pbuf, pev = prev
    pev.synchronize()
    d[po:pe].copy_(pbuf)


def cuda_device(requested: torch.device | str | None, like: torch.Tensor) -> torch.device:
    """The CUDA device a fit runs on: the requested one, else the input's, else
    the current device. There is no CPU path."""
    dev = torch.device(requested) if requested is not None else like.device
    if dev.type == "cuda":
        return dev
    if not torch.cuda.is_available():
        raise RuntimeError("skcq_b200 needs a CUDA device (B200, sm_100a); none is available")
    return torch.device("cuda", torch.cuda.current_device())


@dataclass
class PointSet:
    """Gathered points of one problem set (layouts per include/skcq_b200.h)."""

    metric: int
    nblk: int
    bs: int
    n_pad: int
    n: torch.Tensor  # int32 [nblk]
    n_host: list[int]
    rowmap: torch.Tensor  # int32 [nblk, n_pad]
    X: torch.Tensor  # f32 [nblk, n_pad, bs]
    R: torch.Tensor  # f32 [nblk, n_pad, bs]; the same tensor as X for euclidean
    _A: torch.Tensor | None = None

    @property
    def kp(self) -> int:
        return packed_width(self.metric, self.bs)

    def packed(self) -> torch.Tensor:
        if self._A is None:
            self._A = torch.empty(self.nblk, self.n_pad * self.kp, dtype=torch.float32, device=self.X.device)
            call("skcq_pack_points", self.metric, ptr(self.X), self.nblk, self.n_pad, self.bs, ptr(self._A), stream())
        return self._A


def packed_width(metric: int, bs: int) -> int:
    return int(_lib.load().skcq_packed_width(metric, bs))


TC_MAX_KP = 64  # widest split operand the tensor-core kernel stages (bs <= 20)


# Called after every incremental assignment with (pts, B, C, cnorm, k_pad,
# k_dev, active, labels) when set; tests compare the labels with a full pass.
INCREMENTAL_CHECK: Callable | None = None

# Cost model of an assignment, in ns per point, from B200 measurements of the
# benchmark layer: a tensor-core pass costs about (0.004 + 0.000375 * kp) ns per
# point and 128-centroid tile (kp the packed width); its re-score and the merge
# over every point add about (0.06 + 0.008 * bs) ns per point; the exact
# CUDA-core scan of a moved list costs about (4e-4 + 3.5e-5 * bs) ns per point
# and centroid plus 0.02 ns per point. The model ranks the two incremental
# forms; whether an incremental pass beats a full one is decided from the
# measured times of the run's own passes (the model scaled by them).
INCREMENTAL_MAX_SHARE = 0.95
# Tests set this to take the incremental form whenever moved lists exist.
INCREMENTAL_FORCE = False
# False: every assignment is a full pass over all centroids (the reference's
# schedule, kmeans.py:136-149); same labels, more work.
INCREMENTAL = True


def _tile_ns(kp: int) -> float:
    return 0.004 + 0.000375 * kp


def plan_incremental(m: np.ndarray, p: np.ndarray, n: np.ndarray, k: np.ndarray, bs: int, kp: int, keep: float,
                     calibrated: bool, inc_ratio: float, force: bool = False
                     ) -> tuple[int, int, float, float] | None:
    """The incremental assignment of problems with m moved centroids, p points
    on moved centroids, n points and k centroids each (host arrays): (m_pad,
    p_pad, algorithmic work, model cost in ns), or None when the cost model puts
    a full pass below it. ``keep``: expected share of the p points left for a
    search over all centroids; ``calibrated``: a full pass of the run has been
    timed, so ``inc_ratio`` (measured / modelled time of the run's incremental
    passes) applies. m_pad is 0 when no problem has a moved centroid, negative
    when the moved lists are scored by the exact CUDA-core scan."""
    m, p, n, k = (np.asarray(v, dtype=np.float64) for v in (m, p, n, k))
    if m.size == 0:
        return None
    uk = np.ceil(k / CENT_TILE)
    tile = _tile_ns(kp)
    full = float((n * uk).sum()) * tile
    if full <= 0:
        return None
    tc_m = float((n * (np.ceil(m / CENT_TILE) * tile + 0.06 + 0.008 * bs) * (m > 0)).sum())
    ex_m = float((n * (m * (4e-4 + 3.5e-5 * bs) + 0.02) * (m > 0)).sum()) if bs <= 32 else np.inf
    est = min(tc_m, ex_m) + keep * float((p * uk).sum()) * tile
    if not force:
        if not calibrated:  # no full pass timed yet: the model alone
            if est >= 0.9 * full:
                return None
        elif est * inc_ratio >= INCREMENTAL_MAX_SHARE * full:
            return None
    m_pad = int(np.ceil(m.max() / CENT_TILE)) * CENT_TILE if m.max() > 0 else 0
    if ex_m < tc_m:
        m_pad = -m_pad
    p_pad = int(np.ceil(p.max() / ROWS_PER_UNIT)) * ROWS_PER_UNIT if p.max() > 0 else 0
    work = 2.0 * bs * float((n * m + p * k).sum())
    return m_pad, p_pad, work, est


class IncrementalAssign:
    """State of the exact incremental assignment of one Lloyd run
    (csrc/incremental.cu): a centroid whose cluster kept its members keeps its
    value, so a point assigned to it can only move to a centroid that moved.
    After each update the moved centroids and the points assigned to them are
    listed; the next assignment scores every point against the moved centroids
    only, re-assigns the listed points over all centroids, and merges. The
    labels are those of a full assignment."""

    def __init__(self, pts: PointSet, k_pad: int, k_host: list[int], labels: torch.Tensor) -> None:
        dev = pts.X.device
        self.pts, self.k_pad, self.labels = pts, k_pad, labels
        self.changed = torch.ones(pts.nblk, k_pad, dtype=torch.uint8, device=dev)
        self.prev = torch.empty_like(labels)
        self.mlist = torch.zeros(pts.nblk, k_pad, dtype=torch.int32, device=dev)
        self.plist = torch.zeros(pts.nblk, pts.n_pad, dtype=torch.int32, device=dev)
        self.counts = torch.zeros(2, pts.nblk, dtype=torch.int32, device=dev)  # moved centroids, listed points
        self.counts_host = torch.zeros(2, pts.nblk, dtype=torch.int32, pin_memory=True)
        self.scratch_bytes = int(_lib.load().skcq_moved_lists_scratch_bytes(pts.nblk, pts.n_pad, k_pad))
        self.scratch = torch.empty(max(self.scratch_bytes, 1), dtype=torch.uint8, device=dev)
        self.units_n = np.ceil(np.array(pts.n_host, dtype=np.float64) / ROWS_PER_UNIT)
        self.units_k = np.ceil(np.array(k_host, dtype=np.float64) / CENT_TILE)
        self.k_host = np.array(k_host, dtype=np.float64)
        self.n_host = np.array(pts.n_host, dtype=np.float64)
        self.listed = False
        self.C_old = torch.empty(pts.nblk, k_pad, pts.bs, dtype=torch.float32, device=dev)
        self.cnorm_old = torch.empty(pts.nblk, k_pad, dtype=torch.float32, device=dev)
        self.have_old = False
        self.unres = torch.zeros(pts.nblk, pts.n_pad, dtype=torch.uint8, device=dev)
        self.ulist = torch.zeros(pts.nblk, pts.n_pad, dtype=torch.int32, device=dev)
        self.ucount = torch.zeros(pts.nblk, dtype=torch.int32, device=dev)
        self.ucount_host = torch.zeros(pts.nblk, dtype=torch.int32, pin_memory=True)
        self.unres_rate = 0.5  # share of the points whose centroid moved left for a full search
        self.resolved_pending: torch.Tensor | None = None
        self.counts_prev = np.zeros(pts.nblk)
        self.ms_per_ns: float | None = None  # device ms per model ns (from full passes)
        self.inc_ratio = 1.0  # measured / predicted time of incremental passes
        self.pending = None

    def mark(self, first: bool, mask: torch.Tensor) -> None:
        """Clusters whose members changed in this iteration's assignment."""
        pts = self.pts
        call("skcq_mark_changed", ptr(self.prev), ptr(self.labels), pts.nblk, pts.n_pad, self.k_pad, ptr(pts.n),
             ptr(mask), int(first), ptr(self.changed), stream())

    def lists(self, mask: torch.Tensor, k_dev: torch.Tensor) -> None:
        """After the update: moved centroids and the points assigned to them
        (rows of the problems in ``mask``), counts copied to the host."""
        pts = self.pts
        call("skcq_moved_lists", ptr(self.changed), ptr(self.labels), pts.nblk, pts.n_pad, self.k_pad, ptr(pts.n),
             ptr(k_dev), ptr(mask), ptr(self.mlist), ptr(self.counts[0]), ptr(self.plist), ptr(self.counts[1]),
             ptr(self.scratch), self.scratch_bytes, stream())
        self.counts_host.copy_(self.counts, non_blocking=True)
        self.listed = True

    def full_estimate(self, act: np.ndarray) -> float:
        """Model cost (ns) of a full pass over the problems in ``act``."""
        return float((self.n_host * self.units_k)[act].sum()) * _tile_ns(self.pts.kp)

    def plan(self, act: np.ndarray, force: bool = False) -> tuple[int, int, float, float] | None:
        """(m_pad, p_pad, algorithmic work, model cost in ns) of an incremental
        assignment of the problems in ``act`` (host bool mask), or None when a
        full pass is expected to be faster (``force``: whenever lists exist).
        Reads the counts of the last ``lists`` (the caller synchronised)."""
        if not self.listed or not act.any():
            return None
        return plan_incremental(
            self.counts_host[0].numpy()[act], self.counts_host[1].numpy()[act], self.n_host[act],
            self.k_host[act], self.pts.bs, self.pts.kp, self.unres_rate if self.have_old else 1.0,
            self.ms_per_ns is not None, self.inc_ratio, force)

    def timed(self, kind: str, est: float, fn) -> None:
        """Run one assignment between CUDA events; ``observe`` reads them after
        the iteration's synchronisation."""
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        self.pending = (kind, est, a, b)

    def observe(self) -> None:
        """Update the run's calibration from the last timed assignment: device
        ms per model ns from full passes, the measured / predicted ratio of
        incremental passes, and the share of moved-centroid points that needed
        a full search."""
        if self.resolved_pending is not None:
            act = self.resolved_pending.bool().cpu().numpy()
            self.resolved_pending = None
            flagged = float(self.counts_prev[act].sum())
            if flagged > 0:
                self.unres_rate = 0.5 * self.unres_rate + 0.5 * float(self.ucount_host.numpy()[act].sum()) / flagged
        if self.pending is None:
            return
        kind, est, a, b = self.pending
        self.pending = None
        ms = a.elapsed_time(b)
        if est <= 0:
            return
        if kind == "full":
            self.ms_per_ns = ms / est
        elif kind == "inc" and self.ms_per_ns is not None:
            r = ms / (est * self.ms_per_ns)
            self.inc_ratio = 0.5 * self.inc_ratio + 0.5 * r

    def first_from_seeds(self, C: torch.Tensor, perm: torch.Tensor, k_dev: torch.Tensor,
                         gofs: torch.Tensor | None = None) -> tuple[int, float]:
        """First assignment of a Forgy start (euclidean centroids are points
        X[perm[c]]): a seed point's own centroid is at distance 0, so it is the
        point's nearest centroid unless another centroid lies within rounding of
        it (a tie below the reference's rounding) or has the identical value (an
        exact tie, which the first index wins). Seeds whose value occurs once get
        their own index; every other point (and every seed with a duplicate,
        detected by hashing the centroid bits) is listed for a search over all
        centroids. Row-sharded: ``perm`` holds global point indices and this
        rank's points start at global index ``gofs[b]``; a rank takes the seeds
        it owns. Returns (p_pad, algorithmic work) for ``assign`` with no moved
        centroids."""
        pts, dev = self.pts, self.pts.X.device
        nblk, k_pad = pts.nblk, self.k_pad
        c_idx = torch.arange(k_pad, device=dev)
        # equal centroid values have equal keys; different values sharing a
        # key only send more seeds to the full search
        valid = c_idx[None, :] < k_dev[:, None].long()
        bits = (C + 0.0).view(torch.int32).long() & 0xFFFFFFFF  # -0 and +0 alike
        mult = torch.tensor([0x9E3779B97F4A7C15 - (1 << 64), 0xC2B2AE3D27D4EB4F - (1 << 64),
                             0x165667B19E3779F9, 0x27D4EB2F165667C5] * ((pts.bs + 3) // 4),
                            dtype=torch.int64, device=dev)[:pts.bs]
        h = (bits * mult).sum(-1)  # wraps modulo 2^64
        h = torch.where(valid, h, -(c_idx[None, :].long() + 1) * 0x100000001)  # padding: distinct keys
        hs, order = torch.sort(h, dim=1)
        eq = hs[:, 1:] == hs[:, :-1]
        dup_sorted = torch.zeros_like(hs, dtype=torch.bool)
        dup_sorted[:, 1:] |= eq
        dup_sorted[:, :-1] |= eq
        dup = torch.zeros_like(dup_sorted).scatter_(1, order, dup_sorted)
        own = valid & ~dup  # seeds that take their own index
        local = perm[:, :k_pad]
        if gofs is not None:  # this rank's own points among the seeds
            local = local - gofs.to(dev)[:, None].long()
            own &= (local >= 0) & (local < pts.n[:, None].long())
        b_idx = torch.arange(nblk, device=dev)[:, None].expand(-1, k_pad)[own]
        p_idx = local[own]
        self.labels[b_idx, p_idx] = c_idx[None, :].expand(nblk, -1)[own].to(torch.int32)
        covered = torch.zeros(nblk, pts.n_pad, dtype=torch.bool, device=dev)
        covered[b_idx, p_idx] = True
        need = (torch.arange(pts.n_pad, device=dev)[None, :] < pts.n[:, None].long()) & ~covered
        self.plist.copy_(torch.argsort((~need).to(torch.int8), dim=1, stable=True).to(torch.int32))
        self.counts[0].zero_()
        self.counts[1].copy_(need.sum(1).to(torch.int32))
        p_host = self.counts[1].cpu().numpy().astype(np.float64)
        p_pad = int(np.ceil(p_host.max() / ROWS_PER_UNIT)) * ROWS_PER_UNIT if p_host.max() > 0 else 0
        return p_pad, 2.0 * pts.bs * float((p_host * self.k_host).sum())

    def save_old(self, C: torch.Tensor, cnorm: torch.Tensor, active: torch.Tensor) -> None:
        """Keep the centroids and norms the iteration's assignment used (before
        the update) for the problems that ran it: a moved centroid's previous
        score bounds the unmoved ones'. Converged problems keep the values of
        their last assignment."""
        m = active.bool()
        self.C_old.copy_(torch.where(m[:, None, None], C, self.C_old))
        self.cnorm_old.copy_(torch.where(m[:, None], cnorm, self.cnorm_old))
        self.have_old = True

    def _full_search(self, B, C, cnorm, k_dev, act, plist, pcount, p_pad: int) -> torch.Tensor:
        """Labels of the listed points against all centroids ([nblk][p_pad])."""
        pts, dev, s = self.pts, self.pts.X.device, stream()
        Xf = torch.empty(pts.nblk, p_pad, pts.bs, dtype=torch.float32, device=dev)
        call("skcq_gather_rows", ptr(pts.X), pts.n_pad, ptr(plist), pts.n_pad, ptr(pcount), pts.nblk, p_pad, pts.bs,
             ptr(Xf), s)
        sub = PointSet(pts.metric, pts.nblk, pts.bs, p_pad, pcount, [], plist, Xf, Xf)
        act_f = (act.bool() & (pcount > 0)).to(torch.int32)
        labels_f = torch.zeros(pts.nblk, p_pad, dtype=torch.int32, device=dev)
        assign_call(sub, B, C, cnorm, self.k_pad, k_dev, act_f, labels_f)
        return labels_f

    def assign(self, B, C, cnorm, k_dev, active, m_pad: int, p_pad: int) -> None:
        """Labels of the problems in ``active`` (None: all) from the previous
        labels, in place. With the previous centroids saved, a point whose
        centroid moved keeps to the moved centroids when the best of them beats
        its previous score, and only the rest are searched over all centroids."""
        pts, dev, s = self.pts, self.pts.X.device, stream()
        act = active if active is not None else torch.ones(pts.nblk, dtype=torch.int32, device=dev)
        mcount, pcount = self.counts[0], self.counts[1]
        self.counts_prev = self.counts_host[1].numpy().astype(np.float64).copy()
        zeros = torch.zeros_like(mcount)
        resolve = self.have_old and m_pad != 0
        unres = self.unres if resolve else None
        old = (ptr(self.C_old), ptr(self.cnorm_old)) if resolve else (None, None)
        labels_m = torch.zeros(1, dtype=torch.int32, device=dev)
        merge_m = mcount
        if m_pad < 0:  # short moved lists: exact scores on CUDA cores, merged in place
            call("skcq_assign_moved_exact", pts.metric, ptr(pts.X), ptr(C), ptr(cnorm), pts.nblk, pts.n_pad,
                 self.k_pad, pts.bs, ptr(pts.n), ptr(active), ptr(self.changed), ptr(self.mlist), ptr(mcount),
                 ptr(self.labels), old[0], old[1], ptr(unres), s)
            merge_m = zeros
        elif m_pad > 0:  # every point against the moved centroids
            Cm = torch.empty(pts.nblk, m_pad, pts.bs, dtype=torch.float32, device=dev)
            call("skcq_gather_rows", ptr(C), self.k_pad, ptr(self.mlist), self.k_pad, ptr(mcount), pts.nblk, m_pad,
                 pts.bs, ptr(Cm), s)
            act_m = (act.bool() & (mcount > 0)).to(torch.int32)
            Bm = torch.empty(pts.nblk, m_pad * pts.kp, dtype=torch.float32, device=dev)
            cnm = torch.empty(pts.nblk, m_pad, dtype=torch.float32, device=dev)
            call("skcq_pack_centroids", pts.metric, ptr(Cm), pts.nblk, m_pad, pts.bs, ptr(mcount), ptr(act_m),
                 ptr(Bm), ptr(cnm), s)
            if pts.metric == L2 and resolve:
                # only the points that can move: a point exactly on its unmoved
                # centroid cannot be beaten (label -1 below: not scored)
                labels_m = torch.full((pts.nblk, pts.n_pad), -1, dtype=torch.int32, device=dev)
                call("skcq_mpass_points", ptr(pts.X), ptr(C), ptr(self.labels), ptr(self.changed), ptr(pts.n),
                     ptr(act_m), pts.nblk, pts.n_pad, self.k_pad, pts.bs, ptr(self.unres), s)
                call("skcq_list_points", ptr(self.unres), pts.nblk, pts.n_pad, ptr(pts.n), ptr(act_m),
                     ptr(self.ulist), ptr(self.ucount), ptr(self.scratch), self.scratch_bytes, s)
                self.ucount_host.copy_(self.ucount, non_blocking=True)
                torch.cuda.current_stream().synchronize()
                c_max = int(self.ucount_host.numpy()[act_m.bool().cpu().numpy()].max(initial=0))
                s_pad = int(np.ceil(c_max / ROWS_PER_UNIT)) * ROWS_PER_UNIT
                if s_pad > 0:
                    Xs = torch.empty(pts.nblk, s_pad, pts.bs, dtype=torch.float32, device=dev)
                    call("skcq_gather_rows", ptr(pts.X), pts.n_pad, ptr(self.ulist), pts.n_pad, ptr(self.ucount),
                         pts.nblk, s_pad, pts.bs, ptr(Xs), s)
                    sub = PointSet(pts.metric, pts.nblk, pts.bs, s_pad, self.ucount, [], self.ulist, Xs, Xs)
                    labels_s = torch.zeros(pts.nblk, s_pad, dtype=torch.int32, device=dev)
                    assign_call(sub, Bm, Cm, cnm, m_pad, mcount, (act_m.bool() & (self.ucount > 0)).to(torch.int32),
                                labels_s)
                    call("skcq_scatter_sub", ptr(self.ulist), ptr(self.ucount), ptr(labels_s), pts.nblk, s_pad,
                         pts.n_pad, ptr(labels_m), s)
            else:
                labels_m = torch.zeros(pts.nblk, pts.n_pad, dtype=torch.int32, device=dev)
                assign_call(pts, Bm, Cm, cnm, m_pad, mcount, act_m, labels_m)
        if resolve:
            # phase 0 (the moved centroids) for every point, then a full search
            # for the points it left unresolved
            if m_pad > 0:
                call("skcq_assign_merge", pts.metric, ptr(pts.X), ptr(C), ptr(cnorm), pts.nblk, pts.n_pad,
                     self.k_pad, pts.bs, ptr(pts.n), ptr(active), ptr(self.changed), ptr(self.mlist), ptr(merge_m),
                     ptr(labels_m), ptr(self.ulist), ptr(zeros), 0, None, ptr(self.labels), old[0], old[1],
                     ptr(unres), s)
            call("skcq_list_points", ptr(unres), pts.nblk, pts.n_pad, ptr(pts.n), ptr(act), ptr(self.ulist),
                 ptr(self.ucount), ptr(self.scratch), self.scratch_bytes, s)
            # the unresolved points are a subset of the listed ones, so the
            # listed count pads their search without a host round trip (the
            # tensor-core pass skips units past each problem's count)
            if p_pad > 0:
                labels_f = self._full_search(B, C, cnorm, k_dev, act, self.ulist, self.ucount, p_pad)
                call("skcq_assign_merge", pts.metric, ptr(pts.X), ptr(C), ptr(cnorm), pts.nblk, pts.n_pad,
                     self.k_pad, pts.bs, ptr(pts.n), ptr(active), ptr(self.changed), ptr(self.mlist), ptr(zeros),
                     ptr(labels_m), ptr(self.ulist), ptr(self.ucount), p_pad, ptr(labels_f), ptr(self.labels),
                     None, None, None, s)
            self.ucount_host.copy_(self.ucount, non_blocking=True)
            self.resolved_pending = act
        else:
            labels_f = self._full_search(B, C, cnorm, k_dev, act, self.plist, pcount, p_pad) if p_pad > 0 else None
            call("skcq_assign_merge", pts.metric, ptr(pts.X), ptr(C), ptr(cnorm), pts.nblk, pts.n_pad, self.k_pad,
                 pts.bs, ptr(pts.n), ptr(active), ptr(self.changed), ptr(self.mlist), ptr(merge_m), ptr(labels_m),
                 ptr(self.plist), ptr(pcount), p_pad, ptr(labels_f), ptr(self.labels), None, None, None, s)
        if INCREMENTAL_CHECK is not None:
            INCREMENTAL_CHECK(pts, B, C, cnorm, self.k_pad, k_dev, active, self.labels)


# Euclidean problems of block size 2-4 with at least this many centroids are
# searched through the centroid grid (csrc/assign_grid.cu); the points it
# cannot certify go to the tensor-core pass. False: always the tensor-core pass.
GRID = True
GRID_MIN_K = 8192
# Largest box radius (cells) of the grid's second search of uncertified points
# (0: they go straight to the tensor-core pass).
GRID_RING = 3


def grid_cells(bs: int, k: int) -> int:
    """Grid cells per coordinate for k centroids in bs dimensions: about one
    centroid per cell, within the kernel's limits."""
    g = int(round(k ** (1.0 / bs)))
    cap = {2: 256, 3: 100, 4: 31}[bs]
    return max(2, min(g, cap))


def _grid_assign(pts: PointSet, B, C, cnorm, k_pad: int, k_dev, active, labels) -> None:
    """Labels through the centroid grid; uncertified points (rare: a point whose
    nearest centroid lies beyond its cell neighbourhood) are gathered and
    searched over all centroids on the tensor cores, then scattered back.
    With the timer on, the call is recorded as "assign_grid" (inside the
    caller's "assign" record) with the work of the full pass it replaces, so
    the tensor-core figures can leave it out."""
    T = TIMER
    if not T.enabled:
        _grid_assign_run(pts, B, C, cnorm, k_pad, k_dev, active, labels)
        return
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    _grid_assign_run(pts, B, C, cnorm, k_pad, k_dev, active, labels)
    b.record()
    act = (active.bool() if active is not None else torch.ones(pts.nblk, dtype=torch.bool, device=pts.X.device))
    act_h = act.cpu().numpy()
    pairs = float((pts.n.cpu().numpy().astype(np.float64) * k_dev.cpu().numpy())[act_h].sum())
    work = 2.0 * pts.bs * pairs
    T.records.append(("assign_grid", a, b, work, work * pts.kp / pts.bs,
                      4.0 * pts.kp * float(act_h.sum()) * (pts.n_pad + k_pad)))


def _grid_assign_run(pts: PointSet, B, C, cnorm, k_pad: int, k_dev, active, labels) -> None:
    dev, s = pts.X.device, stream()
    lib = _lib.load()
    G = grid_cells(pts.bs, k_pad)
    nbytes = int(lib.skcq_assign_grid_scratch_bytes(pts.nblk, pts.n_pad, k_pad, pts.bs, G))
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    unres = torch.zeros(pts.nblk, pts.n_pad, dtype=torch.uint8, device=dev)
    act = active if active is not None else torch.ones(pts.nblk, dtype=torch.int32, device=dev)
    call("skcq_assign_grid", ptr(pts.X), ptr(C), ptr(cnorm), pts.nblk, pts.n_pad, k_pad, pts.bs, ptr(pts.n),
         ptr(k_dev), ptr(act), G, GRID_RING, ptr(labels), ptr(unres), ptr(scratch), nbytes, s)
    ulist = torch.empty(pts.nblk, pts.n_pad, dtype=torch.int32, device=dev)
    ucount = torch.zeros(pts.nblk, dtype=torch.int32, device=dev)
    lbytes = 4 * pts.nblk * -(-pts.n_pad // 4096)
    lscr = torch.empty(max(lbytes, 1), dtype=torch.uint8, device=dev)
    call("skcq_list_points", ptr(unres), pts.nblk, pts.n_pad, ptr(pts.n), ptr(act), ptr(ulist), ptr(ucount),
         ptr(lscr), lbytes, s)
    GRID_STATS["points"] += float(pts.n[act.bool()].sum()) if GRID_STATS["enabled"] else 0.0
    c_max = int(ucount.max())
    if GRID_STATS["enabled"]:
        GRID_STATS["fallback"] += float(ucount.sum())
    if c_max == 0:
        return
    s_pad = round_up(c_max, ROWS_PER_UNIT)
    Xs = torch.empty(pts.nblk, s_pad, pts.bs, dtype=torch.float32, device=dev)
    call("skcq_gather_rows", ptr(pts.X), pts.n_pad, ptr(ulist), pts.n_pad, ptr(ucount), pts.nblk, s_pad, pts.bs,
         ptr(Xs), s)
    sub = PointSet(pts.metric, pts.nblk, pts.bs, s_pad, ucount, [], ulist, Xs, Xs)
    labels_s = torch.zeros(pts.nblk, s_pad, dtype=torch.int32, device=dev)
    _scan_call(sub, B, C, cnorm, k_pad, k_dev, (act.bool() & (ucount > 0)).to(torch.int32), labels_s)
    call("skcq_scatter_sub", ptr(ulist), ptr(ucount), ptr(labels_s), pts.nblk, s_pad, pts.n_pad, ptr(labels), s)


# Counts of grid-searched points and of those sent to the full search (tests
# and the kernel bench enable it).
GRID_STATS = {"enabled": False, "points": 0.0, "fallback": 0.0}


def assign_call(pts: PointSet, B, C, cnorm, k_pad: int, k_dev, active, labels) -> None:
    """Labels against all k_dev[b] centroids: the centroid grid for
    low-dimensional euclidean problems with many centroids, else the
    tensor-core pass (+ exact re-score)."""
    if GRID and pts.metric == L2 and 2 <= pts.bs <= 4 and k_pad >= GRID_MIN_K:
        _grid_assign(pts, B, C, cnorm, k_pad, k_dev, active, labels)
    else:
        _scan_call(pts, B, C, cnorm, k_pad, k_dev, active, labels)


def _scan_call(pts: PointSet, B, C, cnorm, k_pad: int, k_dev, active, labels) -> None:
    """Tensor-core assignment (+ exact re-score); blocks wider than the
    tensor-core path stages go to the exact CUDA-core kernel."""
    if pts.kp <= TC_MAX_KP:
        call("skcq_assign", pts.metric, ptr(pts.packed()), ptr(B), ptr(pts.X), ptr(C), ptr(cnorm), pts.nblk,
             pts.n_pad, k_pad, pts.bs, ptr(pts.n), ptr(k_dev), ptr(active), ptr(labels), stream())
    else:
        call("skcq_assign_exact", pts.metric, ptr(pts.X), ptr(C), ptr(cnorm), pts.nblk, pts.n_pad, k_pad, pts.bs,
             ptr(pts.n), ptr(k_dev), ptr(active), ptr(labels), stream())


def gather_block_points(
    w: torch.Tensor, bs: int, n_blocks: int, shared: bool, thr: float, skip_zeros: bool, metric: int
) -> PointSet:
    """Block zero test + compaction + gather (spherical.py:243-248, euclidean.py:455-460)."""
    assert w.dtype == torch.float32 and w.is_cuda and w.stride(1) == 1
    n_rows = w.shape[0]
    nblk = 1 if shared else n_blocks
    npts = n_rows * n_blocks if shared else n_rows
    n_pad = round_up(npts, ROWS_PER_UNIT)
    dev = w.device
    rowmap = torch.empty(nblk, n_pad, dtype=torch.int32, device=dev)
    n = torch.empty(nblk, dtype=torch.int32, device=dev)
    s = stream()
    call("skcq_compact_points", ptr(w), w.stride(0), n_rows, bs, n_blocks, int(shared), float(thr),
         int(skip_zeros), nblk, n_pad, ptr(rowmap), ptr(n), s)
    return _gather(w, bs, n_blocks, shared, metric, rowmap, n, n_pad)


def _gather(w, bs, n_blocks, shared, metric, rowmap, n, n_pad) -> PointSet:
    nblk = rowmap.shape[0]
    dev = w.device
    X = torch.empty(nblk, n_pad, bs, dtype=torch.float32, device=dev)
    R = torch.empty_like(X) if metric == COSINE else None
    call("skcq_gather_points", ptr(w), w.stride(0), bs, n_blocks, int(shared), nblk, ptr(rowmap), ptr(n), n_pad,
         int(metric == COSINE), ptr(X), ptr(R), stream())
    n_host = [int(v) for v in n.cpu().tolist()]
    return PointSet(metric, nblk, bs, n_pad, n, n_host, rowmap, X, R if R is not None else X)


def subsample_points(w, bs, n_blocks, shared, pts: PointSet, perms: list[torch.Tensor | None], m: int) -> PointSet:
    """Training subset ``non_zero[perm[:m]]`` per problem (spherical.py:263-268)."""
    n_train = [min(nb, m) if p is not None else nb for nb, p in zip(pts.n_host, perms, strict=True)]
    n_pad = round_up(max(n_train), ROWS_PER_UNIT)
    rm = torch.zeros(pts.nblk, n_pad, dtype=torch.int32, device=w.device)
    for b, p in enumerate(perms):
        if p is None:
            rm[b, : pts.n_host[b]] = pts.rowmap[b, : pts.n_host[b]]
        else:
            rm[b, : n_train[b]] = pts.rowmap[b][p[:m].to(w.device)]
    n = torch.tensor(n_train, dtype=torch.int32, device=w.device)
    return _gather(w, bs, n_blocks, shared, pts.metric, rm, n, n_pad)


@dataclass
class KmeansRun:
    """Result of one batched Lloyd run (skcq/codebook/kmeans.py:109-249)."""

    C: torch.Tensor  # f32 [nblk, k_pad, bs]
    k_pad: int
    k_host: list[int]
    labels: torch.Tensor  # int32 [nblk, n_pad] of the final assignment
    iters_run: list[int]
    converged: list[bool]
    moved: np.ndarray  # [max_iters, nblk]
    n_empty: np.ndarray  # [max_iters, nblk]
    cnorm: torch.Tensor = field(repr=False, default=None)

    def final_moved(self, b: int) -> float:
        it = self.iters_run[b]
        return float(self.moved[it - 1, b]) if it > 0 else 0.0


def lloyd(
    pts: PointSet,
    K: int,
    max_iters: int,
    init_cosine: Callable[[int, int], torch.Tensor] | None = None,
    init_perms: list[torch.Tensor | None] | None = None,
    shard=None,
    n_global: torch.Tensor | None = None,
    gofs: torch.Tensor | None = None,
) -> KmeansRun:
    """Run every problem of ``pts`` to convergence or ``max_iters``.

    Cosine problems start from ``init_cosine(k_eff, bs)`` (the Sobol directions
    of kmeans.py:69-74); euclidean problems from ``X[b][init_perms[b][:k_eff]]``
    (kmeans.py:201-202). Problems with no points are left inactive.

    With ``shard`` (a ``distributed.RowShard``), ``pts`` holds this rank's
    slice of every problem: ``n_global`` points in all, this rank's first at
    global index ``gofs``; sums and counts are summed over ranks each
    iteration and the reseed merges every rank's candidates.
    """
    dev = pts.X.device
    nblk, bs, n_pad, metric = pts.nblk, pts.bs, pts.n_pad, pts.metric
    forgy = False
    n_all = [int(v) for v in n_global.tolist()] if shard is not None else pts.n_host
    k_host = [min(K, nb) for nb in n_all]
    k_pad = round_up(max(k_host + [1]), CENT_TILE)
    kp = pts.kp
    s = stream()
    k_dev = torch.tensor(k_host, dtype=torch.int32, device=dev)
    active = (torch.tensor(n_all, device=dev) > 0).to(torch.int32)
    C = torch.zeros(nblk, k_pad, bs, dtype=torch.float32, device=dev)
    if metric == COSINE:
        cache: dict[int, torch.Tensor] = {}
        for b, kb in enumerate(k_host):
            if kb > 0:
                if kb not in cache:
                    cache[kb] = init_cosine(kb, bs).to(device=dev, dtype=torch.float32)
                C[b, :kb] = cache[kb]
    else:
        perm = torch.zeros(nblk, k_pad, dtype=torch.int64, device=dev)
        forgy = True
        for b, kb in enumerate(k_host):
            if kb > 0:
                perm[b, :kb] = init_perms[b][:kb].to(dev)
        if shard is None:
            call("skcq_init_from_points", ptr(pts.X), n_pad, bs, nblk, ptr(perm), k_pad, ptr(k_dev), k_pad, ptr(C),
                 s)
        else:
            from skcq_b200 import distributed

            C.copy_(distributed.owned_init(pts.X, perm, k_dev, gofs.to(dev), pts.n))
            shard.all_reduce_sum_(C)
    B = torch.empty(nblk, k_pad * kp, dtype=torch.float32, device=dev)
    cnorm = torch.empty(nblk, k_pad, dtype=torch.float32, device=dev)
    sums = torch.zeros(nblk, k_pad, bs, dtype=torch.float32, device=dev)
    counts = torch.zeros(nblk, k_pad, dtype=torch.int32, device=dev)
    labels = torch.zeros(nblk, n_pad, dtype=torch.int32, device=dev)
    n_empty = torch.zeros(nblk, dtype=torch.int32, device=dev)
    scratch = torch.empty(int(_lib.load().skcq_reseed_scratch_bytes(nblk, k_pad)), dtype=torch.uint8, device=dev)
    converged = torch.zeros(nblk, dtype=torch.int32, device=dev)
    iters_run = torch.zeros(nblk, dtype=torch.int32, device=dev)
    moved = torch.zeros(max(max_iters, 1), nblk, dtype=torch.float32, device=dev)
    nempty_hist = torch.zeros(max(max_iters, 1), nblk, dtype=torch.int32, device=dev)
    act_host = torch.empty(nblk, dtype=torch.int32, pin_memory=True)
    T = TIMER
    nk = np.array(pts.n_host, dtype=np.float64) * np.array(k_host, dtype=np.float64)
    # exact incremental assignment after the first iteration (row-sharded
    # problems too: the change marks are OR-ed over the ranks, so every rank
    # keeps the same centroids and lists the same moved ones)
    inc = IncrementalAssign(pts, k_pad, k_host, labels) if INCREMENTAL else None
    act = (np.array(n_all) > 0)
    def prepare() -> None:
        """The next assignment's device work that needs no host decision:
        packing the centroids and keeping the labels it starts from. Queued
        before the iteration's synchronisation, so the GPU has it to run while
        the host plans."""
        T.run("pack_centroids", lambda: call("skcq_pack_centroids", metric, ptr(C), nblk, k_pad, bs, ptr(k_dev),
                                             ptr(active), ptr(B), ptr(cnorm), s))
        if inc is not None:
            inc.prev.copy_(labels)

    if max_iters > 0:
        prepare()
    for it in range(max_iters):
        plan = inc.plan(act, force=INCREMENTAL_FORCE) if inc is not None else None
        # the seed shortcut pays when seeds are a large share of the points
        # (K = 65536 over 98,304 points: two thirds); with few seeds, gathering
        # the rest costs more than it saves
        if it == 0 and inc is not None and forgy and sum(k_host) >= 0.25 * max(sum(n_all), 1):
            p_pad, work = inc.first_from_seeds(C, perm, k_dev, gofs if shard is not None else None)
            nbytes = 4.0 * kp * float(act.sum()) * (p_pad + k_pad)
            T.run("assign", lambda: inc.assign(B, C, cnorm, k_dev, active, 0, p_pad), work, work * kp / bs, nbytes)
        elif plan is None:
            # algorithmic work: 2*n*k*bs flops over the active problems
            work = 2.0 * bs * float(nk[act].sum())
            # the split operands each active problem's tensor-core pass reads once
            nbytes = 4.0 * kp * float(act.sum()) * (n_pad + k_pad)
            full_pass = lambda: assign_call(pts, B, C, cnorm, k_pad, k_dev, active, labels)  # noqa: E731
            if inc is not None:
                est = inc.full_estimate(act)
                T.run("assign", lambda: inc.timed("full", est, full_pass), work, work * kp / bs, nbytes)
            else:
                T.run("assign", full_pass, work, work * kp / bs, nbytes)
        else:
            m_pad, p_pad, work, est = plan
            nbytes = 4.0 * kp * float(act.sum()) * (n_pad + abs(m_pad) + p_pad + k_pad)
            T.run("assign", lambda: inc.timed("inc", est, lambda: inc.assign(B, C, cnorm, k_dev, active, m_pad,
                                                                             p_pad)), work, work * kp / bs, nbytes)
        if inc is not None:
            inc.mark(it == 0, active)
            if shard is not None:
                shard.all_reduce_max_(inc.changed)
        T.run("update", lambda: call("skcq_update", ptr(pts.R), ptr(labels), nblk, n_pad, k_pad, bs, ptr(pts.n),
                                     ptr(k_dev), ptr(active), ptr(sums), ptr(counts),
                                     ptr(inc.changed) if inc is not None else None, s))
        if shard is None:
            T.run("reseed", lambda: call("skcq_reseed", metric, ptr(pts.X), ptr(C), ptr(labels), nblk, n_pad, k_pad,
                                         bs, ptr(pts.n), ptr(k_dev), ptr(active), ptr(sums), ptr(counts),
                                         ptr(n_empty), ptr(scratch), s))
        else:
            _sharded_reseed(shard, pts, C, labels, k_pad, k_dev, active, sums, counts, n_empty, scratch, gofs)
        ran = active.clone() if inc is not None else None
        if inc is not None:
            inc.save_old(C, cnorm, active)
        T.run("finalize", lambda: call("skcq_finalize", metric, ptr(sums), ptr(counts), ptr(n_empty), nblk, k_pad,
                                       bs, ptr(k_dev), ptr(active), ptr(converged), ptr(iters_run), ptr(moved),
                                       ptr(nempty_hist), it, ptr(C), ptr(inc.changed) if inc else None, s))
        if inc is not None:
            T.run("moved_lists", lambda: inc.lists(ran, k_dev))
        act_host.copy_(active, non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        if it + 1 < max_iters:
            prepare()
        done.synchronize()  # the iteration's results, not the queued preparation
        if inc is not None:
            inc.observe()
        act = act_host.numpy().astype(bool)
        if not act.any():
            break
    _lib.poll_device_error()
    # final assignment with the final centroids (kmeans.py:190 / 246)
    call("skcq_pack_centroids", metric, ptr(C), nblk, k_pad, bs, ptr(k_dev), None, ptr(B), ptr(cnorm), s)
    every = np.array(n_all) > 0
    plan = inc.plan(every, force=INCREMENTAL_FORCE) if inc is not None and max_iters > 0 else None
    if plan is None:
        work = 2.0 * bs * float(nk.sum())
        T.run("assign", lambda: assign_call(pts, B, C, cnorm, k_pad, k_dev, None, labels), work, work * kp / bs,
              4.0 * kp * nblk * (n_pad + k_pad))
    else:
        m_pad, p_pad, work, _ = plan
        T.run("assign", lambda: inc.assign(B, C, cnorm, k_dev, None, m_pad, p_pad), work, work * kp / bs,
              4.0 * kp * nblk * (n_pad + abs(m_pad) + p_pad + k_pad))
    return KmeansRun(
        C=C, k_pad=k_pad, k_host=k_host, labels=labels,
        iters_run=[int(v) for v in iters_run.cpu().tolist()],
        converged=[bool(v) for v in converged.cpu().tolist()],
        moved=moved.cpu().numpy(), n_empty=nempty_hist.cpu().numpy(), cnorm=cnorm,
    )


def _sharded_reseed(shard, pts: PointSet, C, labels, k_pad, k_dev, active, sums, counts, n_empty, scratch,
                    gofs) -> None:
    """Sum sums/counts over ranks, then reseed empty clusters from the merged
    worst-fit candidates of all ranks (same choice as skcq_reseed on the
    unsharded problem)."""
    from skcq_b200 import distributed

    shard.all_reduce_sum_(sums)
    shard.all_reduce_sum_(counts)
    empty = distributed.empty_clusters(counts, k_dev, active)
    ne = empty.sum(1)
    n_empty.copy_(ne.to(torch.int32))
    m_max = int(ne.max().item()) if ne.numel() else 0
    if m_max == 0:
        return
    dev = pts.X.device
    keys = torch.full((pts.nblk, m_max), distributed.INT64_MAX, dtype=torch.int64, device=dev)
    vecs = torch.zeros(pts.nblk, m_max, pts.bs, dtype=torch.float32, device=dev)
    call("skcq_reseed_candidates", pts.metric, ptr(pts.X), ptr(C), ptr(labels), pts.nblk, pts.n_pad, k_pad, pts.bs,
         ptr(pts.n), ptr(k_dev), ptr(active), ptr(counts), ptr(gofs.to(dev)), m_max, ptr(keys), ptr(vecs),
         ptr(n_empty), ptr(scratch), stream())
    distributed.merge_reseed(shard.all_gather(keys), shard.all_gather(vecs), empty, sums)


def assign(pts: PointSet, run: KmeansRun) -> torch.Tensor:
    """Labels of ``pts`` against the (already packed) centroids of ``run``."""
    dev = pts.X.device
    B = torch.empty(pts.nblk, run.k_pad * pts.kp, dtype=torch.float32, device=dev)
    k_dev = torch.tensor(run.k_host, dtype=torch.int32, device=dev)
    labels = torch.zeros(pts.nblk, pts.n_pad, dtype=torch.int32, device=dev)
    s = stream()
    call("skcq_pack_centroids", pts.metric, ptr(run.C), pts.nblk, run.k_pad, pts.bs, ptr(k_dev), None, ptr(B),
         ptr(run.cnorm), s)
    assign_call(pts, B, run.C, run.cnorm, run.k_pad, k_dev, None, labels)
    return labels


def scatter_labels(pts: PointSet, labels: torch.Tensor, shared: bool, n_rows: int, n_blocks: int) -> torch.Tensor:
    idxs = torch.empty(n_blocks, n_rows, dtype=torch.int64, device=labels.device)
    call("skcq_scatter_labels", ptr(labels), ptr(pts.rowmap), ptr(pts.n), pts.nblk, pts.n_pad, int(shared), n_rows,
         n_blocks, ptr(idxs), stream())
    return idxs


def row_zero_mask(w: torch.Tensor, thr: float) -> torch.Tensor:
    out = torch.empty(w.shape[0], dtype=torch.uint8, device=w.device)
    call("skcq_row_zero_mask", ptr(w), w.stride(0), w.shape[0], w.shape[1], float(thr), ptr(out), stream())
    return out


def centroids_bf16(C: torch.Tensor, k_pad: int, bs: int, K: int) -> torch.Tensor:
    nblk = C.shape[0]
    out = torch.empty(nblk, bs, K, dtype=torch.bfloat16, device=C.device)
    call("skcq_centroids_to_bf16", ptr(C), nblk, k_pad, bs, K, ptr(out), stream())
    return out


def remainder_bf16(w: torch.Tensor, col0: int) -> torch.Tensor | None:
    rem = w.shape[1] - col0
    if rem <= 0:
        return None
    out = torch.empty(w.shape[0], rem, dtype=torch.bfloat16, device=w.device)
    call("skcq_copy_remainder", ptr(w), w.stride(0), w.shape[0], col0, rem, ptr(out), stream())
    return out


def ssvq_fold(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(folded f32, signs int8) of ssvq.py:43-53."""
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    w = w.contiguous() if w.stride(-1) != 1 else w
    n_rows, in_dim = w.shape
    folded = torch.empty(n_rows, in_dim, dtype=torch.float32, device=w.device)
    signs = torch.empty(n_rows, in_dim, dtype=torch.int8, device=w.device)
    call("skcq_ssvq_fold", ptr(w), int(w.dtype == torch.bfloat16), w.stride(0), n_rows, in_dim, ptr(folded),
         ptr(signs), None, stream())
    return folded, signs


def quantize_centroids_(cb: torch.Tensor, bits: int) -> torch.Tensor:
    """In-place int<bits> fake quantisation of a (n_blocks, bs, K) bf16 tensor."""
    assert cb.dtype == torch.bfloat16 and cb.is_contiguous()
    K = cb.shape[-1]
    call("skcq_quantize_centroids", ptr(cb), cb.numel() // K, K, int(bits), stream())
    return cb


def quantize_scales_int(scales: torch.Tensor, bits: int) -> tuple[torch.Tensor | None, torch.Tensor]:
    """(quantised scales or None when max|s| == 0, q_scale 0-d f32)."""
    s = scales.float().contiguous()
    out = torch.empty(s.shape, dtype=torch.int8 if bits <= 8 else torch.int16, device=s.device)
    q = torch.empty(1, dtype=torch.float32, device=s.device)
    call("skcq_quantize_scales", ptr(s), s.numel(), int(bits), ptr(out), ptr(q), stream())
    q_scale = q.reshape(())
    if float(q_scale) == 0.0:
        return None, q_scale
    return out, q_scale


# ---------------------------------------------------------------------------
# Composite decode
# ---------------------------------------------------------------------------

_SCALE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2, torch.int8: 3, torch.int16: 4}


def _lib_dtype(dt: torch.dtype) -> int:
    """SKCQ_DTYPE_* of a float tensor dtype (f32 or bf16)."""
    return {torch.float32: 0, torch.bfloat16: 1}[dt]


@dataclass
class CodecView:
    """Device tensors of one codebook of a composite, ready for the C ABI."""

    kind: int  # 0 spherical, 1 euclidean
    bs: int
    n_blocks: int
    K: int
    shared: bool
    cent: torch.Tensor  # bf16 (n_cb, bs, K), contiguous
    idxs: torch.Tensor  # int64 (n_blocks, >= n_rows) with unit column stride
    scales: torch.Tensor | None = None
    q_scale: float = 1.0
    rem: torch.Tensor | None = None  # bf16 (n_rows, rem) contiguous
    signs: torch.Tensor | None = None  # int8 (n_rows, >= sign_cols)
    sign_cols: int = 0
    cent_t: torch.Tensor | None = None  # bf16 (n_cb, K, bs): centroid values contiguous

    def transposed(self) -> torch.Tensor:
        """(n_cb, K, bs) copy of ``cent`` (built once per view) for the decode's
        one-sector centroid gathers."""
        if self.cent_t is None:
            n_cb = self.cent.shape[0]
            self.cent_t = torch.empty(n_cb, self.K, self.bs, dtype=self.cent.dtype, device=self.cent.device)
            call("skcq_transpose_codebook", ptr(self.cent), _lib_dtype(self.cent.dtype), n_cb, self.bs, self.K,
                 ptr(self.cent_t), stream())
        return self.cent_t

    def desc(self) -> _lib.CodecDesc:
        d = _lib.CodecDesc()
        d.kind, d.bs, d.n_blocks, d.K, d.shared = self.kind, self.bs, self.n_blocks, self.K, int(self.shared)
        d.cent = ptr(self.cent)
        d.idxs = ptr(self.idxs)
        d.idx_ld = self.idxs.stride(0) if self.idxs.dim() == 2 and self.n_blocks > 0 else 0
        if self.scales is not None:
            d.scales = ptr(self.scales)
            d.scale_dtype = _SCALE_CODES[self.scales.dtype]
            d.q_scale = float(self.q_scale)
            d.scale_ld = self.scales.stride(0)
        if self.rem is not None:
            d.rem = ptr(self.rem)
            d.rem_cols = self.rem.shape[1]
        if self.signs is not None:
            d.signs = ptr(self.signs)
            d.sign_cols = self.sign_cols
            d.sign_ld = self.signs.stride(0)
        if self.cent_t is not None:
            d.cent_t = ptr(self.cent_t)
        return d


def reconstruct(views: list[CodecView], n_rows: int, in_dim: int, raw: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """sum of the codecs' reconstructions, or ``raw - sum`` when raw is given."""
    dev = views[0].cent.device
    if out is None:
        out = torch.empty(n_rows, in_dim, dtype=torch.float32, device=dev)
    for v in views:
        if v.cent.dtype == torch.bfloat16 and v.K > 1:
            v.transposed()
    arr = (_lib.CodecDesc * len(views))(*[v.desc() for v in views])
    call("skcq_reconstruct", _lib.C.cast(arr, _lib.C.c_void_p), len(views), n_rows, in_dim,
         ptr(raw), raw.stride(0) if raw is not None else 0, ptr(out), out.stride(0), stream())
    return out


def refit_scales(primary: CodecView, raw: torch.Tensor, recon: torch.Tensor, row_zero: torch.Tensor,
                 scales: torch.Tensor) -> None:
    d = primary.desc()
    d.scale_dtype = 0
    d.scale_ld = scales.stride(0)
    call("skcq_refit_scales", _lib.C.addressof(d), ptr(raw), raw.stride(0), ptr(recon), recon.stride(0),
         raw.shape[0], ptr(row_zero), ptr(scales), stream())
