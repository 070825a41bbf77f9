"""Kernel micro-benchmark: time one engine kernel on synthetic shapes.

    python -m skcq_b200.kernel_bench assign --metric l2 --bs 4 --K 65536 --blocks 64 --rows 98304 --reps 3
    python -m skcq_b200.kernel_bench prefill --experts 128 --tokens 16384 --reps 3
    python -m skcq_b200.kernel_bench dequant --experts 32 --reps 3
    python -m skcq_b200.kernel_bench decode --experts 32 --tokens 1 --reps 3
    python -m skcq_b200.kernel_bench update --metric cosine --bs 8 --K 4096 --blocks 128 --rows 98304 --reps 3
    python -m skcq_b200.kernel_bench reconstruct --rows 98304 --reps 3

The forward cases build random codebook modules with the config-2 codebook
shapes (primary bs=8 K=4096 with bf16 scales, residuals bs=16 K=4096 and
bs=4 K=65536; hidden 2048, intermediate 768) and uniform random indices.
`prefill` times every launch of one CodebookExperts forward (Zipf(1.1)
routing, top-8) with CUDA events; `dequant` decodes one gate projection's
experts; `decode` runs one routed step of T tokens.

`update` times the Lloyd centroid update (segmented sum of the points into
their clusters' sums and counts) on random labels; `reconstruct` times one
streaming reconstruction pass of a gate projection (98304 x 2048 by default)
from random config-2 codebooks (primary bs=8 K=4096 with bf16 scales, residuals
bs=16 K=4096 and bs=4 K=65536, int64 indices as in the CWR), as the AQLM
residual ``raw - sum``.

Prints one JSON line per case with the mean CUDA-event time per launch and the
algorithmic work rate (bytes for the HBM-bound cases, against the measured
copy bandwidth in MEASURED_PEAKS.json). Useful as the target of a profiler capture (few launches,
bounded device memory).
"""

from __future__ import annotations

import argparse
import json

import torch

from skcq_b200 import _engine, _lib
from skcq_b200._lib import call, ptr, stream


def assign_case(metric: int, bs: int, K: int, blocks: int, rows: int, reps: int, warmup: int) -> dict:
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(rows, blocks * bs, generator=g, device=dev) * 0.02
    pts = _engine.gather_block_points(w, bs, blocks, False, 0.0, False, metric)
    del w
    k_pad = _engine.round_up(K, _engine.CENT_TILE)
    C = torch.randn(blocks, k_pad, bs, generator=g, device=dev) * 0.02
    if metric == _engine.COSINE:
        C = torch.nn.functional.normalize(C, dim=-1)
    k_dev = torch.full((blocks,), K, dtype=torch.int32, device=dev)
    B = torch.empty(blocks, k_pad * pts.kp, device=dev)
    cnorm = torch.empty(blocks, k_pad, device=dev)
    labels = torch.empty(blocks, pts.n_pad, dtype=torch.int32, device=dev)
    A = pts.packed()
    s = stream()
    call("skcq_pack_centroids", metric, ptr(C), blocks, k_pad, bs, ptr(k_dev), None, ptr(B), ptr(cnorm), s)

    def launch():
        call("skcq_assign", metric, ptr(A), ptr(B), ptr(pts.X), ptr(C), ptr(cnorm), blocks, pts.n_pad, k_pad, bs,
             ptr(pts.n), ptr(k_dev), None, ptr(labels), s)

    for _ in range(warmup):
        launch()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in ev:
        a.record()
        launch()
        b.record()
    torch.cuda.synchronize()
    _lib.poll_device_error()
    ms = sum(a.elapsed_time(b) for a, b in ev) / reps
    elems = float(rows) * K * blocks
    res = {
        "case": "assign", "metric": "cosine" if metric == 0 else "l2", "bs": bs, "K": K, "blocks": blocks,
        "rows": rows, "kp": pts.kp, "ms_per_launch": ms, "elements_per_s": elems / (ms / 1e3),
        "algorithmic_tflops": 2 * bs * elems / (ms / 1e3) / 1e12,
        "issued_tf32_tflops": 2 * pts.kp * elems / (ms / 1e3) / 1e12,
        "a_bytes": A.numel() * 4, "b_bytes": B.numel() * 4,
    }
    if metric == _engine.L2 and 2 <= bs <= 4 and k_pad >= _engine.GRID_MIN_K:
        # the centroid grid (plus the tensor-core search of uncertified points)
        # against the tensor-core pass above, on the same points and centroids
        lab_g = torch.empty_like(labels)

        def grid():
            _engine.assign_call(pts, B, C, cnorm, k_pad, k_dev, None, lab_g)

        ring_default = _engine.GRID_RING
        by_ring = {}
        try:
            for ring in (0, 2, 3):  # largest box radius of the second search of uncertified points
                _engine.GRID_RING = ring
                for _ in range(max(warmup, 1)):
                    grid()
                torch.cuda.synchronize()
                times = []
                for _ in range(reps):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    grid()
                    b.record()
                    torch.cuda.synchronize()
                    times.append(a.elapsed_time(b))
                by_ring[ring] = sum(times) / len(times)
        finally:
            _engine.GRID_RING = ring_default
        times = [by_ring[ring_default]]
        _engine.GRID_STATS.update(enabled=True, points=0.0, fallback=0.0)
        try:
            grid()
        finally:
            _engine.GRID_STATS["enabled"] = False
        launch()
        torch.cuda.synchronize()
        _lib.poll_device_error()
        same = (lab_g[:, :rows] == labels[:, :rows]).float().mean().item()
        gms = sum(times) / len(times)
        res["grid"] = {"ms_per_call": gms, "speedup_vs_tensor_pass": ms / gms, "cells_per_coordinate":
                       _engine.grid_cells(bs, k_pad), "fallback_share":
                       _engine.GRID_STATS["fallback"] / max(_engine.GRID_STATS["points"], 1.0),
                       "labels_equal_tensor_pass": same, "ring_max": ring_default,
                       "ms_per_call_by_ring_max": by_ring}
    return res


def _hbm_peak() -> float:
    import json
    from pathlib import Path

    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0  # fallback measurement on this GPU type


def _time(launch, prepare, reps: int, warmup: int) -> float:
    for _ in range(warmup):
        prepare()
        launch()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(reps):
        prepare()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        launch()
        b.record()
        torch.cuda.synchronize()
        total += a.elapsed_time(b)
    _lib.poll_device_error()
    return total / reps


def update_case(metric: int, bs: int, K: int, blocks: int, rows: int, reps: int, warmup: int) -> dict:
    """skcq_update on random labels. Algorithmic bytes: each point's coordinates
    and label read once, every cluster's sum and count written once."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(rows, blocks * bs, generator=g, device=dev) * 0.02
    pts = _engine.gather_block_points(w, bs, blocks, False, 0.0, False, metric)
    del w
    k_pad = _engine.round_up(K, _engine.CENT_TILE)
    k_dev = torch.full((blocks,), K, dtype=torch.int32, device=dev)
    labels = torch.randint(0, K, (blocks, pts.n_pad), generator=g, device=dev, dtype=torch.int32)
    sums = torch.empty(blocks, k_pad, bs, device=dev)
    counts = torch.empty(blocks, k_pad, dtype=torch.int32, device=dev)
    s = stream()

    def prepare():
        sums.zero_()
        counts.zero_()

    ms = _time(lambda: call("skcq_update", ptr(pts.R), ptr(labels), blocks, pts.n_pad, k_pad, bs, ptr(pts.n),
                            ptr(k_dev), None, ptr(sums), ptr(counts), None, s), prepare, reps, warmup)
    n_pts = float(sum(pts.n_host))
    algo = n_pts * (bs * 4 + 4) + blocks * K * (bs + 1) * 4.0
    gbs = algo / (ms / 1e3) / 1e9
    return {"case": "update", "metric": "cosine" if metric == 0 else "l2", "bs": bs, "K": K, "blocks": blocks,
            "rows": rows, "ms_per_launch": ms, "algorithmic_bytes": algo, "achieved_gbs": gbs,
            "frac_hbm": gbs / _hbm_peak()}


def reconstruct_case(rows: int, reps: int, warmup: int, in_dim: int = 2048) -> dict:
    """One skcq_reconstruct pass, raw - (primary + 2 residuals). Algorithmic
    bytes: indices, scales, raw and output streamed once, each centroid table
    read once."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    views = []
    table_bytes = idx_bytes = 0
    for kind, bs, K, scaled in ((0, 8, 4096, True), (1, 16, 4096, False), (1, 4, 65536, False)):
        nb = in_dim // bs
        cent = (torch.randn(nb, bs, K, generator=g, device=dev) * 0.05).to(torch.bfloat16)
        idxs = torch.randint(0, K, (nb, rows), generator=g, device=dev, dtype=torch.int64)
        scales = (torch.rand(rows, nb, generator=g, device=dev) * 0.1).to(torch.bfloat16) if scaled else None
        views.append(_engine.CodecView(kind=kind, bs=bs, n_blocks=nb, K=K, shared=False, cent=cent, idxs=idxs,
                                       scales=scales))
        table_bytes += cent.numel() * 2
        idx_bytes += idxs.numel() * 8 + (scales.numel() * 2 if scales is not None else 0)
    raw = torch.randn(rows, in_dim, generator=g, device=dev) * 0.02
    out = torch.empty(rows, in_dim, device=dev)
    ms = _time(lambda: _engine.reconstruct(views, rows, in_dim, raw=raw, out=out), lambda: None, reps, warmup)
    algo = float(idx_bytes + table_bytes + raw.numel() * 4 + out.numel() * 4)
    gbs = algo / (ms / 1e3) / 1e9
    return {"case": "reconstruct", "rows": rows, "in_dim": in_dim, "ms_per_launch": ms, "algorithmic_bytes": algo,
            "index_and_scale_bytes": float(idx_bytes), "table_bytes": float(table_bytes), "achieved_gbs": gbs,
            "frac_hbm": gbs / _hbm_peak()}


def _random_module(E: int, out_dim: int, in_dim: int, gen: torch.Generator):
    from skcq_b200.codebook_experts import CodebookModule, _CodebookLayer

    dev = gen.device
    layers = []
    for i, (bs, K) in enumerate([(8, 4096), (16, 4096), (4, 65536)]):
        nb = in_dim // bs
        cb = (torch.randn(nb, bs, K, generator=gen, device=dev) * 0.05).to(torch.bfloat16)
        a = torch.randint(0, K, (E, nb, out_dim), generator=gen, device=dev)
        sc = (torch.rand(E, nb, out_dim, generator=gen, device=dev) * 0.1).to(torch.bfloat16) if i == 0 else None
        layers.append(_CodebookLayer(cb, a, nb, bs, out_dim, K, scales=sc))
    return CodebookModule(torch.nn.ModuleList(layers), len(layers), out_dim)


def _experts(E: int, gen: torch.Generator):
    from skcq_b200.codebook_experts import CodebookExperts

    H, I = 2048, 768
    ex = CodebookExperts(_random_module(E, I, H, gen), _random_module(E, I, H, gen), _random_module(E, H, I, gen),
                         E, torch.nn.functional.silu)
    ex.check_errors = False
    return ex


def forward_case(kind: str, E: int, T: int, reps: int, warmup: int) -> dict:
    """Median device time of one forward-path call and per-launch stage times."""
    import skcq_b200.codebook_experts as ce

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    if kind == "dequant":
        gate = _random_module(E, 768, 2048, g)
        KC, NT = 2048 // 64, 768 // 256
        W = torch.empty(E * NT * KC * 16384, dtype=torch.bfloat16, device=dev)

        def fn():
            gate.dequant_into(W, None, E, 2048)

        work = {"weights": E * 768 * 2048}
    else:
        ex = _experts(E, g)
        if kind == "prefill":
            ranks = torch.randperm(E, generator=g, device=dev).float() + 1
            u = torch.rand(T, E, generator=g, device=dev).clamp_(1e-20, 1)
            logits = -1.1 * torch.log(ranks)[None] - torch.log(-torch.log(u))
        else:
            logits = torch.randn(T, E, generator=g, device=dev)
        topw, topi = torch.topk(torch.softmax(logits, -1), 8, dim=-1)
        x = torch.randn(T, 2048, generator=g, device=dev).to(torch.bfloat16)

        def fn():
            ex(x, topi, topw)

        work = {"tokens": T, "flops": 2.0 * T * 8 * 3 * 2048 * 768}
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    stages: dict[str, list] = {}
    orig = ce.call

    def timed(name, *args):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        rc = orig(name, *args)
        b.record()
        stages.setdefault(name, []).append((a, b))
        return rc

    total = []
    for _ in range(reps):
        stages.clear()
        ce.call = timed
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        try:
            a.record()
            fn()
            b.record()
        finally:
            ce.call = orig
        torch.cuda.synchronize()
        total.append(a.elapsed_time(b))
    _lib.poll_device_error()
    ms = sorted(total)[len(total) // 2]
    return {"case": kind, "experts": E, "tokens": T, "ms": ms, **work,
            "stages_ms": {k: [round(x.elapsed_time(y), 4) for x, y in v] for k, v in stages.items()}}


def lloyd_case(metric: int, bs: int, K: int, blocks: int, rows: int, iters: int) -> dict:
    """One batched Lloyd run (Student-t(5) block rows at std 0.02, Sobol start
    for cosine, Forgy for euclidean) with every assignment timed: the
    incremental schedule against the all-full-pass schedule on the same
    points."""
    from skcq_b200.codebook.kmeans import sobol_first_orthant

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    z = torch.randn(rows, blocks * bs, generator=g, device=dev)
    chi2 = torch.randn(5, rows, blocks * bs, generator=g, device=dev).square_().sum(0)
    w = z / torch.sqrt(chi2 / 5.0) * (0.02 / (5.0 / 3.0) ** 0.5)
    del z, chi2
    pts = _engine.gather_block_points(w, bs, blocks, False, 0.0, False, metric)
    del w
    gp = torch.Generator().manual_seed(1)
    perms = [torch.randperm(nb, generator=gp) for nb in pts.n_host]
    out = {"case": "lloyd", "metric": "cosine" if metric == 0 else "l2", "bs": bs, "K": K, "blocks": blocks,
           "rows": rows, "iters": iters}
    for label, inc in (("incremental", True), ("full", False)):
        _engine.INCREMENTAL = inc
        try:
            for timed in (False, True):  # one untimed run first (kernel set-up)
                _engine.TIMER.reset()
                _engine.TIMER.enabled = timed
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                if metric == _engine.COSINE:
                    run = _engine.lloyd(pts, K, iters, init_cosine=lambda kk, dd: sobol_first_orthant(kk, dd, dev))
                else:
                    run = _engine.lloyd(pts, K, iters, init_perms=perms)
                b.record()
                torch.cuda.synchronize()
        finally:
            _engine.INCREMENTAL = True
            _engine.TIMER.enabled = False
        full_work = 2.0 * bs * float(sum(pts.n_host)) * K
        assigns = [(round(s.elapsed_time(e), 3), round(work / full_work, 4))
                   for name, s, e, work, _, _ in _engine.TIMER.records if name == "assign"]
        out[label] = {"ms": a.elapsed_time(b), "iters_run": max(run.iters_run),
                      "assign_ms": round(sum(x for x, _ in assigns), 2),
                      "assignments": [{"ms": x, "work_share": y} for x, y in assigns]}
    _lib.poll_device_error()
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["assign", "prefill", "dequant", "decode", "update", "reconstruct", "lloyd"])
    ap.add_argument("--iters", type=int, default=25)
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--metric", default="l2", choices=["cosine", "l2"])
    ap.add_argument("--bs", type=int, default=4)
    ap.add_argument("--K", type=int, default=65536)
    ap.add_argument("--blocks", type=int, default=64)
    ap.add_argument("--rows", type=int, default=98304)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--grid", choices=["on", "off"], default="on",
                    help="centroid-grid search for low-dimensional euclidean problems (off: tensor-core pass)")
    a = ap.parse_args()
    _lib.load()
    _engine.GRID = a.grid == "on"
    metric = _engine.COSINE if a.metric == "cosine" else _engine.L2
    if a.kernel == "assign":
        res = assign_case(metric, a.bs, a.K, a.blocks, a.rows, a.reps, a.warmup)
    elif a.kernel == "update":
        res = update_case(metric, a.bs, a.K, a.blocks, a.rows, a.reps, a.warmup)
    elif a.kernel == "lloyd":
        res = lloyd_case(metric, a.bs, a.K, a.blocks, a.rows, a.iters)
    elif a.kernel == "reconstruct":
        res = reconstruct_case(a.rows, a.reps, a.warmup)
    else:
        res = forward_case(a.kernel, a.experts, a.tokens, a.reps, a.warmup)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
