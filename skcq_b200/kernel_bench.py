"""Kernel micro-benchmark: time one engine kernel on synthetic shapes.

    python -m skcq_b200.kernel_bench assign --metric l2 --bs 4 --K 65536 --blocks 64 --rows 98304 --reps 3

Prints one JSON line per case with the mean CUDA-event time per launch and the
algorithmic work rate. Useful as the target of a profiler capture (few launches,
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
    return {
        "case": "assign", "metric": "cosine" if metric == 0 else "l2", "bs": bs, "K": K, "blocks": blocks,
        "rows": rows, "kp": pts.kp, "ms_per_launch": ms, "elements_per_s": elems / (ms / 1e3),
        "algorithmic_tflops": 2 * bs * elems / (ms / 1e3) / 1e12,
        "issued_tf32_tflops": 2 * pts.kp * elems / (ms / 1e3) / 1e12,
        "a_bytes": A.numel() * 4, "b_bytes": B.numel() * 4,
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["assign"])
    ap.add_argument("--metric", default="l2", choices=["cosine", "l2"])
    ap.add_argument("--bs", type=int, default=4)
    ap.add_argument("--K", type=int, default=65536)
    ap.add_argument("--blocks", type=int, default=64)
    ap.add_argument("--rows", type=int, default=98304)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    a = ap.parse_args()
    _lib.load()
    metric = _engine.COSINE if a.metric == "cosine" else _engine.L2
    print(json.dumps(assign_case(metric, a.bs, a.K, a.blocks, a.rows, a.reps, a.warmup)), flush=True)


if __name__ == "__main__":
    main()
