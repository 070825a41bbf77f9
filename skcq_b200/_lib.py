"""ctypes binding of ``libskcq_b200.so`` (the C ABI in ``include/skcq_b200.h``).

Every call passes raw device pointers and the current CUDA stream; a non-zero
status raises ``RuntimeError`` carrying ``skcq_last_error()``. There is no
fallback: if the library is missing the import of any compute path fails.
"""

from __future__ import annotations

import ctypes as C
import os
import re
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "libskcq_b200.so"

P = C.c_void_p
I = C.c_int
L = C.c_int64
F = C.c_float


class CodecDesc(C.Structure):
    """``skcq_codec_desc``: one codebook of a composite (include/skcq_b200.h)."""

    _fields_ = [
        ("kind", I), ("bs", I), ("n_blocks", I), ("K", I), ("shared", I),
        ("cent", P), ("idxs", P), ("idx_ld", L),
        ("scales", P), ("scale_dtype", I), ("q_scale", F), ("scale_ld", L),
        ("rem", P), ("rem_cols", I),
        ("signs", P), ("sign_cols", I), ("sign_ld", L),
        ("cent_t", P),
    ]


# name -> argtypes (restype is int unless listed in _RESTYPES)
_SIGS: dict[str, list] = {
    "skcq_last_error": [C.c_char_p, C.c_size_t],
    "skcq_abi_version": [],
    "skcq_poll_device_error": [P],
    "skcq_packed_width": [I, I],
    "skcq_compact_points": [P, L, I, I, I, I, F, I, I, I, P, P, P],
    "skcq_gather_points": [P, L, I, I, I, I, P, P, I, I, P, P, P],
    "skcq_pack_points": [I, P, I, I, I, P, P],
    "skcq_init_from_points": [P, I, I, I, P, L, P, I, P, P],
    "skcq_pack_centroids": [I, P, I, I, I, P, P, P, P, P],
    "skcq_assign": [I, P, P, P, P, P, I, I, I, I, P, P, P, P, P],
    "skcq_assign_exact": [I, P, P, P, I, I, I, I, P, P, P, P, P],
    "skcq_assign_grid_scratch_bytes": [I, I, I, I, I],
    "skcq_assign_grid": [P, P, P, I, I, I, I, P, P, P, I, I, P, P, P, C.c_size_t, P],
    "skcq_update": [P, P, I, I, I, I, P, P, P, P, P, P, P],
    "skcq_reseed_scratch_bytes": [I, I],
    "skcq_reseed": [I, P, P, P, I, I, I, I, P, P, P, P, P, P, P, P],
    "skcq_reseed_noalloc": [I, P, P, P, I, I, I, I, P, P, P, P, P, P, P],
    "skcq_reseed_candidates": [I, P, P, P, I, I, I, I, P, P, P, P, P, I, P, P, P, P, P],
    "skcq_finalize": [I, P, P, P, I, I, I, P, P, P, P, P, P, I, P, P, P],
    "skcq_mark_changed": [P, P, I, I, I, P, P, I, P, P],
    "skcq_moved_lists_scratch_bytes": [I, I, I],
    "skcq_moved_lists": [P, P, I, I, I, P, P, P, P, P, P, P, P, C.c_size_t, P],
    "skcq_gather_rows": [P, I, P, I, P, I, I, I, P, P],
    "skcq_assign_merge": [I, P, P, P, I, I, I, I, P, P, P, P, P, P, P, P, I, P, P, P, P, P, P],
    "skcq_assign_moved_exact": [I, P, P, P, I, I, I, I, P, P, P, P, P, P, P, P, P, P],
    "skcq_list_points": [P, I, I, P, P, P, P, P, C.c_size_t, P],
    "skcq_mpass_points": [P, P, P, P, P, P, I, I, I, I, P, P],
    "skcq_scatter_sub": [P, P, P, I, I, I, P, P],
    "skcq_flip_check": [P, P, P, I, I, I, I, P, P, P],
    "skcq_apply_flip": [P, I, I, I, P, P],
    "skcq_scatter_labels": [P, P, P, I, I, I, I, I, P, P],
    "skcq_row_zero_mask": [P, L, I, I, F, P, P],
    "skcq_spherical_scales": [P, L, I, I, I, I, P, I, P, P, P, P],
    "skcq_centroids_to_bf16": [P, I, I, I, I, P, P],
    "skcq_copy_remainder": [P, L, I, I, I, P, P],
    "skcq_ssvq_fold": [P, I, L, I, I, P, P, P, P],
    "skcq_quantize_centroids": [P, I, I, I, P],
    "skcq_quantize_scales": [P, L, I, P, P, P],
    "skcq_reconstruct": [P, I, I, I, P, L, P, L, P],
    "skcq_refit_scales": [P, P, L, P, L, I, P, P, P],
    "skcq_pack_indices16": [P, L, I, P, P],
    "skcq_transpose_codebook": [P, I, I, I, I, P, P],
    "skcq_pack_sign_masks": [P, I, I, L, I, I, P, P],
    "skcq_lut_build": [P, P, I, L, I, P, P],
    "skcq_selftest_wait_timeout": [C.c_longlong, P],
    "skcq_route_sort": [P, I, I, I, P, P, P, P, P, C.c_size_t, I, P],
    "skcq_route_sort_scratch_bytes": [I, I, I],
    "skcq_codebook_forward": [P, I, P, I, L, P, I, P, P, P, I, I, I, I, I, I, P, L, P],
    "skcq_sum_splits": [P, I, L, I, P, I, L, P],
    "skcq_swiglu": [P, P, I, L, P, P],
    "skcq_combine": [P, I, I, L, P, P, P, I, I, I, I, P, I, P],
    "skcq_prefill_plan": [P, I, I, P, P],
    "skcq_prefill_pack": [I, P, I, L, P, I, P, L, I, P, I, P, P],
    "skcq_prefill_dequant": [P, I, P, I, I, I, I, P, P],
    "skcq_prefill_gemm": [P, P, P, I, I, I, P, I, L, P],
    "skcq_prefill_gemm_swiglu": [P, P, P, I, I, I, P, P],
    "skcq_ep_layout": [I, I, I, I, P],
    "skcq_ep_alloc": [C.c_size_t, C.POINTER(P), P],
    "skcq_ep_open": [P, C.POINTER(P)],
    "skcq_ep_close": [P],
    "skcq_ep_free": [P],
    "skcq_ep_dispatch": [P, I, L, P, P, I, I, I, I, P, P, I, I, I, I, I, P, P, P],
    "skcq_ep_unpack": [P, I, I, I, I, I, P, P, P],
    "skcq_ep_return": [P, I, I, L, P, P, P, P, P, P, I, I, I, I, I, I, I, I, P],
    "skcq_ep_gather": [P, P, I, I, I, I, I, I, P, I, P],
}
_RESTYPES = {"skcq_reseed_scratch_bytes": C.c_size_t, "skcq_assign_grid_scratch_bytes": C.c_size_t, "skcq_route_sort_scratch_bytes": C.c_size_t,
             "skcq_moved_lists_scratch_bytes": C.c_size_t}

_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Load (once) and type the shared library; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("SKCQ_B200_LIB", _LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"skcq_b200 CUDA library not found at {path}; build it with `python -m skcq_b200.build`"
        )
    lib = C.CDLL(str(path))
    for name, args in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, I)
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    load().skcq_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


# Kernels each entry point launches (for launch accounting by the benchmark).
_KERNELS_PER_CALL = {
    "skcq_compact_points": 1, "skcq_gather_points": 1, "skcq_pack_points": 1, "skcq_init_from_points": 1,
    "skcq_pack_centroids": 1, "skcq_assign": 2, "skcq_assign_exact": 1, "skcq_assign_grid": 6, "skcq_update": 1, "skcq_reseed": 1, "skcq_reseed_noalloc": 1, "skcq_reseed_candidates": 1,
    "skcq_finalize": 1, "skcq_flip_check": 1, "skcq_apply_flip": 1, "skcq_scatter_labels": 1,
    "skcq_row_zero_mask": 1, "skcq_spherical_scales": 1, "skcq_centroids_to_bf16": 1, "skcq_copy_remainder": 1,
    "skcq_ssvq_fold": 1, "skcq_quantize_centroids": 1, "skcq_quantize_scales": 3, "skcq_reconstruct": 1,
    "skcq_refit_scales": 1, "skcq_pack_indices16": 1, "skcq_transpose_codebook": 1, "skcq_pack_sign_masks": 1,
    "skcq_lut_build": 1, "skcq_selftest_wait_timeout": 1,
    "skcq_route_sort": 1, "skcq_sum_splits": 1, "skcq_swiglu": 1, "skcq_combine": 1,
    "skcq_prefill_plan": 1, "skcq_prefill_pack": 1, "skcq_prefill_dequant": 1, "skcq_prefill_gemm": 1,
    "skcq_mark_changed": 2, "skcq_moved_lists": 4, "skcq_gather_rows": 1, "skcq_assign_merge": 2,
    "skcq_assign_moved_exact": 1, "skcq_list_points": 2,
    "skcq_mpass_points": 1, "skcq_scatter_sub": 1,
    "skcq_prefill_gemm_swiglu": 1, "skcq_ep_dispatch": 3, "skcq_ep_unpack": 1, "skcq_ep_return": 1,
    "skcq_ep_gather": 1,
}


class LaunchCounter:
    """Counts kernel launches made through ``call`` while enabled."""

    def __init__(self) -> None:
        self.enabled = False
        self.kernels = 0
        self.calls: dict[str, int] = {}

    def reset(self) -> None:
        self.kernels = 0
        self.calls = {}


LAUNCHES = LaunchCounter()


def call(name: str, *args) -> int:
    """Call ``name`` and raise ``RuntimeError`` on a non-zero status."""
    rc = getattr(load(), name)(*args)
    if rc != 0:
        raise RuntimeError(f"{name} failed ({rc}): {last_error()}")
    if LAUNCHES.enabled:
        # the grouped forward launches one kernel per codebook layer (argument 1)
        if name == "skcq_codebook_forward":
            LAUNCHES.kernels += args[1]  # one kernel per codebook layer
        elif name == "skcq_route_sort":
            LAUNCHES.kernels += 3 if args[8] else 1  # multi-CTA form when given scratch
        else:
            LAUNCHES.kernels += _KERNELS_PER_CALL.get(name, 0)
        LAUNCHES.calls[name] = LAUNCHES.calls.get(name, 0) + 1
    return rc


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("skcq_b200 kernels take CUDA tensors")
    return t.data_ptr()


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def poll_device_error() -> None:
    """Raise if a kernel recorded a device-side error since the last poll:
    ``DeviceTimeoutError`` when a bounded wait ran out (the job may be retried),
    ``RuntimeError`` for a failed data check (a bug or invalid input)."""
    from skcq_b200.errors import WAIT_TIMEOUT_CODES, DeviceTimeoutError

    rc = load().skcq_poll_device_error(stream())
    if rc == 0:
        return
    msg = last_error()
    m = re.search(r"\(code (\d+)\)", msg)
    code = int(m.group(1)) if m else -1
    if rc == -3 and code in WAIT_TIMEOUT_CODES:
        raise DeviceTimeoutError(f"skcq_poll_device_error: {msg}", code)
    raise RuntimeError(f"skcq_poll_device_error failed ({rc}): {msg}")
