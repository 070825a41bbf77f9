"""Pin the CPU oracle against vectors produced by the SKCQ reference itself.

The fixtures under tests/golden/ were written by tests/golden/make_golden.py
running the reference (CPU torch). These tests need neither the reference nor
a GPU.
"""

from __future__ import annotations

import numpy as np
import pytest

from _helpers import PermReplay, bf16_from_bits, load_golden, rel_err, sobol_np, sub
from oracle import codecs as oc
from oracle import forward as of
from oracle import kmeans as ok


def test_assign_matches_reference():
    g = load_golden("assign")
    s = ok.scores_cosine(g["cos_data"], g["cos_cent"].T)
    lab = ok.assign_cosine(g["cos_data"], g["cos_cent"].T)
    margin = ok.top2_margin(s, True)
    m = margin > 1e-6
    assert (lab[m] == g["cos_labels"][m]).all()
    assert (lab == g["cos_labels"]).mean() > 0.999
    s2 = ok.scores_l2(g["l2_data"], g["l2_cent"].T)
    lab2 = ok.assign_l2(g["l2_data"], g["l2_cent"].T)
    m2 = ok.top2_margin(s2, False) > 1e-9
    assert (lab2[m2] == g["l2_labels"][m2]).all()


@pytest.mark.parametrize("name", ["cos_a", "cos_empty", "l2_a", "l2_empty"])
def test_kmeans_fit_matches_reference(name):
    g = sub(load_golden("kmeans"), name + "__")
    n, d, k, iters, is_cos = (int(v) for v in g["meta"])
    data = g["data"]
    if is_cos:
        cent, labels, log = ok.fit_cosine(data, data, k, iters, sobol_np(min(k, n), d))
    else:
        cent, labels, log = ok.fit_euclidean(data, k, iters, PermReplay.from_case(g)(n))
    assert rel_err(cent, g["centroids"]) < 1e-5
    assert (labels == g["labels"]).mean() > 0.99
    ev = g["ev_int"]
    iter_rows = ev[ev[:, 0] == 1]
    assert [e for _, e in log.iters] == list(iter_rows[:, 2])  # n_empty per iteration
    np.testing.assert_allclose([m for m, _ in log.iters], g["ev_moved"][ev[:, 0] == 1], rtol=1e-4, atol=1e-7)
    done = ev[ev[:, 0] == 2][0]
    assert log.iters_run == done[1] and int(log.converged) == done[2]
    if name.endswith("empty"):
        assert any(e > 0 for _, e in log.iters), "fixture must exercise the empty-cluster reseed"


def _spec(name: str, meta_res: int):
    kw = {
        "base": {}, "single": {"k_list": (16,)}, "ssvq": {"sign_split": True},
        "noncomm": {"block_size": 10, "rbs": 12}, "asym": {"k_list": (16, 8)},
        "shared": {"shared": True}, "int8cb": {"k_list": (16, 8), "codebook_bits": 8},
        "skipz": {"norm_threshold": 1e-5, "skip_zeros": True},
        "ressign": {"res_sign_split": True, "k_list": (16, 16, 8)}, "rem13": {"k_list": (16,)},
    }[name]
    bs = kw.get("block_size", 4)
    k_list = kw.get("k_list", (16, 16))
    thr = kw.get("norm_threshold", 1e-9)
    prim = ("spherical", oc.SphericalCfg(bs, k_list[0], shared=kw.get("shared", False), max_iters=10,
                                         norm_threshold=thr, skip_zeros=kw.get("skip_zeros", False)))
    if kw.get("sign_split"):
        prim = ("ssvq", prim)
    res = []
    for kc in k_list[1:]:
        r = ("euclidean", oc.EuclideanCfg(kw.get("rbs") or bs, kc, shared=kw.get("shared", False),
                                         max_iters=10, norm_threshold=thr, skip_zeros=False))
        if kw.get("res_sign_split"):
            r = ("ssvq", r)
        res.append(r)
    assert len(res) == meta_res
    return prim, res, kw.get("codebook_bits", 16), thr


CODEC_CASES = ["base", "single", "ssvq", "noncomm", "asym", "shared", "int8cb", "skipz", "ressign", "rem13"]


def _check_codec(prefix: str, codec: oc.Codec, cwr: dict, g: dict) -> None:
    if f"{prefix}signs" in g:
        assert (cwr["signs"] == g[f"{prefix}signs"]).mean() > 0.98  # signs of near-zero errors may flip
        codec, cwr = codec.inner, cwr["inner"]
    agree = (cwr["idxs"] == g[f"{prefix}idxs"]).mean()
    assert agree > 0.98, f"{prefix} idx agreement {agree}"
    cent = bf16_from_bits(g[f"{prefix}cent_bf16"])
    assert rel_err(codec.centroids, cent) < 1e-2
    if f"{prefix}rem_bf16" in g:
        assert rel_err(cwr["remainder"], bf16_from_bits(g[f"{prefix}rem_bf16"])) < 1e-2


def codec_logs(c: oc.Codec) -> list:
    return codec_logs(c.inner) if c.kind == "ssvq" else c.logs


# relative top-2 gap below which a k-means trajectory depends on rounding order
TIE = 1e-6
STRICT_SEEN: set[str] = set()


@pytest.mark.parametrize("name", CODEC_CASES)
def test_aqlm_fit_matches_reference(name):
    """Strict parity where the oracle's trajectory has no near-tie; otherwise the
    reference itself is rounding-order dependent and only quality must agree."""
    g = sub(load_golden("codecs"), name + "__")
    prim, res, bits, thr = _spec(name, int(g["meta"][2]))
    primary, residuals, cwr = oc.aqlm_fit(prim, res, g["w"], sobol_np, PermReplay.from_case(g),
                                          codebook_bits=bits, norm_threshold=thr)
    recon = oc.aqlm_reconstruct(primary, residuals, cwr)
    w = g["w"].astype(np.float64)
    e_ref = np.linalg.norm(w - g["recon"]) / np.linalg.norm(w)
    e_or = np.linalg.norm(w - recon) / np.linalg.norm(w)
    logs = [lg for c in [primary, *residuals] for lg in codec_logs(c)]
    if not all(lg.min_margin > TIE for lg in logs):
        assert abs(e_or - e_ref) <= 0.15 * e_ref
        return
    STRICT_SEEN.add(name)
    assert rel_err(recon, g["recon"]) < 2e-3
    assert abs(e_or - e_ref) <= 1e-3 * e_ref + 1e-7
    if any(lg.exact_ties for lg in logs):
        return  # labels among bit-identical centroids are interchangeable
    _check_codec("c0_", primary, cwr["primary"], g)
    for i, (r, rc) in enumerate(zip(residuals, cwr["residuals"], strict=True)):
        _check_codec(f"c{i + 1}_", r, rc, g)
    if "fwd" in g:
        layers = of.layers_from_fit([primary, *residuals], [cwr["primary"], *cwr["residuals"]], 8)
        fwd = np.stack([of.module_forward(layers, g["hidden"], e) for e in range(g["fwd"].shape[0])])
        assert rel_err(fwd, g["fwd"]) < 2e-3


def test_enough_strict_codec_cases():
    """Most of the reference's unit-test configurations must pin strictly."""
    for name in CODEC_CASES:
        if name not in STRICT_SEEN:
            try:
                test_aqlm_fit_matches_reference(name)
            except AssertionError:
                pass
    assert len(STRICT_SEEN) >= 8, sorted(STRICT_SEEN)


def test_int8_scale_quant_matches_reference():
    g = sub(load_golden("codecs"), "sq8__")
    prim, res, _, _ = _spec("base", 1)
    primary, residuals, cwr = oc.aqlm_fit(prim, res, g["w"], sobol_np, PermReplay.from_case(g), norm_threshold=1e-9)
    oc.quantize_scales(cwr["primary"], primary, "int8")
    assert cwr["primary"]["scales"].dtype == np.int8
    assert abs(primary.q_scale - g["q_scale"][0]) < 1e-6 * abs(g["q_scale"][0])
    assert (cwr["primary"]["scales"] == g["scales_q"]).mean() > 0.98
    assert rel_err(oc.aqlm_reconstruct(primary, residuals, cwr), g["recon"]) < 5e-3


def test_experts_forward_matches_reference():
    g = load_golden("experts")
    replay = PermReplay.from_case(g)
    mods = []
    for w, out_dim in ((g["wg"], 8), (g["wu"], 8), (g["wd"], 12)):
        prim = ("spherical", oc.SphericalCfg(4, 16, max_iters=10, norm_threshold=1e-9, skip_zeros=False))
        res = [("euclidean", oc.EuclideanCfg(4, 8, max_iters=10, norm_threshold=1e-9, skip_zeros=False))]
        p, rs, cwr = oc.aqlm_fit(prim, res, w, sobol_np, replay, norm_threshold=1e-9)
        mods.append(of.layers_from_fit([p, *rs], [cwr["primary"], *cwr["residuals"]], out_dim))
    y = of.experts_forward(mods[0], mods[1], mods[2], 4, g["hidden"], g["topi"], g["topw"])
    assert rel_err(y, g["y"]) < 2e-3


def test_config1_matches_reference():
    """The CPU-runnable 768x2048 matrix: SSVQ spherical bs=8 K=256 + euclidean bs=4 K=256."""
    g = load_golden("config1")
    w = bf16_from_bits(g["w_bf16"]).reshape(768, 2048)
    prim = ("ssvq", ("spherical", oc.SphericalCfg(8, 256, max_iters=20)))
    res = [("euclidean", oc.EuclideanCfg(4, 256, max_iters=20, skip_zeros=False))]
    primary, residuals, cwr = oc.aqlm_fit(prim, res, w, sobol_np, PermReplay.from_case(g))
    recon = oc.aqlm_reconstruct(primary, residuals, cwr)
    rel = float(np.linalg.norm(w - recon) / np.linalg.norm(w))
    assert abs(rel - g["rel_fro_err"][0]) < 1e-3 * g["rel_fro_err"][0]
    assert rel_err(recon[::37], g["recon_rows"]) < 5e-3
    assert (cwr["primary"]["inner"]["idxs"] == g["c0_idxs"]).mean() > 0.99
    assert (cwr["residuals"][0]["idxs"] == g["c1_idxs"]).mean() > 0.95
    ev = g["ev_int"]
    ref_iters = ev[ev[:, 0] == 2][:, 1]
    our_iters = np.array([lg.iters_run for lg in primary.inner.logs + residuals[0].logs])
    assert (our_iters == ref_iters).mean() > 0.95
