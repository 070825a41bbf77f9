"""GPU parity of the codebook-build path against the oracle and the reference's
golden vectors. Every test here runs the CUDA kernels through the C ABI."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _helpers import PermReplay, bf16_from_bits, load_golden, rel_err, sobol_np, sub
from oracle import codecs as oc
from oracle import kmeans as ok

pytestmark = pytest.mark.gpu

TIE = 1e-6  # relative top-2 gap below which labels may legitimately differ


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from skcq_b200 import _lib

    _lib.load()


def _problem(metric: int, nblk: int, n: int, bs: int, K: int, seed: int):
    """Random problem set through the product's own gather/pack path."""
    from skcq_b200 import _engine

    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, nblk * bs, generator=g) * 0.05
    if metric == _engine.L2:
        w = w * torch.rand(n, 1, generator=g)  # varied norms
    wd = w.cuda()
    pts = _engine.gather_block_points(wd, bs, nblk, False, 0.0, False, metric)
    C = torch.randn(nblk, K, bs, generator=g) * 0.05
    if metric == _engine.COSINE:
        C = torch.nn.functional.normalize(C, dim=-1)
    return w, pts, C


def _labels(pts, C, exact: bool):
    from skcq_b200 import _engine
    from skcq_b200._lib import call, ptr, stream

    nblk, K, bs = C.shape
    k_pad = _engine.round_up(K, _engine.CENT_TILE)
    Cd = torch.zeros(nblk, k_pad, bs, device="cuda")
    Cd[:, :K] = C.cuda()
    run = _engine.KmeansRun(C=Cd, k_pad=k_pad, k_host=[K] * nblk, labels=None, iters_run=[], converged=[],
                            moved=None, n_empty=None, cnorm=torch.empty(nblk, k_pad, device="cuda"))
    lab = _engine.assign(pts, run)
    if exact:
        k_dev = torch.full((nblk,), K, dtype=torch.int32, device="cuda")
        call("skcq_assign_exact", pts.metric, ptr(pts.X), ptr(Cd), ptr(run.cnorm), nblk, pts.n_pad, k_pad, bs,
             ptr(pts.n), ptr(k_dev), None, ptr(lab), stream())
    torch.cuda.synchronize()
    return lab[:, : pts.n_host[0]].cpu().numpy()


def _check_assign(metric, bs, K, n, nblk, seed):
    w, pts, C = _problem(metric, nblk, n, bs, K, seed=seed)
    lab_tc = _labels(pts, C, exact=False)
    lab_ex = _labels(pts, C, exact=True)
    for b in range(nblk):
        x = w[:, b * bs : (b + 1) * bs].numpy()
        c = C[b].numpy()
        if metric == 0:
            s = ok.scores_cosine(ok.normalize_rows(x), c.T)
        else:
            s = ok.scores_l2(x, c.T)
        maximise = metric == 0
        ref = s.argmax(1) if maximise else s.argmin(1)
        sm = s if maximise else -s
        part = np.partition(sm, -2, axis=1)[:, -2:]
        rel = (part[:, 1] - part[:, 0]) / (np.abs(part[:, 1]) + np.abs(part[:, 0]) + 1e-30)
        m = rel > 1e-5
        assert (lab_tc[b][m] == ref[m]).all(), f"block {b}: {(lab_tc[b][m] != ref[m]).sum()} tensor-core mismatches"
        assert (lab_ex[b][m] == ref[m]).all()
        assert (lab_tc[b] == ref).mean() > 0.999


@pytest.mark.parametrize("metric", [0, 1])
@pytest.mark.parametrize("bs,K,n,nblk", [(4, 300, 1000, 3), (8, 256, 768, 5), (16, 4096, 2048, 2),
                                          (6, 1000, 777, 2), (12, 129, 513, 2), (8, 4096, 4096, 2)])
def test_assign_matches_oracle(metric, bs, K, n, nblk):
    _check_assign(metric, bs, K, n, nblk, seed=bs * 1000 + K + metric)


@pytest.mark.parametrize("metric,bs,K", [(1, 4, 1000), (0, 4, 700), (0, 8, 500), (1, 16, 300)])
def test_assign_many_units_per_cta(metric, bs, K):
    """More 256-point work units than two per SM, two problems: every persistent
    CTA runs several units and crosses from one problem to the next, so the
    per-unit point reload (into tensor memory for packed widths <= 16, into
    shared memory otherwise) and the centroid-ring hand-over between units are
    exercised; K is not a multiple of either tile width."""
    from skcq_b200 import _engine

    n, nblk = 40000, 2
    units = nblk * _engine.round_up(n, _engine.ROWS_PER_UNIT) // _engine.ROWS_PER_UNIT
    assert units > 2 * torch.cuda.get_device_properties(0).multi_processor_count
    _check_assign(metric, bs, K, n, nblk, seed=7 * K + bs + metric)


def _kmeans_case(name):
    g = sub(load_golden("kmeans"), name + "__")
    n, d, k, iters, is_cos = (int(v) for v in g["meta"])
    return g, n, d, k, iters, is_cos


@pytest.mark.parametrize("name", ["cos_a", "cos_empty", "l2_a", "l2_empty"])
def test_kmeans_experiment_matches_reference(name, monkeypatch):
    from skcq_b200.codebook import KmeansConfig, KmeansExperiment
    from skcq_b200.codebook.events import KmeansDoneEvent, KmeansIterEvent

    g, n, d, k, iters, is_cos = _kmeans_case(name)
    monkeypatch.setattr(torch, "randperm", PermReplay.from_case(g).torch_patch())
    data = torch.from_numpy(g["data"]).cuda()
    exp = KmeansExperiment(KmeansConfig(metric="cosine" if is_cos else "euclidean", k=k, max_iters=iters,
                                        device=torch.device("cuda"), name=name, chunk_size=64,
                                        raw_data=data if is_cos else None))
    its, done = [], []
    exp.on(KmeansIterEvent, its.append)
    exp.on(KmeansDoneEvent, done.append)
    cent, labels = exp.fit(data)
    # oracle on the same inputs decides whether the trajectory is tie-free
    if is_cos:
        _, _, log = ok.fit_cosine(g["data"], g["data"], k, iters, sobol_np(min(k, n), d))
    else:
        _, _, log = ok.fit_euclidean(g["data"], k, iters, PermReplay.from_case(g)(n))
    ev = g["ev_int"]
    if log.min_margin <= 1e-5:  # trajectory passes a near-tie: only quality must agree
        assert abs(done[0].iters_run - ev[ev[:, 0] == 2][0][1]) <= 3
        return
    assert [e.n_empty for e in its] == list(ev[ev[:, 0] == 1][:, 2])
    assert done[0].iters_run == ev[ev[:, 0] == 2][0][1]
    assert rel_err(cent.cpu().numpy(), g["centroids"]) < 1e-5
    assert (labels.cpu().numpy() == g["labels"]).all()


CODEC_CASES = ["base", "single", "ssvq", "noncomm", "asym", "shared", "int8cb", "skipz", "ressign", "rem13"]
# cases of test_aqlm_fit_matches_reference that passed through a near-tie and
# were held only to the quality tolerance (reported by the test after them)
LOOSE_CASES: list[str] = []


def _product_aqlm(name):
    from skcq_b200 import codebook as cb

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
    prim = cb.SphericalCodebook(cb.SphericalCodebookConfig(block_size=bs, K=k_list[0], shared=kw.get("shared", False),
                                                           max_iters=10, norm_threshold=thr,
                                                           skip_zeros=kw.get("skip_zeros", False)))
    if kw.get("sign_split"):
        prim = cb.SSVQCodebook(prim)
    res = []
    for kc in k_list[1:]:
        r = cb.EuclideanCodebook(cb.EuclideanCodebookConfig(block_size=kw.get("rbs") or bs, K=kc,
                                                            shared=kw.get("shared", False), max_iters=10,
                                                            norm_threshold=thr, skip_zeros=False))
        if kw.get("res_sign_split"):
            r = cb.SSVQCodebook(r)
        res.append(r)
    return cb.AQLMCodebook(prim, res, cb.AQLMCodebookConfig(norm_threshold=thr,
                                                            codebook_bits=kw.get("codebook_bits", 16)))


@pytest.mark.parametrize("name", CODEC_CASES)
def test_aqlm_fit_matches_reference(name, monkeypatch):
    import test_oracle_golden as T

    g = sub(load_golden("codecs"), name + "__")
    prim, res, bits, thr = T._spec(name, int(g["meta"][2]))
    primary, residuals, ocwr = oc.aqlm_fit(prim, res, g["w"], sobol_np, PermReplay.from_case(g),
                                           codebook_bits=bits, norm_threshold=thr)
    logs = [lg for c in [primary, *residuals] for lg in T.codec_logs(c)]
    monkeypatch.setattr(torch, "randperm", PermReplay.from_case(g).torch_patch())
    aqlm = _product_aqlm(name)
    w = torch.from_numpy(g["w"]).cuda()
    cwr = aqlm.fit(w)
    recon = aqlm.reconstruct(cwr).cpu().numpy()
    wn = g["w"].astype(np.float64)
    e_ref = np.linalg.norm(wn - g["recon"]) / np.linalg.norm(wn)
    e_gpu = np.linalg.norm(wn - recon) / np.linalg.norm(wn)
    if not all(lg.min_margin > TIE for lg in logs):
        # the reference's own trajectory passes a near-tie: its result depends
        # on rounding order, so only the quality is compared
        LOOSE_CASES.append(name)
        assert abs(e_gpu - e_ref) <= 0.15 * e_ref
        return
    assert abs(e_gpu - e_ref) <= 1e-3 * e_ref + 1e-7
    assert rel_err(recon, g["recon"]) < 2e-3


def test_loose_branch_count():
    """At most two of the ten reference configurations pass a near-tie (the
    oracle's logs decide, not the GPU result); the rest were held to 1e-3."""
    print(f"codec cases on the near-tie branch: {len(LOOSE_CASES)} of {len(CODEC_CASES)} {sorted(LOOSE_CASES)}")
    assert len(LOOSE_CASES) <= 2, sorted(LOOSE_CASES)


def test_config1_matches_reference(monkeypatch):
    """W 768x2048 bf16; SSVQ spherical bs=8 K=256 + euclidean bs=4 K=256, 20 iterations."""
    from skcq_b200 import codebook as cb
    from skcq_b200.codebook.events import KmeansDoneEvent

    g = load_golden("config1")
    monkeypatch.setattr(torch, "randperm", PermReplay.from_case(g).torch_patch())
    w = torch.from_numpy(bf16_from_bits(g["w_bf16"]).reshape(768, 2048)).to(torch.bfloat16).cuda()
    primary = cb.SSVQCodebook(cb.SphericalCodebook(cb.SphericalCodebookConfig(block_size=8, K=256, max_iters=20)))
    residual = cb.EuclideanCodebook(cb.EuclideanCodebookConfig(block_size=4, K=256, max_iters=20, skip_zeros=False))
    aqlm = cb.AQLMCodebook(primary, [residual], cb.AQLMCodebookConfig())
    done = []
    aqlm.on(KmeansDoneEvent, done.append)
    cwr = aqlm.fit(w)
    recon = aqlm.reconstruct(cwr).cpu().numpy()
    wf = w.float().cpu().numpy()
    rel = float(np.linalg.norm(wf - recon) / np.linalg.norm(wf))
    assert abs(rel - g["rel_fro_err"][0]) < 1e-3 * g["rel_fro_err"][0], (rel, g["rel_fro_err"][0])
    assert (cwr.primary.inner.idxs.cpu().numpy() == g["c0_idxs"]).mean() > 0.99
    assert (cwr.residuals[0].idxs.cpu().numpy() == g["c1_idxs"]).mean() > 0.95
    assert rel_err(recon[::37], g["recon_rows"]) < 5e-3
    ev = g["ev_int"]
    ref_iters = ev[ev[:, 0] == 2][:, 1]
    assert len(done) == len(ref_iters)
    assert (np.array([d.iters_run for d in done]) == ref_iters).mean() > 0.95


def test_reconstruct_bit_exact_vs_oracle(monkeypatch):
    """Decode is deterministic single-rounding arithmetic: identical payloads
    decode to identical bits (aqlm.py:137-141)."""
    g = sub(load_golden("codecs"), "ressign__")
    monkeypatch.setattr(torch, "randperm", PermReplay.from_case(g).torch_patch())
    aqlm = _product_aqlm("ressign")
    cwr = aqlm.fit(torch.from_numpy(g["w"]).cuda())
    recon = aqlm.reconstruct(cwr).cpu().numpy()
    # oracle decode of the product's own payload
    p = oc.Codec("spherical", oc.SphericalCfg(4, 16), centroids=aqlm.primary.directions.float().cpu().numpy())
    parts = [oc.spherical_reconstruct(p, {"idxs": cwr.primary.idxs.cpu().numpy(),
                                          "scales": cwr.primary.scales.cpu().numpy(), "remainder": None})]
    for r, rc in zip(aqlm.residuals, cwr.residuals, strict=True):
        inner = oc.Codec("euclidean", oc.EuclideanCfg(4, r.inner.K), centroids=r.inner.centroids.float().cpu().numpy())
        x = oc.euclidean_reconstruct(inner, {"idxs": rc.inner.idxs.cpu().numpy(), "remainder": None})
        parts.append(x * rc.signs.cpu().numpy().astype(np.float32))
    ref = parts[0]
    for x in parts[1:]:
        ref = ref + x
    assert np.array_equal(recon, ref)


def _realistic_problem(metric: int, nblk: int, n: int, bs: int, K: int, seed: int):
    """Student-t(5) block rows at std 0.02 (the benchmark layer's distribution);
    centroids are K of the problem's own points (Forgy-style, as k-means
    starts and stays near), slightly perturbed, so top-2 margins are as small
    as a real fit makes them."""
    from skcq_b200 import _engine

    g = torch.Generator().manual_seed(seed)
    z = torch.randn(n, nblk * bs, generator=g)
    chi2 = torch.randn(5, n, nblk * bs, generator=g).square().sum(0)
    w = z / torch.sqrt(chi2 / 5.0) * (0.02 / (5.0 / 3.0) ** 0.5)
    pts = _engine.gather_block_points(w.cuda(), bs, nblk, False, 0.0, False, metric)
    C = torch.empty(nblk, K, bs)
    for b in range(nblk):
        idx = torch.randperm(n, generator=g)[:K]
        C[b] = w[idx, b * bs:(b + 1) * bs] * (1.0 + 0.01 * torch.randn(K, bs, generator=g))
    if metric == _engine.COSINE:
        C = torch.nn.functional.normalize(C, dim=-1)
    return w, pts, C


def _oracle_check_rows(metric, x, c, lab, rows):
    """(mismatches above the 1e-5 relative margin, rows below it) for the
    sampled rows, against the oracle's fp32 scores."""
    xs = x[rows]
    if metric == 0:
        s = ok.scores_cosine(ok.normalize_rows(xs), c.T)
        ref, sm = s.argmax(1), s
    else:
        s = ok.scores_l2(xs, c.T)
        ref, sm = s.argmin(1), -s
    part = np.partition(sm, -2, axis=1)[:, -2:]
    rel = (part[:, 1] - part[:, 0]) / (np.abs(part[:, 1]) + np.abs(part[:, 0]) + 1e-30)
    m = rel > 1e-5
    return int((lab[rows][m] != ref[m]).sum()), int((~m).sum())


@pytest.mark.parametrize("metric,bs,K,nblk", [
    (1, 4, 65536, 2),   # second residual of the benchmark layer
    (0, 8, 4096, 2),    # its primary
    (1, 16, 4096, 2),   # its first residual
    (0, 12, 65536, 1),  # full-model primary (non-dividing block size 12)
    (1, 6, 16384, 2),   # full-model residual
])
def test_assign_bench_shapes_match_oracle(metric, bs, K, nblk):
    """The benchmark's assignment shapes at 98,304 points per problem: labels
    bit-exact against the oracle on 2,048 sampled rows per problem wherever
    the relative top-2 margin exceeds 1e-5 (rows below it are counted)."""
    n = 98304
    w, pts, C = _realistic_problem(metric, nblk, n, bs, K, seed=bs * 131 + K + metric)
    lab = _labels(pts, C, exact=False)
    rng = np.random.default_rng(K + bs)
    near_ties = 0
    for b in range(nblk):
        rows = np.sort(rng.choice(n, 2048, replace=False))
        x = w[:, b * bs:(b + 1) * bs].numpy()
        bad, ties = _oracle_check_rows(metric, x, C[b].numpy(), lab[b], rows)
        near_ties += ties
        assert bad == 0, f"block {b}: {bad} labels differ above the margin"
    print(f"metric={metric} bs={bs} K={K}: {near_ties} of {2048 * nblk} sampled rows below the 1e-5 margin")


def test_config1_assign_on_reference_centroids():
    """Config 1 (768 x 2048, SSVQ spherical bs=8 K=256 + euclidean bs=4 K=256):
    for 16 primary and 16 residual blocks the reference's k-means input and
    final fp32 centroids are replayed through the GPU assignment; labels equal
    the reference's own final labels wherever the relative top-2 margin
    exceeds 1e-5."""
    from skcq_b200 import _engine

    g = load_golden("config1")
    for tag, metric in (("c0", _engine.COSINE), ("c1", _engine.L2)):
        data, cent, ref_lab = g[f"{tag}_fit_data"], g[f"{tag}_fit_cent"], g[f"{tag}_fit_labels"].astype(np.int64)
        nblk, n, bs = data.shape
        w = torch.from_numpy(np.ascontiguousarray(data.transpose(1, 0, 2).reshape(n, nblk * bs)))
        pts = _engine.gather_block_points(w.cuda(), bs, nblk, False, 0.0, False, metric)
        lab = _labels(pts, torch.from_numpy(cent), exact=False)
        total_ties = 0
        for b in range(nblk):
            x, c = data[b], cent[b]
            if metric == _engine.COSINE:
                s = ok.scores_cosine(ok.normalize_rows(x), c.T)
                sm = s
            else:
                s = ok.scores_l2(x, c.T)
                sm = -s
            part = np.partition(sm, -2, axis=1)[:, -2:]
            rel = (part[:, 1] - part[:, 0]) / (np.abs(part[:, 1]) + np.abs(part[:, 0]) + 1e-30)
            m = rel > 1e-5
            total_ties += int((~m).sum())
            assert (lab[b][m] == ref_lab[b][m]).all(), (tag, b, int((lab[b][m] != ref_lab[b][m]).sum()))
        print(f"config1 {tag}: {total_ties} of {nblk * n} rows below the 1e-5 margin")


def test_quantize_spherical_scales_matches_oracle():
    """int<N> scale quantisation (spherical.py:45-71) on the GPU equals the
    oracle bit for bit: the same q_scale and the same rounded levels, for the
    fitted scales of a reference case and for signed random scales with
    zeros, at 4, 8 and 16 bits."""
    import test_oracle_golden as T
    from skcq_b200 import _engine

    g = sub(load_golden("codecs"), "sq8__")
    prim, res, _, _ = T._spec("base", 1)
    primary, _, cwr = oc.aqlm_fit(prim, res, g["w"], sobol_np, PermReplay.from_case(g), norm_threshold=1e-9)
    fitted = cwr["primary"]["scales"].astype(np.float32)
    rnd = np.random.default_rng(5).standard_normal((300, 70)).astype(np.float32) * 0.03
    rnd[::7] = 0.0
    for scales in (fitted, rnd):
        for bits in (4, 8, 16):
            oc_cwr = {"scales": scales.copy()}
            codec = oc.Codec("spherical", oc.SphericalCfg(4, 16))
            oc.quantize_scales(oc_cwr, codec, f"int{bits}")
            q, q_scale = _engine.quantize_scales_int(torch.from_numpy(scales).cuda(), bits)
            assert float(q_scale) == codec.q_scale
            assert np.array_equal(q.cpu().numpy(), oc_cwr["scales"])
