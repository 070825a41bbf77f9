"""Generate golden vectors by running the SKCQ reference itself (CPU torch).

Run in a container where the reference source tree is present:

    python tests/golden/make_golden.py --ref <path of the reference checkout>

(or set SKCQ_REFERENCE to that path).

Writes ``tests/golden/*.npz``. Each case records the inputs, the random draws
the reference consumed (every ``torch.randperm`` call, captured in order) and
the reference outputs, so the oracle and the CUDA path can be replayed on
exactly the same initial centroids. The reference is never needed at test
time; only these fixtures are.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


class RandpermRecorder:
    """Wrap ``torch.randperm`` and keep every permutation it returns."""

    def __init__(self) -> None:
        self.perms: list[np.ndarray] = []
        self._orig = torch.randperm

    def __enter__(self):
        def rec(*a, **kw):
            p = self._orig(*a, **kw)
            self.perms.append(p.cpu().numpy().astype(np.int32))
            return p

        torch.randperm = rec
        return self

    def __exit__(self, *exc):
        torch.randperm = self._orig


def pack_perms(perms: list[np.ndarray]) -> dict:
    lens = np.array([len(p) for p in perms], dtype=np.int64)
    flat = np.concatenate(perms) if perms else np.zeros(0, np.int32)
    return {"perm_lens": lens, "perm_flat": flat}


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy()


class EventLog:
    def __init__(self, exp, events_mod) -> None:
        self.rows: list[tuple] = []
        ev = events_mod
        exp.on(ev.KmeansStartEvent, lambda e: self.rows.append((0, e.k, e.n_points, e.block_idx, e.n_blocks, 0.0)))
        exp.on(ev.KmeansIterEvent, lambda e: self.rows.append((1, e.iter, e.n_empty, 0, 0, e.moved)))
        exp.on(ev.KmeansDoneEvent, lambda e: self.rows.append((2, e.iters_run, int(e.converged), 0, 0, e.final_moved)))

    def arrays(self) -> dict:
        a = np.array(self.rows, dtype=np.float64).reshape(-1, 6)
        return {"ev_int": a[:, :5].astype(np.int64), "ev_moved": a[:, 5]}


def case_assign(out: Path, km) -> None:
    g = torch.Generator().manual_seed(101)
    data = torch.nn.functional.normalize(torch.randn(600, 8, generator=g), dim=-1)
    cent = torch.nn.functional.normalize(torch.randn(96, 8, generator=g), dim=-1)
    lab_cos = km.assign_cosine(data, cent.t().contiguous(), 128, torch.device("cpu"))
    x = torch.randn(600, 4, generator=g) * 0.01
    c = torch.randn(200, 4, generator=g) * 0.01
    lab_l2 = km.assign_l2(x, c.t().contiguous(), 128, torch.device("cpu"))
    np.savez_compressed(
        out / "assign.npz",
        cos_data=data.numpy(), cos_cent=cent.numpy(), cos_labels=lab_cos.numpy(),
        l2_data=x.numpy(), l2_cent=c.numpy(), l2_labels=lab_l2.numpy(),
    )


def case_kmeans(out: Path, km, events) -> None:
    res = {}
    specs = [
        ("cos_a", "cosine", 400, 8, 32, 15, 7),
        ("cos_empty", "cosine", 60, 4, 48, 12, 8),
        ("l2_a", "euclidean", 400, 4, 32, 15, 9),
        ("l2_empty", "euclidean", 200, 2, 80, 12, 27),
    ]
    for name, metric, n, d, k, iters, seed in specs:
        torch.manual_seed(seed)
        if not name.endswith("empty"):
            data = torch.randn(n, d) * 0.05
        else:
            # a few tight clusters with small noise: many empty clusters, no exact ties
            nc, noise = (3, 0.004) if metric == "cosine" else (5, 0.01)
            centers = torch.randn(nc, d) * 0.05
            data = centers[torch.arange(n) % nc] + noise * torch.randn(n, d)
        exp = km.KmeansExperiment(km.KmeansConfig(
            metric=metric, k=k, max_iters=iters, device=torch.device("cpu"), name=name,
            chunk_size=64, raw_data=data if metric == "cosine" else None,
        ))
        log = EventLog(exp, events)
        with RandpermRecorder() as rec:
            cent, labels = exp.fit(data)
        arrs = {"data": data.numpy(), "centroids": cent.numpy(), "labels": labels.numpy(),
                "meta": np.array([n, d, k, iters, 1 if metric == "cosine" else 0]), **log.arrays(),
                **pack_perms(rec.perms)}
        for kk, v in arrs.items():
            res[f"{name}__{kk}"] = v
    np.savez_compressed(out / "kmeans.npz", **res)


def _aqlm_small(cb, block_size=4, k_list=(16, 16), shared=False, sign_split=False, rbs=None,
                norm_threshold=1e-9, skip_zeros=False, codebook_bits=16, res_sign_split=False):
    primary = cb.SphericalCodebook(cb.SphericalCodebookConfig(
        block_size=block_size, K=k_list[0], shared=shared, max_iters=10,
        norm_threshold=norm_threshold, skip_zeros=skip_zeros))
    if sign_split:
        primary = cb.SSVQCodebook(primary)
    residuals = []
    for kc in k_list[1:]:
        r = cb.EuclideanCodebook(cb.EuclideanCodebookConfig(
            block_size=rbs or block_size, K=kc, shared=shared, max_iters=10,
            norm_threshold=norm_threshold, skip_zeros=False))
        if res_sign_split:
            r = cb.SSVQCodebook(r)
        residuals.append(r)
    return cb.AQLMCodebook(primary, residuals, cb.AQLMCodebookConfig(
        norm_threshold=norm_threshold, codebook_bits=codebook_bits))


def _dump_codec(prefix: str, codec, cwr, res: dict) -> None:
    from skcq.codebook import SSVQCodebook
    if isinstance(codec, SSVQCodebook):
        res[f"{prefix}signs"] = cwr.signs.numpy()
        codec, cwr = codec.inner, cwr.inner
    res[f"{prefix}idxs"] = cwr.idxs.numpy()
    res[f"{prefix}cent_bf16"] = bf16_bits(codec.centroids_tensor)
    if hasattr(cwr, "scales"):
        res[f"{prefix}scales"] = cwr.scales.float().numpy()
    if cwr.remainder is not None:
        res[f"{prefix}rem_bf16"] = bf16_bits(cwr.remainder)


def case_codecs(out: Path, cb, experts_mod) -> None:
    """The reference unit-test configurations (tests/test_codebook.py) + forwards."""
    res = {}
    specs = [
        # name, seed, rows, in_dim, scale, kwargs
        ("base", 1, 32, 12, 0.1, {}),
        ("single", 2, 32, 12, 0.1, {"k_list": (16,)}),
        ("ssvq", 3, 32, 12, 0.3, {"sign_split": True}),
        ("noncomm", 5, 32, 34, 0.1, {"block_size": 10, "rbs": 12}),
        ("asym", 13, 32, 12, 0.1, {"k_list": (16, 8)}),
        ("shared", 6, 64, 12, 0.3, {"shared": True}),
        ("int8cb", 21, 48, 16, 0.2, {"k_list": (16, 8), "codebook_bits": 8}),
        ("skipz", 22, 32, 12, 0.1, {"norm_threshold": 1e-5, "skip_zeros": True}),
        ("ressign", 23, 32, 12, 0.2, {"res_sign_split": True, "k_list": (16, 16, 8)}),
        ("rem13", 24, 8, 13, 0.1, {"k_list": (16,)}),
    ]
    for name, seed, rows, in_dim, scale, kw in specs:
        torch.manual_seed(seed)
        w = torch.randn(rows, in_dim) * scale
        if name == "skipz":
            w[0] = 0
            w[5, 4:8] = 0
        aqlm = _aqlm_small(cb, **kw)
        with RandpermRecorder() as rec:
            cwr = aqlm.fit(w)
        recon = aqlm.reconstruct(cwr)
        p = f"{name}__"
        res[p + "w"] = w.numpy()
        res[p + "recon"] = recon.numpy()
        res[p + "meta"] = np.array([rows, in_dim, len(aqlm.residuals)])
        for kk, v in pack_perms(rec.perms).items():
            res[p + kk] = v
        _dump_codec(p + "c0_", aqlm.primary, cwr.primary, res)
        for i, (r, rc) in enumerate(zip(aqlm.residuals, cwr.residuals, strict=True)):
            _dump_codec(p + f"c{i + 1}_", r, rc, res)
        if name in ("base", "ssvq", "asym", "noncomm", "single"):
            out_dim = 8
            mod = experts_mod.CodebookModule.from_cwr(aqlm, cwr, out_dim=out_dim).to(torch.float32)
            g = torch.Generator().manual_seed(seed + 100)
            hidden = torch.randn(5, in_dim, generator=g)
            res[p + "hidden"] = hidden.numpy()
            res[p + "fwd"] = np.stack([mod(hidden, expert_idx=e).detach().numpy() for e in range(rows // out_dim)])
    # int8 scale quantisation (tests/test_codebook.py:352-365)
    torch.manual_seed(15)
    w = torch.randn(32, 12) * 0.3
    aqlm = _aqlm_small(cb)
    with RandpermRecorder() as rec:
        cwr = aqlm.fit(w)
    cb.quantize_spherical_scales(cwr.primary, aqlm.primary, "int8")
    res["sq8__w"] = w.numpy()
    res["sq8__scales_q"] = cwr.primary.scales.numpy()
    res["sq8__q_scale"] = np.array([float(aqlm.primary.scale_quant.q_scale)])
    res["sq8__recon"] = aqlm.reconstruct(cwr).numpy()
    for kk, v in pack_perms(rec.perms).items():
        res["sq8__" + kk] = v
    np.savez_compressed(out / "codecs.npz", **res)


def case_experts(out: Path, cb, experts_mod) -> None:
    """CodebookExperts.forward on a tiny MoE (4 experts, hidden 12, inter 8, top-2)."""
    torch.manual_seed(31)
    E, H, I = 4, 12, 8
    wg = torch.randn(E * I, H) * 0.2
    wu = torch.randn(E * I, H) * 0.2
    wd = torch.randn(E * H, I) * 0.2
    res = {"wg": wg.numpy(), "wu": wu.numpy(), "wd": wd.numpy()}
    mods = []
    perms = []
    for name, w, out_dim, bs in (("g", wg, I, 4), ("u", wu, I, 4), ("d", wd, H, 4)):
        aqlm = _aqlm_small(cb, block_size=bs, k_list=(16, 8))
        with RandpermRecorder() as rec:
            cwr = aqlm.fit(w)
        perms += rec.perms
        mods.append(experts_mod.CodebookModule.from_cwr(aqlm, cwr, out_dim=out_dim).to(torch.float32))
        _dump_codec(f"{name}_c0_", aqlm.primary, cwr.primary, res)
        _dump_codec(f"{name}_c1_", aqlm.residuals[0], cwr.residuals[0], res)
    ex = experts_mod.CodebookExperts(mods[0], mods[1], mods[2], E, torch.nn.functional.silu)
    g = torch.Generator().manual_seed(77)
    hidden = torch.randn(6, H, generator=g)
    logits = torch.randn(6, E, generator=g)
    topw, topi = torch.topk(torch.softmax(logits, -1), 2, dim=-1)
    topw = topw / topw.sum(-1, keepdim=True)
    y = ex(hidden, topi, topw)
    res.update({"hidden": hidden.numpy(), "topi": topi.numpy(), "topw": topw.numpy(), "y": y.detach().numpy()})
    res.update(pack_perms(perms))
    np.savez_compressed(out / "experts.npz", **res)


def case_config1(out: Path, cb, bpw_mod) -> None:
    """The CPU-runnable single expert matrix: W 768x2048 bf16, N(0, 0.02^2) times a
    per-row lognormal(0, 0.3) scale, seed 0; SSVQ spherical bs=8 K=256 + euclidean
    bs=4 K=256, 20 iterations."""
    torch.manual_seed(0)
    w = (torch.randn(768, 2048) * 0.02 * torch.exp(0.3 * torch.randn(768, 1))).to(torch.bfloat16)
    primary = cb.SSVQCodebook(cb.SphericalCodebook(cb.SphericalCodebookConfig(block_size=8, K=256, max_iters=20)))
    residual = cb.EuclideanCodebook(cb.EuclideanCodebookConfig(block_size=4, K=256, max_iters=20, skip_zeros=False))
    aqlm = cb.AQLMCodebook(primary, [residual], cb.AQLMCodebookConfig())
    log = EventLog(aqlm, __import__("skcq.codebook.events", fromlist=["x"]))
    # every 16th primary block and every 32nd residual block: the k-means input
    # and the reference's final fp32 centroids and labels, so the GPU
    # assignment can be checked against the reference on its own centroids
    km_cls = __import__("skcq.codebook.kmeans", fromlist=["x"]).KmeansExperiment
    orig_fit = km_cls.fit
    fits: list[tuple] = []

    def recording_fit(self, data):
        c, lab = orig_fit(self, data)
        fits.append((data.detach().clone(), c.detach().clone(), lab.detach().clone()))
        return c, lab

    km_cls.fit = recording_fit
    try:
        with RandpermRecorder() as rec:
            cwr = aqlm.fit(w)
    finally:
        km_cls.fit = orig_fit
    recon = aqlm.reconstruct(cwr)
    wf = w.float()
    rel = ((wf - recon).norm() / wf.norm()).item()
    bpw = bpw_mod.bits_per_weight_kmeans(n_rows=768, in_dim=2048, n_blocks=256, block_size=8, n_codebooks=2,
                                         k_per_codebook=[256, 256], shared_codebook=False, sign_split=True,
                                         scale_bits_per_elem=16, bs_per_codebook=[8, 4])
    res = {"w_bf16": bf16_bits(w), "rel_fro_err": np.array([rel]), "bpw": np.array([bpw]),
           "recon_rows": recon[::37].numpy(), "recon_sum": np.array([recon.double().sum().item()]),
           "recon_abs_sum": np.array([recon.double().abs().sum().item()]), **log.arrays(),
           **pack_perms(rec.perms)}
    res["c0_idxs"] = cwr.primary.inner.idxs.numpy().astype(np.uint8)
    res["c0_scales"] = cwr.primary.inner.scales.numpy()
    res["c0_signs_packed"] = np.packbits(cwr.primary.signs.numpy() > 0, axis=1)
    res["c0_cent_bf16"] = bf16_bits(aqlm.primary.centroids_tensor)
    res["c1_idxs"] = cwr.residuals[0].idxs.numpy().astype(np.uint8)
    res["c1_cent_bf16"] = bf16_bits(aqlm.residuals[0].centroids_tensor)
    assert len(fits) == 256 + 512
    for tag, first, step, count in (("c0", 0, 16, 16), ("c1", 256, 32, 16)):
        pick = [fits[first + i * step] for i in range(count)]
        res[f"{tag}_fit_blocks"] = np.arange(count, dtype=np.int64) * step
        res[f"{tag}_fit_data"] = np.stack([f[0].numpy() for f in pick]).astype(np.float32)
        res[f"{tag}_fit_cent"] = np.stack([f[1].numpy() for f in pick]).astype(np.float32)
        res[f"{tag}_fit_labels"] = np.stack([f[2].numpy() for f in pick]).astype(np.int16)
    np.savez_compressed(out / "config1.npz", **res)
    print(f"config1: rel_fro_err={rel:.5f} bpw={bpw:.3f}")


VQ_SPECS = [
    # name, projection, block_size, K, n_codebooks, metric, residual_k, residual_sign_split, shared, sign_split,
    # max_iters, scale_dtype, residual_block_sizes, codebook_bits
    ("cos_int8", "gate", 4, 16, 2, "cosine", 8, None, False, True, 8, "int8", None, 8),
    ("euc_shared", "down", 4, 16, 2, "euclidean", 8, True, True, False, 8, "bf16", 6, 16),
]


def case_vq(out: Path, vq_experiment, vq_runner) -> None:
    """The sweep runner (skcq/vq/experiment.py VQRunExperiment.fit) on two small
    configurations, and the integer / fp8 baselines (skcq/vq/runner.py)."""
    res = {}
    torch.manual_seed(41)
    w = torch.randn(64, 40) * 0.05
    res["int_w"] = w.numpy()
    for name, fn in vq_runner.integer_schemes(8):
        recon, bpw = fn(w.clone())
        res[f"int__{name}__recon"] = recon.float().numpy()
        res[f"int__{name}__bpw"] = np.array([bpw])
    for (name, proj, bs, K, ncb, metric, rk, rss, shared, ss, iters, sdt, rbs, cbits) in VQ_SPECS:
        torch.manual_seed(43)
        E, H, I = 4, 16, 8
        rows, in_dim = (E * I, H) if proj != "down" else (E * H, I + 6)
        w = torch.randn(rows, in_dim) * 0.1
        cfg = vq_experiment.VQRunConfig(
            projection=proj, in_dim=in_dim, num_experts=E, hidden_size=H, intermediate_size=I, block_size=bs, K=K,
            n_codebooks=ncb, metric=metric, residual_k=rk, residual_sign_split=rss, shared_codebook=shared,
            sign_split=ss, max_iters=iters, scale_dtype=sdt, residual_block_sizes=rbs, codebook_bits=cbits,
            layer_idx=3, device=torch.device("cpu"), chunk_budget_mb=64)
        with RandpermRecorder() as rec:
            row = vq_experiment.VQRunExperiment(cfg).fit(w)
        res[f"vq__{name}__w"] = w.numpy()
        res[f"vq__{name}__err"] = np.array([row["rel_fro_err"]])
        res[f"vq__{name}__bpw"] = np.array([row["bits_per_weight"]])
        res[f"vq__{name}__scheme"] = np.array([row["scheme"]])
        res[f"vq__{name}__rbs"] = np.array(row["residual_block_sizes"], dtype=np.int64)
        for kk, v in pack_perms(rec.perms).items():
            res[f"vq__{name}__{kk}"] = v
        print(f"vq {name}: {row['scheme']} err={row['rel_fro_err']:.5f} bpw={row['bits_per_weight']:.3f}")
    np.savez_compressed(out / "vq.npz", **res)


# (layer, tokens) per MoE call; layer 0 is called twice, layer 3 only in the base capture
METRIC_CALLS = [(0, 40), (1, 40), (0, 24), (2, 64), (3, 16)]


def case_metrics(out: Path, metrics, eval_model) -> None:
    """Routing agreement, KLD, token log-likelihoods and sliding-window perplexity
    (skcq/metrics.py, skcq/eval_model.py) on seeded synthetic captures and a tiny
    deterministic language model (tests/_helpers.py: TinyLM, CharTokenizer)."""
    sys.path.insert(0, str(HERE.parent))
    from _helpers import CharTokenizer, TinyLM, perturb_routing, routing_calls

    def capture(calls):
        cap = metrics.RoutingCapture()
        for layer, ids, w in calls:
            cap.layer_index.append(layer)
            cap.top_k_index.append(ids)
            cap.top_k_weights.append(w)
        return cap

    res = {}
    # pair a: with weights, layer 3 missing from the quantized capture
    base = routing_calls(51, METRIC_CALLS)
    quant = perturb_routing(base[:-1], 52)
    # pair b: no weights, layer 1 with a different token count (skipped)
    base_b = routing_calls(53, METRIC_CALLS[:4], weights=False)
    quant_b = perturb_routing(base_b, 54)
    quant_b[1] = (1, quant_b[1][1][:30], quant_b[1][2])
    for tag, (bc, qc) in {"a": (base, quant), "b": (base_b, quant_b)}.items():
        summ = metrics.routing_agreement(capture(bc), capture(qc))
        for side, calls in (("base", bc), ("quant", qc)):
            res[f"rt_{tag}__{side}__layers"] = np.array([c[0] for c in calls], dtype=np.int64)
            for i, (_, ids, w) in enumerate(calls):
                res[f"rt_{tag}__{side}__idx{i}"] = ids.numpy()
                res[f"rt_{tag}__{side}__w{i}"] = w.numpy()
        for key in ("common_layers", "total_tokens", "set_agreement", "weight_cosine", "routing_jsd"):
            res[f"rt_{tag}__{key}"] = np.array([summ[key]], dtype=np.float64)
        res[f"rt_{tag}__per_layer"] = np.array([[d["layer"], d["tokens"], d["set_agreement"]]
                                                for d in summ["per_layer"]], dtype=np.float64)
        print(f"routing {tag}: {summ['set_agreement']:.4f} cos {summ['weight_cosine']:.6f} jsd {summ['routing_jsd']:.6f}")

    rs = np.random.RandomState(7)
    text = "".join(rs.choice(list("abcdefghij klmnop"), size=300))
    tok = CharTokenizer()
    model, model_q = TinyLM(seed=5), TinyLM(seed=5, noise=0.05)
    ids = tok(text).input_ids
    ref_logits = metrics.capture_reference_logits(model, ids, max_length=64)
    res["lm_text"] = np.array([text])
    res["lm_ref_logits"] = ref_logits.numpy()
    res["lm_kld"] = np.array([metrics.kld_against_reference(model_q, ids, ref_logits)])
    res["lm_tll"] = metrics.token_log_likelihoods(model_q, ids[:, :80]).numpy()
    res["lm_ppl"] = np.array([eval_model.compute_perplexity(model_q, tok, text, max_length=48, stride=16)])
    res["lm_ppl_base"] = np.array([eval_model.compute_perplexity(model, tok, text, max_length=48, stride=16)])
    print(f"lm: kld {res['lm_kld'][0]:.6f} ppl {res['lm_ppl'][0]:.4f} base {res['lm_ppl_base'][0]:.4f}")
    np.savez_compressed(out / "metrics.npz", **res)


def fake_moe(n_layers: int = 1, E: int = 4, H: int = 12, I: int = 8, seed: int = 0):
    """A Hugging-Face-layout MoE holding only what the build driver reads:
    config.text_config sizes and model.language_model.layers[i].mlp.experts
    with gate_up_proj (E, 2I, H) and down_proj (E, H, I)."""
    import types

    g = torch.Generator().manual_seed(seed)
    layers = []
    for _ in range(n_layers):
        experts = types.SimpleNamespace(gate_up_proj=torch.nn.Parameter(torch.randn(E, 2 * I, H, generator=g) * 0.1),
                                        down_proj=torch.nn.Parameter(torch.randn(E, H, I, generator=g) * 0.1))
        layers.append(types.SimpleNamespace(mlp=types.SimpleNamespace(experts=experts)))
    text = types.SimpleNamespace(layers=layers)
    cfg = types.SimpleNamespace(text_config=types.SimpleNamespace(moe_intermediate_size=I, hidden_size=H,
                                                                  num_experts=E))
    return types.SimpleNamespace(config=cfg, model=types.SimpleNamespace(language_model=text))


def case_extract(out: Path, quantize_mod, config_mod) -> None:
    """The build driver (skcq/quantize.py extract_and_build_codebooks) over a
    one-layer MoE of 4 experts (hidden 12, intermediate 8): spherical primary
    K=16 (3 blocks for gate/up, 2 for down) and a euclidean residual K=8,
    5 iterations, every randperm draw recorded."""
    torch.manual_seed(3)
    model = fake_moe(n_layers=1)
    params = config_mod.CodebookParams(k_gate=16, k_up=16, k_down=16, n_blocks_gate_up=3, n_blocks_down=2,
                                       max_iters=5, norm_threshold=1e-9, skip_zeros=False, residual_k=8)
    with RandpermRecorder() as rec:
        res = quantize_mod.extract_and_build_codebooks(model, params, progress=False)
    ex = model.model.language_model.layers[0].mlp.experts
    out_d = {"gate_up": ex.gate_up_proj.data.numpy(), "down": ex.down_proj.data.numpy(), **pack_perms(rec.perms)}
    for name, (aqlm, cwr) in res[0].items():
        out_d[f"{name}__recon"] = aqlm.reconstruct(cwr).numpy()
        out_d[f"{name}__c0_idxs"] = cwr.primary.idxs.numpy()
        out_d[f"{name}__c1_idxs"] = cwr.residuals[0].idxs.numpy()
        out_d[f"{name}__c0_cent_bf16"] = bf16_bits(aqlm.primary.centroids_tensor)
        out_d[f"{name}__c1_cent_bf16"] = bf16_bits(aqlm.residuals[0].centroids_tensor)
    np.savez_compressed(out / "extract.npz", **out_d)
    print("extract: " + ", ".join(f"{k}" for k in res[0]))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SKCQ_REFERENCE"),
                    help="the reference checkout (default: $SKCQ_REFERENCE)")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref or set SKCQ_REFERENCE")
    sys.path.insert(0, args.ref)
    torch.set_num_threads(8)
    import skcq.codebook as cb
    import skcq.codebook.events as events
    import skcq.codebook.kmeans as km
    import skcq.codebook_experts as experts_mod
    import skcq.config as config_mod
    import skcq.eval_model as eval_model
    import skcq.metrics as metrics
    import skcq.quantize as quantize_mod
    import skcq.vq.bpw as bpw_mod
    import skcq.vq.experiment as vq_experiment
    import skcq.vq.runner as vq_runner

    todo = (args.only.split(",") if args.only
            else ["assign", "kmeans", "codecs", "experts", "config1", "vq", "metrics", "extract"])
    if "assign" in todo:
        case_assign(HERE, km)
    if "kmeans" in todo:
        case_kmeans(HERE, km, events)
    if "codecs" in todo:
        case_codecs(HERE, cb, experts_mod)
    if "experts" in todo:
        case_experts(HERE, cb, experts_mod)
    if "config1" in todo:
        case_config1(HERE, cb, bpw_mod)
    if "vq" in todo:
        case_vq(HERE, vq_experiment, vq_runner)
    if "metrics" in todo:
        case_metrics(HERE, metrics, eval_model)
    if "extract" in todo:
        case_extract(HERE, quantize_mod, config_mod)


if __name__ == "__main__":
    main()
