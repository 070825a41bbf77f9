"""Model-level metrics (skcq_b200.metrics / skcq_b200.eval_model) against values
the reference's own functions computed on the same inputs (tests/golden/metrics.npz,
written by tests/golden/make_golden.py from skcq/metrics.py and skcq/eval_model.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _helpers import CharTokenizer, TinyLM, load_golden, sub
from skcq_b200 import eval_model, metrics


@pytest.fixture(scope="module")
def g():
    return load_golden("metrics")


def _capture(d: dict, side: str) -> metrics.RoutingCapture:
    cap = metrics.RoutingCapture()
    for i, layer in enumerate(d[f"{side}__layers"]):
        cap.layer_index.append(int(layer))
        cap.top_k_index.append(torch.from_numpy(d[f"{side}__idx{i}"]))
        cap.top_k_weights.append(torch.from_numpy(d[f"{side}__w{i}"]))
    return cap


@pytest.mark.parametrize("tag", ["a", "b"])
def test_routing_agreement_matches_reference(g, tag):
    d = sub(g, f"rt_{tag}__")
    out = metrics.routing_agreement(_capture(d, "base"), _capture(d, "quant"))
    assert out["common_layers"] == int(d["common_layers"][0])
    assert out["total_tokens"] == int(d["total_tokens"][0])
    for key in ("set_agreement", "weight_cosine", "routing_jsd"):
        assert out[key] == pytest.approx(float(d[key][0]), rel=1e-6, abs=1e-9), key
    per = np.array([[p["layer"], p["tokens"], p["set_agreement"]] for p in out["per_layer"]])
    np.testing.assert_allclose(per, d["per_layer"], rtol=1e-6)


def test_routing_agreement_identical_captures(g):
    cap = _capture(sub(g, "rt_a__"), "base")
    out = metrics.routing_agreement(cap, cap)
    assert out["set_agreement"] == 1.0
    assert out["weight_cosine"] == pytest.approx(1.0, abs=1e-6)
    assert out["routing_jsd"] == pytest.approx(0.0, abs=1e-7)


def test_lm_metrics_match_reference(g):
    text = str(g["lm_text"][0])
    tok = CharTokenizer()
    model, model_q = TinyLM(seed=5), TinyLM(seed=5, noise=0.05)
    ids = tok(text).input_ids
    ref = metrics.capture_reference_logits(model, ids, max_length=64)
    np.testing.assert_allclose(ref.numpy(), g["lm_ref_logits"], rtol=1e-6, atol=1e-6)
    assert metrics.kld_against_reference(model_q, ids, ref) == pytest.approx(float(g["lm_kld"][0]), rel=1e-5)
    np.testing.assert_allclose(metrics.token_log_likelihoods(model_q, ids[:, :80]).numpy(), g["lm_tll"],
                               rtol=1e-6, atol=1e-6)
    for m, key in ((model_q, "lm_ppl"), (model, "lm_ppl_base")):
        ppl = eval_model.compute_perplexity(m, tok, text, max_length=48, stride=16)
        assert ppl == pytest.approx(float(g[key][0]), rel=1e-5)


def test_kld_token_chunking_does_not_change_the_value(g):
    text = str(g["lm_text"][0])
    tok = CharTokenizer()
    ids = tok(text).input_ids
    ref = metrics.capture_reference_logits(TinyLM(seed=5), ids, max_length=64)
    q = TinyLM(seed=5, noise=0.05)
    a = metrics.kld_against_reference(q, ids, ref)
    b = metrics.kld_against_reference(q, ids, ref, token_chunk=7)
    assert a == pytest.approx(b, rel=1e-6)


class _Experts(torch.nn.Module):
    def forward(self, hidden, top_k_index=None, top_k_weights=None):
        return hidden


class _Layer(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.mlp = torch.nn.Module()
        self.mlp.experts = _Experts()


class _Model(torch.nn.Module):
    """Hugging Face layout: model.model.layers[i].mlp.experts."""

    def __init__(self, n_layers: int):
        super().__init__()
        self.model = torch.nn.Module()
        self.model.layers = torch.nn.ModuleList([_Layer() for _ in range(n_layers)])


def test_install_routing_capture_records_every_call_in_order():
    model = _Model(3)
    cap, handles = metrics.install_routing_capture(model)
    h = torch.randn(5, 8)
    idx = [torch.randint(0, 16, (5, 4)) for _ in range(4)]
    w = torch.rand(5, 4)
    layers = model.model.layers
    layers[0].mlp.experts(h, idx[0], w)
    layers[2].mlp.experts(h, idx[1])  # no weights
    layers[1].mlp.experts(h, idx[2], w)
    layers[0].mlp.experts(h, idx[3], w)  # a layer called twice
    layers[1].mlp.experts(h)  # no routing tensor: ignored
    assert cap.layer_index == [0, 2, 1, 0]
    for got, want in zip(cap.top_k_index, [idx[0], idx[1], idx[2], idx[3]]):
        assert torch.equal(got, want)
    assert cap.top_k_weights[1].numel() == 0 and torch.equal(cap.top_k_weights[0], w)
    assert [len(v) for v in cap.per_layer_index_tensors().values()] == [2, 1, 1]
    metrics.remove_hooks(handles)
    layers[0].mlp.experts(h, idx[0], w)
    assert cap.num_calls() == 4
    cap.reset()
    assert cap.num_calls() == 0


def test_calibration_text_from_a_local_file(tmp_path):
    p = tmp_path / "c.txt"
    p.write_text("one\ntwo\nthree\n")
    assert eval_model.get_calibration_text(2, path=p) == "one\ntwo"


def _text(n: int = 200) -> str:
    rs = np.random.RandomState(3)
    return "".join(rs.choice(list("abcdefgh ijk"), size=n))


def test_evaluate_quantized_flow_on_a_tiny_moe():
    """The eval flow (dense baseline, replacement, quantized metrics) with a
    replacement that perturbs the dense experts: summary keys as the reference's,
    identical models give zero divergence."""
    from _helpers import DenseExperts, TinyMoE
    from skcq_b200.eval_quantized import evaluate_quantized

    tok = CharTokenizer()
    same = evaluate_quantized(TinyMoE(seed=1), tok, _text(), [], 4, kld_tokens=64, max_length=48, stride=16,
                              replace=lambda m, mods, e: None)
    assert same["kld_base_to_quant"] == pytest.approx(0.0, abs=1e-9)
    assert same["ppl_ratio"] == pytest.approx(1.0, rel=1e-9)
    assert same["routing"]["set_agreement"] == 1.0 and same["routing"]["common_layers"] == 2

    def perturb(model, _mods, _e):
        g = torch.Generator().manual_seed(9)
        for layer in model.model.layers:
            ex = layer.mlp.experts
            noisy = DenseExperts(ex.gate_up_proj.shape[0], ex.gate_up_proj.shape[2], ex.I, g)
            with torch.no_grad():
                noisy.gate_up_proj.copy_(ex.gate_up_proj * (1 + 0.05 * torch.randn(ex.gate_up_proj.shape, generator=g)))
                noisy.down_proj.copy_(ex.down_proj * (1 + 0.05 * torch.randn(ex.down_proj.shape, generator=g)))
            layer.mlp.experts = noisy

    out = evaluate_quantized(TinyMoE(seed=1), tok, _text(), [], 4, kld_tokens=64, max_length=48, stride=16,
                             replace=perturb)
    assert set(out) == {"baseline_ppl", "quantized_ppl", "ppl_ratio", "ppl_delta", "kld_base_to_quant",
                        "kld_tokens", "routing"}
    assert out["kld_base_to_quant"] > 0 and out["routing"]["total_tokens"] == 2 * 64
    assert out["ppl_ratio"] == pytest.approx(1.0, abs=0.2)


@pytest.mark.gpu
def test_evaluate_quantized_with_codebook_experts():
    """Fit codebooks to a tiny MoE's experts on the GPU, install CodebookExperts
    with replace_experts and evaluate: the quantized model stays close to the
    dense one (same routing for most tokens, small KL)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from _helpers import TinyMoE
    from skcq_b200 import codebook as cb
    from skcq_b200.codebook_experts import CodebookModule
    from skcq_b200.eval_quantized import evaluate_quantized

    torch.manual_seed(0)
    model = TinyMoE(H=32, I=16, E=4, seed=2).cuda()
    E, H, I = 4, 32, 16
    modules = []
    for layer in model.model.layers:
        ex = layer.mlp.experts
        rows = {"gate": (ex.gate_up_proj[:, :I, :].reshape(-1, H), I),
                "up": (ex.gate_up_proj[:, I:, :].reshape(-1, H), I),
                "down": (ex.down_proj.reshape(-1, I), H)}
        mods = {}
        for name, (w, out_dim) in rows.items():
            prim = cb.SphericalCodebook(cb.SphericalCodebookConfig(block_size=4, K=64, max_iters=20,
                                                                   norm_threshold=1e-9, skip_zeros=False))
            res = [cb.EuclideanCodebook(cb.EuclideanCodebookConfig(block_size=4, K=64, max_iters=20,
                                                                   norm_threshold=1e-9, skip_zeros=False))]
            aqlm = cb.AQLMCodebook(prim, res, cb.AQLMCodebookConfig(norm_threshold=1e-9))
            cwr = aqlm.fit(w.detach().float())
            mods[name] = CodebookModule.from_cwr(aqlm, cwr, out_dim=out_dim).to(torch.float32).cuda()
        modules.append(mods)
    out = evaluate_quantized(model, CharTokenizer(), _text(), modules, E, kld_tokens=96, max_length=64, stride=32)
    from skcq_b200.codebook_experts import CodebookExperts

    assert all(isinstance(layer.mlp.experts, CodebookExperts) for layer in model.model.layers)
    assert 0 <= out["kld_base_to_quant"] < 0.05
    assert out["routing"]["set_agreement"] > 0.8
    assert out["ppl_ratio"] == pytest.approx(1.0, abs=0.05)
