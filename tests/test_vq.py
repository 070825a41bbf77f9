"""Sweep runner (skcq/vq/experiment.py) and its integer / fp8 baselines
(skcq/vq/runner.py) against rows the reference computed (tests/golden/vq.npz)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _helpers import PermReplay, load_golden, sub
from skcq_b200.vq.runner import integer_schemes

SPECS = {
    "cos_int8": ("gate", 4, 16, 2, "cosine", 8, None, False, True, 8, "int8", None, 8),
    "euc_shared": ("down", 4, 16, 2, "euclidean", 8, True, True, False, 8, "bf16", 6, 16),
}


def _check_schemes(device: str) -> None:
    g = load_golden("vq")
    w = torch.from_numpy(g["int_w"]).to(device)
    names = [n for n, _ in integer_schemes(8)]
    assert names == [k.split("__")[1] for k in g if k.startswith("int__") and k.endswith("__bpw")]
    for name, fn in integer_schemes(8):
        recon, bpw = fn(w.clone())
        assert bpw == pytest.approx(float(g[f"int__{name}__bpw"][0]), rel=1e-12), name
        got, ref = recon.float().cpu().numpy(), g[f"int__{name}__recon"]
        if device == "cpu":
            assert np.array_equal(got, ref), name
        else:
            # CUDA elementwise kernels may contract q * scale + min into one
            # rounding; a value on a rounding boundary can then land one step away
            diff = np.abs(got - ref)
            close = diff <= 1e-6 * np.abs(ref).max()
            assert close.mean() > 0.999, (name, close.mean())
            assert diff.max() <= (ref.max() - ref.min()) / 2 + 1e-6, name


def test_integer_schemes_match_reference():
    _check_schemes("cpu")


@pytest.mark.gpu
def test_integer_schemes_on_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    _check_schemes("cuda")


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(SPECS))
def test_vq_run_matches_reference(name, monkeypatch):
    """Same scheme label, bits per weight exactly and rel_fro_err within 5%
    (near-tied k-means trajectories may differ in rounding order)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from skcq_b200.vq.experiment import VQDoneEvent, VQRunConfig, VQRunExperiment

    g = sub(load_golden("vq"), f"vq__{name}__")
    proj, bs, K, ncb, metric, rk, rss, shared, ss, iters, sdt, rbs, cbits = SPECS[name]
    w = torch.from_numpy(g["w"])
    E, H, I = 4, 16, 8
    cfg = VQRunConfig(projection=proj, in_dim=w.shape[1], num_experts=E, hidden_size=H, intermediate_size=I,
                      block_size=bs, K=K, n_codebooks=ncb, metric=metric, residual_k=rk, residual_sign_split=rss,
                      shared_codebook=shared, sign_split=ss, max_iters=iters, scale_dtype=sdt,
                      residual_block_sizes=rbs, codebook_bits=cbits, layer_idx=3, device=torch.device("cuda"),
                      chunk_budget_mb=64)
    monkeypatch.setattr(torch, "randperm", PermReplay.from_case(g).torch_patch())
    exp = VQRunExperiment(cfg)
    done = []
    exp.on(VQDoneEvent, done.append)
    row = exp.fit(w)
    assert row["scheme"] == str(g["scheme"][0])
    assert row["residual_block_sizes"] == [int(v) for v in g["rbs"]]
    assert row["bits_per_weight"] == pytest.approx(float(g["bpw"][0]), rel=1e-12)
    assert row["rel_fro_err"] == pytest.approx(float(g["err"][0]), rel=0.05)
    assert done and done[0].row is row and exp.result is row


@pytest.mark.parametrize("name", list(SPECS))
def test_vq_plan_label_and_bits_match_reference(name):
    """The configuration's scheme label, residual block-size list and bits per
    weight (host logic only) equal the reference's row."""
    from skcq_b200.vq.bpw import bits_per_weight_kmeans
    from skcq_b200.codebook.spherical import scale_bits_per_elem
    from skcq_b200.vq.experiment import VQRunConfig, VQRunExperiment, _plan

    g = sub(load_golden("vq"), f"vq__{name}__")
    proj, bs, K, ncb, metric, rk, rss, shared, ss, iters, sdt, rbs, cbits = SPECS[name]
    n_rows, in_dim = g["w"].shape
    cfg = VQRunConfig(projection=proj, in_dim=in_dim, num_experts=4, hidden_size=16, intermediate_size=8,
                      block_size=bs, K=K, n_codebooks=ncb, metric=metric, residual_k=rk, residual_sign_split=rss,
                      shared_codebook=shared, sign_split=ss, max_iters=iters, scale_dtype=sdt,
                      residual_block_sizes=rbs, codebook_bits=cbits, layer_idx=3, device=None, chunk_budget_mb=64)
    plan = _plan(cfg)
    assert plan.label == str(g["scheme"][0])
    row = VQRunExperiment(cfg)._row(plan, 0.0, 1.0)
    assert row["residual_block_sizes"] == [int(v) for v in g["rbs"]]
    bpw = bits_per_weight_kmeans(
        n_rows, in_dim, in_dim // bs, bs, ncb, plan.ks, shared_codebook=shared, sign_split=ss,
        scale_bits_per_elem=scale_bits_per_elem(sdt), bs_per_codebook=plan.block_sizes, codebook_bits=cbits,
        residual_sign_split=plan.residual_sign_split, primary_metric=metric)
    assert bpw == pytest.approx(float(g["bpw"][0]), rel=1e-12)
