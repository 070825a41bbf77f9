"""Config models, AQLM assembly rules and the build driver's row slicing
(skcq/config.py, skcq/quantize.py; tests/test_codebook.py:139-230)."""

from __future__ import annotations

import types

import pytest
import torch

from skcq_b200.codebook import EuclideanCodebook, SphericalCodebook, SSVQCodebook
from skcq_b200.config import CodebookParams, ExperimentConfig, LayerOverride, build_aqlm_codebook
from skcq_b200.quantize import get_text_model, layer_params, projection_rows


def _inner(cb):
    return cb.inner if isinstance(cb, SSVQCodebook) else cb


def test_defaults_match_reference():
    p = CodebookParams()
    assert (p.k_gate, p.k_up, p.k_down, p.n_blocks_gate_up, p.n_blocks_down, p.n_codebooks) == (4096, 4096, 4096, 1,
                                                                                                   1, 2)
    assert (p.max_iters, p.norm_threshold, p.skip_zeros, p.chunk_budget_mb) == (100, 0.001, True, 2048)
    assert p.residual_k is None and p.residual_block_sizes is None and p.residual_sign_split is None


def test_assembly_rules():
    """config.py:137-197: spherical primary of bs = in_dim // n_blocks, euclidean
    residuals with skip_zeros=False, codebook_bits fixed at 16."""
    p = CodebookParams(max_iters=7, norm_threshold=1e-4, skip_zeros=True)
    a = build_aqlm_codebook(p, k=32, n_blocks=3, n_codebooks=3, in_dim=12, out_dim=8, num_experts=4)
    assert isinstance(a.primary, SphericalCodebook)
    c = a.primary.config
    assert (c.block_size, c.K, c.max_iters, c.norm_threshold, c.skip_zeros) == (4, 32, 7, 1e-4, True)
    assert len(a.residuals) == 2
    for r in a.residuals:
        assert isinstance(r, EuclideanCodebook)
        assert (r.config.block_size, r.config.K, r.config.skip_zeros) == (4, 32, False)
    assert a.config.codebook_bits == 16 and a.config.out_dim == 8 and a.config.num_experts == 4
    # n_blocks 0 -> whole row is one block; num_experts 0 -> None
    a0 = build_aqlm_codebook(p, k=8, n_blocks=0, n_codebooks=1, in_dim=12, out_dim=8)
    assert a0.primary.config.block_size == 12 and a0.config.num_experts is None


def test_residual_lists():
    """residual_k / residual_block_sizes index residual c at [c-1];
    residual_sign_split indexes [c] (config.py:116-134)."""
    p = CodebookParams(residual_k=[8, 16], residual_block_sizes=[6, 3], residual_sign_split=[False, True])
    a = build_aqlm_codebook(p, k=32, n_blocks=2, n_codebooks=3, in_dim=24, out_dim=8)
    r1, r2 = a.residuals
    assert isinstance(r1, SSVQCodebook) and isinstance(r2, EuclideanCodebook)
    assert (_inner(r1).config.K, _inner(r1).config.block_size) == (8, 6)
    assert (r2.config.K, r2.config.block_size) == (16, 3)
    p2 = CodebookParams(residual_k=8, residual_block_sizes=5, residual_sign_split=True)
    b = build_aqlm_codebook(p2, k=32, n_blocks=2, n_codebooks=2, in_dim=24, out_dim=8)
    assert isinstance(b.residuals[0], SSVQCodebook)
    assert (_inner(b.residuals[0]).config.K, _inner(b.residuals[0]).config.block_size) == (8, 5)
    assert isinstance(b.primary, SphericalCodebook)  # never sign-split


def test_overrides_and_yaml(tmp_path):
    cfg = ExperimentConfig(defaults=CodebookParams(k_gate=256), layer_overrides={3: LayerOverride(k_gate=64,
                                                                                                  max_iters=5)})
    assert cfg.params_for_layer(0).k_gate == 256
    p3 = cfg.params_for_layer(3)
    assert (p3.k_gate, p3.max_iters, p3.k_up) == (64, 5, 4096)
    path = tmp_path / "cfg.yaml"
    cfg.to_yaml(path)
    back = ExperimentConfig.from_yaml(path)
    assert back == cfg
    assert layer_params(cfg.defaults, cfg.layer_overrides, 3) == p3


def _fake_moe(n_layers=2, E=4, H=12, I=8, seed=0):
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


def test_projection_rows_match_reference_slicing():
    """quantize.py:56-61: expert-major rows of gate, up and down."""
    m = _fake_moe()
    rows = projection_rows(get_text_model(m).layers[0].mlp.experts, 8, 12)
    gu = m.model.language_model.layers[0].mlp.experts.gate_up_proj.data
    dn = m.model.language_model.layers[0].mlp.experts.down_proj.data
    assert [r[0] for r in rows] == ["gate", "up", "down"]
    assert torch.equal(rows[0][1], gu[:, :8, :].reshape(-1, 12)) and rows[0][2] == 8
    assert torch.equal(rows[1][1], gu[:, 8:, :].reshape(-1, 12)) and rows[1][2] == 8
    assert torch.equal(rows[2][1], dn.reshape(-1, 8)) and rows[2][2] == 12


def test_cuda_worker_hook_is_used():
    from skcq_b200.quantize import extract_and_build_codebooks

    calls = []

    class Worker:
        def build_codebook(self, rows, **kw):
            calls.append((tuple(rows.shape), kw["name"], kw["k"], kw["n_blocks"], kw["out_dim"], kw["num_experts"]))
            return ("aqlm", "cwr")

    params = CodebookParams(k_gate=16, k_up=8, k_down=4, n_blocks_gate_up=3, n_blocks_down=2)
    res = extract_and_build_codebooks(_fake_moe(), params, {1: LayerOverride(k_up=32)}, cuda_worker=Worker(),
                                      progress=False)
    assert len(res) == 2 and set(res[0]) == {"gate", "up", "down"}
    assert calls[0] == ((32, 12), "L0.gate", 16, 3, 8, 4)
    assert calls[1] == ((32, 12), "L0.up", 8, 3, 8, 4)
    assert calls[2] == ((48, 8), "L0.down", 4, 2, 12, 4)
    assert calls[4][1:3] == ("L1.up", 32)


@pytest.mark.gpu
def test_extract_and_build_on_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from skcq_b200.quantize import extract_and_build_codebooks

    torch.manual_seed(3)
    params = CodebookParams(k_gate=16, k_up=16, k_down=16, n_blocks_gate_up=3, n_blocks_down=2, max_iters=5,
                            norm_threshold=1e-9, skip_zeros=False, residual_k=8)
    res = extract_and_build_codebooks(_fake_moe(n_layers=1), params, progress=False)
    for name, (aqlm, cwr) in res[0].items():
        rows = dict((n, r) for n, r, _ in projection_rows(
            _fake_moe(n_layers=1).model.language_model.layers[0].mlp.experts, 8, 12))[name]
        recon = aqlm.reconstruct(cwr).cpu()
        err = ((recon - rows.float()).norm() / rows.float().norm()).item()
        assert err < 0.6, (name, err)
        assert cwr.primary.idxs.shape[1] == rows.shape[0]


@pytest.mark.gpu
def test_extract_and_build_matches_reference(monkeypatch):
    """The build driver over a one-layer MoE (4 experts, hidden 12,
    intermediate 8; spherical K=16 primary + euclidean K=8 residual, 5
    iterations) against the reference's own extract_and_build_codebooks on
    the same weights and the same recorded randperm draws: every projection's
    reconstruction within 2e-3 and rel_fro_err within 1e-3 relative, and the
    same primary and residual indices (the oracle finds every k-means
    trajectory of this case tie-free)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import numpy as np

    from _helpers import PermReplay, load_golden
    from skcq_b200.quantize import extract_and_build_codebooks

    g = load_golden("extract")
    model = _fake_moe(n_layers=1)
    ex = model.model.language_model.layers[0].mlp.experts
    ex.gate_up_proj.data.copy_(torch.from_numpy(g["gate_up"]))
    ex.down_proj.data.copy_(torch.from_numpy(g["down"]))
    monkeypatch.setattr(torch, "randperm", PermReplay.from_case(g).torch_patch())
    params = CodebookParams(k_gate=16, k_up=16, k_down=16, n_blocks_gate_up=3, n_blocks_down=2, max_iters=5,
                            norm_threshold=1e-9, skip_zeros=False, residual_k=8)
    res = extract_and_build_codebooks(model, params, device=torch.device("cuda"), progress=False)
    rows = dict((n, r) for n, r, _ in projection_rows(ex, 8, 12))
    for name, (aqlm, cwr) in res[0].items():
        w = rows[name].double().numpy()
        recon = aqlm.reconstruct(cwr).double().cpu().numpy()
        ref = g[f"{name}__recon"].astype(np.float64)
        e_gpu = np.linalg.norm(w - recon) / np.linalg.norm(w)
        e_ref = np.linalg.norm(w - ref) / np.linalg.norm(w)
        assert abs(e_gpu - e_ref) <= 1e-3 * e_ref, (name, e_gpu, e_ref)
        assert np.linalg.norm(recon - ref) / np.linalg.norm(ref) < 2e-3, name
        assert np.array_equal(cwr.primary.idxs.cpu().numpy(), g[f"{name}__c0_idxs"]), name
        assert np.array_equal(cwr.residuals[0].idxs.cpu().numpy(), g[f"{name}__c1_idxs"]), name
