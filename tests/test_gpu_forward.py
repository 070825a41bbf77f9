"""GPU parity of the codebook-expert forward (skcq/codebook_experts.py) through
the C ABI: CodebookModule against the oracle forward and the dense
reconstruction, bf16 tolerance, state-dict round trip, the reference's failure
modes, and CodebookExperts against the oracle and the reference's outputs."""

from __future__ import annotations

import io

import numpy as np
import pytest
import torch

from _helpers import PermReplay, load_golden, rel_err, sub
from oracle import forward as of

pytestmark = pytest.mark.gpu

FWD_CASES = ["base", "single", "ssvq", "noncomm", "asym"]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _fit(name, monkeypatch):
    import test_gpu_build as B

    g = sub(load_golden("codecs"), name + "__")
    monkeypatch.setattr(torch, "randperm", PermReplay.from_case(g).torch_patch())
    aqlm = B._product_aqlm(name)
    cwr = aqlm.fit(torch.from_numpy(g["w"]).cuda())
    return g, aqlm, cwr


def _oracle_layers(mod):
    """The module's own buffers as oracle layer dicts (f32, scales dequantised)."""
    out = []
    for lay in mod.layers:
        s = None
        if lay.scales is not None:
            s = lay.scales.detach().float().cpu().numpy()
            if not lay.scales.is_floating_point():
                s = s * float(lay.scale_q_scale)
        out.append({
            "codebook": lay.codebook.detach().float().cpu().numpy(),
            "assignments": lay.assignments.cpu().numpy(),
            "scales": s,
            "remainder": lay.remainder.float().cpu().numpy(),
            "signs": lay.signs.cpu().numpy() if lay.signs is not None else None,
            "block_size": lay.block_size,
            "forward_mode": lay.forward_mode,
        })
    return out


@pytest.mark.parametrize("name", FWD_CASES)
def test_module_matches_oracle_and_reconstruction(name, monkeypatch):
    """forward == oracle module forward on the same buffers, and
    == hidden @ reconstruct(cwr)[e].T (tests/test_codebook.py:74-122)."""
    from skcq_b200.codebook_experts import CodebookModule

    g, aqlm, cwr = _fit(name, monkeypatch)
    mod = CodebookModule.from_cwr(aqlm, cwr, out_dim=8).to(torch.float32).cuda()
    hidden = torch.from_numpy(g["hidden"]).cuda()
    layers = _oracle_layers(mod)
    w = aqlm.reconstruct(cwr).double().cpu()
    w = w.reshape(-1, 8, w.shape[1])
    outs = []
    for e in range(w.shape[0]):
        out = mod(hidden, expert_idx=e)
        assert out.dtype == torch.float32 and out.shape == (hidden.shape[0], 8)
        out = out.double().cpu()
        outs.append(out.numpy())
        assert rel_err(out.numpy(), of.module_forward(layers, g["hidden"], e)) < 1e-6, f"expert {e}"
        assert np.allclose(out.numpy(), g["hidden"].astype(np.float64) @ w[e].numpy().T, atol=1e-5, rtol=1e-5)
    # where the fit itself reproduces the reference's, so does the forward
    if rel_err(aqlm.reconstruct(cwr).cpu().numpy(), g["recon"]) < 2e-3:
        assert rel_err(np.stack(outs), g["fwd"]) < 2e-3


def test_module_on_reference_payload():
    """The reference's own fitted payload (golden, 'base') loaded into the module
    reproduces the reference module's outputs, independent of any fit."""
    from _helpers import bf16_from_bits
    from skcq_b200.codebook_experts import CodebookModule

    g = sub(load_golden("codecs"), "base__")
    rows, in_dim = int(g["meta"][0]), int(g["meta"][1])
    E, out_dim, bs = rows // 8, 8, 4
    nb = in_dim // bs
    mod = CodebookModule.empty(nb, bs, out_dim, [16, 16], E)
    sd = mod.state_dict()
    for c in range(2):
        cent = bf16_from_bits(g[f"c{c}_cent_bf16"]).reshape(nb, bs, 16)
        sd[f"layers.{c}.codebook"] = torch.from_numpy(cent).float()
        idx = g[f"c{c}_idxs"].reshape(nb, E, out_dim).transpose(1, 0, 2)
        sd[f"layers.{c}.assignments"] = torch.from_numpy(np.ascontiguousarray(idx)).long()
    sc = g["c0_scales"].reshape(E, out_dim, nb).transpose(0, 2, 1)
    sd["layers.0.scales"] = torch.from_numpy(np.ascontiguousarray(sc)).float()
    mod = mod.to(torch.float32)
    mod.load_state_dict(sd)
    mod = mod.cuda()
    hidden = torch.from_numpy(g["hidden"]).cuda()
    out = np.stack([mod(hidden, expert_idx=e).cpu().numpy() for e in range(E)])
    # centroids are stored as bf16 in the fixture; the reference ran on f32 ones
    assert rel_err(out, g["fwd"]) < 1e-2
    ref = np.stack([of.module_forward(_oracle_layers(mod), g["hidden"], e) for e in range(E)])
    assert rel_err(out, ref) < 1e-6


def test_bf16_module_within_bf16_tolerance(monkeypatch):
    from skcq_b200.codebook_experts import CodebookModule

    g, aqlm, cwr = _fit("base", monkeypatch)
    mod32 = CodebookModule.from_cwr(aqlm, cwr, out_dim=8).to(torch.float32).cuda()
    mod16 = CodebookModule.from_cwr(aqlm, cwr, out_dim=8).to(torch.bfloat16).cuda()
    hidden = torch.from_numpy(g["hidden"]).cuda()
    for e in range(4):
        a = mod32(hidden, e).double()
        b16 = mod16(hidden.to(torch.bfloat16), e)
        assert b16.dtype == torch.bfloat16
        b = b16.double()
        cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
        # the forward tolerance for bf16 (bf16 inputs, scales and output):
        # max error <= 1e-2 of the output's max, cosine >= 0.9999
        assert (a - b).abs().max().item() <= 1e-2 * a.abs().max().item()
        assert cos >= 0.9999


def test_state_dict_round_trip(monkeypatch):
    """tests/test_codebook.py:294-324: save, load, identical outputs."""
    from skcq_b200.codebook_experts import CodebookModule

    g, aqlm, cwr = _fit("ssvq", monkeypatch)
    mod = CodebookModule.from_cwr(aqlm, cwr, out_dim=8).to(torch.bfloat16).cuda()
    hidden = torch.randn(6, 12, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).cuda()
    before = mod(hidden, expert_idx=2)
    buf = io.BytesIO()
    torch.save(mod.state_dict_with_meta(), buf)
    buf.seek(0)
    loaded = CodebookModule.load(buf).cuda()
    assert loaded.primary.signs is not None
    assert torch.equal(before, loaded(hidden, expert_idx=2))


def test_shared_codebook_fails_like_reference(monkeypatch):
    """A shared codebook cannot drive the per-expert forward: the reference's
    gather fails (codebook_experts.py:49); so does this one, loudly."""
    from skcq_b200.codebook_experts import CodebookModule

    g, aqlm, cwr = _fit("shared", monkeypatch)
    mod = CodebookModule.from_cwr(aqlm, cwr, out_dim=8).to(torch.float32).cuda()
    with pytest.raises(RuntimeError):
        mod(torch.randn(3, 12).cuda(), 0)


def test_experts_forward_matches_oracle(monkeypatch):
    """CodebookExperts.forward (codebook_experts.py:454-481) on a 4-expert top-2 MoE."""
    from skcq_b200 import codebook as cb
    from skcq_b200.codebook_experts import CodebookExperts, CodebookModule

    g = load_golden("experts")
    monkeypatch.setattr(torch, "randperm", PermReplay.from_case(g).torch_patch())
    mods = []
    for w, out_dim in ((g["wg"], 8), (g["wu"], 8), (g["wd"], 12)):
        prim = cb.SphericalCodebook(cb.SphericalCodebookConfig(block_size=4, K=16, max_iters=10,
                                                               norm_threshold=1e-9, skip_zeros=False))
        res = [cb.EuclideanCodebook(cb.EuclideanCodebookConfig(block_size=4, K=8, max_iters=10,
                                                               norm_threshold=1e-9, skip_zeros=False))]
        aqlm = cb.AQLMCodebook(prim, res, cb.AQLMCodebookConfig(norm_threshold=1e-9))
        cwr = aqlm.fit(torch.from_numpy(w).cuda())
        mods.append(CodebookModule.from_cwr(aqlm, cwr, out_dim=out_dim).to(torch.float32).cuda())
    ex = CodebookExperts(mods[0], mods[1], mods[2], 4, torch.nn.functional.silu)
    hidden = torch.from_numpy(g["hidden"]).cuda()
    y = ex(hidden, torch.from_numpy(g["topi"]).cuda(), torch.from_numpy(g["topw"]).cuda())
    assert y.dtype == torch.float32 and y.shape == hidden.shape
    y = y.cpu().numpy()
    ref = of.experts_forward(*[_oracle_layers(m) for m in mods], 4, g["hidden"], g["topi"], g["topw"])
    assert rel_err(y, ref) < 1e-6
    assert rel_err(y, g["y"]) < 2e-3


def test_experts_generic_activation_and_unrouted_expert(monkeypatch):
    """A non-SiLU act_fn goes through the module's own activation; an expert
    that no token selects contributes nothing (codebook_experts.py:465-467)."""
    from skcq_b200.codebook_experts import CodebookExperts

    E, H, I, T = 4, 32, 16, 10
    gate = _random_module(E, I, H, [(4, 16, True), (4, 8, False)], seed=11)
    up = _random_module(E, I, H, [(4, 16, True), (4, 8, False)], seed=12)
    down = _random_module(E, H, I, [(4, 16, True), (4, 8, False)], seed=13)
    gen = torch.Generator().manual_seed(14)
    hidden = torch.randn(T, H, generator=gen)
    topi = torch.randint(0, 3, (T, 2), generator=gen)  # expert 3 never routed
    topi[:, 1] = (topi[:, 0] + 1) % 3
    topw = torch.rand(T, 2, generator=gen)
    ex = CodebookExperts(gate, up, down, E, torch.nn.functional.gelu)
    y = ex(hidden.cuda(), topi.cuda(), topw.cuda()).cpu().numpy()
    ref = np.zeros((T, H), np.float64)
    Wg, Wu, Wd = ([_dense_from_module(m, e).numpy() for e in range(E)] for m in (gate, up, down))
    hd = hidden.double().numpy()
    for t in range(T):
        for j in range(2):
            e = int(topi[t, j])
            gt = torch.nn.functional.gelu(torch.from_numpy(hd[t] @ Wg[e].T)).numpy()
            ref[t] += float(topw[t, j]) * ((gt * (hd[t] @ Wu[e].T)) @ Wd[e].T)
    assert rel_err(y, ref) < 1e-5


def _random_module(E, out_dim, in_dim, specs, seed, dtype=torch.float32):
    """CodebookModule with random buffers: specs = [(bs, K, scaled)]."""
    from skcq_b200.codebook_experts import CodebookModule, _CodebookLayer

    g = torch.Generator().manual_seed(seed)
    layers = []
    for bs, K, scaled in specs:
        nb = in_dim // bs
        rem = in_dim - nb * bs
        layers.append(_CodebookLayer(
            (torch.randn(nb, bs, K, generator=g) * 0.05).to(dtype),
            torch.randint(0, K, (E, nb, out_dim), generator=g),
            nb, bs, out_dim, K,
            remainder=(torch.randn(E, out_dim, rem, generator=g) * 0.02).to(dtype) if rem else None,
            scales=(torch.rand(E, nb, out_dim, generator=g) * 0.1).to(dtype) if scaled else None,
        ))
    return CodebookModule(torch.nn.ModuleList(layers), len(layers), out_dim).cuda()


def _dense_from_module(mod, e):
    """W_e (out, in) f64 from the module's own buffers (the math of _codebook_pass)."""
    out_dim = mod.out_dim
    parts = []
    for lay in mod.layers:
        cb = lay.codebook.detach().double().cpu()
        a = lay.assignments[e].cpu()
        nb, bs = lay.n_blocks, lay.block_size
        w = torch.zeros(out_dim, nb * bs + lay.rem, dtype=torch.float64)
        cols = torch.gather(cb, 2, a[:, None, :].expand(nb, bs, out_dim))  # (nb, bs, out)
        if lay.scales is not None:
            cols = cols * lay.scales[e].detach().double().cpu()[:, None, :]
        w[:, : nb * bs] = cols.permute(2, 0, 1).reshape(out_dim, nb * bs)
        if lay.rem:
            w[:, nb * bs:] = lay.remainder[e].double().cpu()
        parts.append(w)
    width = max(p.shape[1] for p in parts)
    return sum(torch.nn.functional.pad(p, (0, width - p.shape[1])) for p in parts)


def test_decode_shapes_match_dense():
    """Production codebook shapes (bs 8/16/4, K 4096/4096/65536; 16-bit indices
    above 32767) on 4 experts of 768 x 2048 with a 13-column remainder on the
    last codebook, decode batch of 8 tokens."""
    mod = _random_module(4, 768, 2061, [(8, 4096, True), (16, 4096, False), (4, 65536, False)], seed=5)
    x = torch.randn(8, 2061, generator=torch.Generator().manual_seed(6)).cuda()
    for e in (0, 3):
        out = mod(x, e).double().cpu()
        ref = x.double().cpu() @ _dense_from_module(mod, e).t()
        assert rel_err(out.numpy(), ref.numpy()) < 1e-5


def test_grouped_segments_match_per_expert():
    """run_segments over all experts at once equals per-expert calls
    (prefill: 300 rows routed unevenly to 8 experts, one expert empty)."""
    mod = _random_module(8, 96, 256, [(8, 256, True), (4, 256, False)], seed=21)
    gen = torch.Generator().manual_seed(22)
    counts = [40, 0, 100, 7, 1, 52, 60, 40]
    rows = torch.randn(sum(counts), 256, generator=gen).cuda()
    seg = torch.tensor(np.concatenate([[0], np.cumsum(counts)]), dtype=torch.int32).cuda()
    for n_split in (1, 3):
        part, S = mod.run_segments(rows, seg, None, 8, n_split=n_split)
        assert S == n_split and part.shape == (n_split, rows.shape[0], 96)
        y = part.sum(0).cpu()
        start = 0
        for e, c in enumerate(counts):
            if c:
                ye = mod(rows[start:start + c], e).cpu()
                assert rel_err(y[start:start + c].numpy(), ye.numpy()) < 1e-6
            start += c


def test_invalid_routing_raises():
    """An expert id outside [0, num_experts) raises, as the reference's one_hot does."""
    from skcq_b200.codebook_experts import CodebookExperts

    gate = _random_module(4, 8, 16, [(4, 16, True)], seed=31)
    up = _random_module(4, 8, 16, [(4, 16, True)], seed=32)
    down = _random_module(4, 16, 8, [(4, 16, True)], seed=33)
    ex = CodebookExperts(gate, up, down, 4, torch.nn.functional.silu)
    topi = torch.tensor([[0, 1], [2, 4]]).cuda()
    with pytest.raises(RuntimeError):
        ex(torch.randn(2, 16).cuda(), topi, torch.ones(2, 2).cuda())
    # the device stays usable and valid routing works afterwards
    y = ex(torch.randn(2, 16).cuda(), torch.tensor([[0, 1], [2, 3]]).cuda(), torch.ones(2, 2).cuda())
    assert torch.isfinite(y).all()


def test_out_of_range_assignment_raises():
    from skcq_b200.codebook_experts import CodebookModule, _CodebookLayer

    lay = _CodebookLayer(torch.randn(2, 4, 16), torch.full((1, 2, 8), 16, dtype=torch.long), 2, 4, 8, 16)
    mod = CodebookModule(torch.nn.ModuleList([lay]), 1, 8).cuda()
    with pytest.raises(RuntimeError):
        mod(torch.randn(3, 8).cuda(), 0)


def test_expert_index_semantics():
    mod = _random_module(3, 8, 16, [(4, 16, True)], seed=41)
    x = torch.randn(2, 16).cuda()
    assert torch.equal(mod(x, -1), mod(x, 2))
    with pytest.raises(IndexError):
        mod(x, 3)


def test_large_batch_route_sort_order():
    """Route sort of 4096 tokens x top-8 over 128 experts (chunked warp-ranking
    path) and over 300 experts (owner-scan path): the grouped result equals
    the per-token reference order."""
    from skcq_b200.codebook_experts import CodebookExperts

    for E in (128, 300):
        T, H, I = 512 if E == 300 else 4096, 32, 16
        gen = torch.Generator().manual_seed(E)
        gate = _random_module(E, I, H, [(8, 32, True)], seed=51)
        up = _random_module(E, I, H, [(8, 32, True)], seed=52)
        down = _random_module(E, H, I, [(8, 32, True)], seed=53)
        hidden = torch.randn(T, H, generator=gen)
        topi = torch.rand(T, E, generator=gen).argsort(-1)[:, :8]
        topw = torch.rand(T, 8, generator=gen)
        y = CodebookExperts(gate, up, down, E, torch.nn.functional.silu)(hidden.cuda(), topi.cuda(), topw.cuda())
        # reference loop on the GPU modules (codebook_experts.py:462-480)
        ref = torch.zeros(T, H).cuda()
        mask = torch.nn.functional.one_hot(topi.cuda(), E).permute(2, 1, 0)
        for e in range(E):
            pos, tok = torch.where(mask[e])
            if tok.numel() == 0:
                continue
            xs = hidden.cuda()[tok]
            inter = torch.nn.functional.silu(gate(xs, e)) * up(xs, e)
            ref.index_add_(0, tok, down(inter, e) * topw.cuda()[tok, pos, None])
        assert rel_err(y.cpu().numpy(), ref.cpu().numpy()) < 1e-5


# ---- tensor-core prefill path --------------------------------------------------


def _prefill_case(E, H, I, T, k, specs_gu, specs_d, seed, signs=False):
    from skcq_b200.codebook_experts import CodebookExperts

    gate = _random_module(E, I, H, specs_gu, seed=seed, dtype=torch.bfloat16)
    up = _random_module(E, I, H, specs_gu, seed=seed + 1, dtype=torch.bfloat16)
    down = _random_module(E, H, I, specs_d, seed=seed + 2, dtype=torch.bfloat16)
    if signs:
        g = torch.Generator().manual_seed(seed + 3)
        lay = gate.layers[0]
        sg = torch.where(torch.rand(E, I, lay.n_blocks * lay.block_size, generator=g) < 0.5, -1, 1).to(torch.int8)
        lay.register_buffer("signs", sg.cuda())
        lay.sign_cov = sg.shape[-1]
    ex = CodebookExperts(gate, up, down, E, torch.nn.functional.silu)
    gen = torch.Generator().manual_seed(seed + 4)
    hidden = torch.randn(T, H, generator=gen).to(torch.bfloat16)
    topi = torch.rand(T, E, generator=gen).argsort(-1)[:, :k]
    topw = torch.rand(T, k, generator=gen)
    return ex, hidden.cuda(), topi.cuda(), topw.cuda()


@pytest.mark.parametrize("case", ["base", "ragged", "bs12", "signs"])
def test_prefill_tensor_core_path_matches_gather_path(case):
    """The tcgen05 prefill path (decode weights once, grouped bf16 GEMM) agrees
    with the fp32 gather path within bf16 tolerance (max rel 1e-2, cos 0.9999)."""
    from skcq_b200 import _lib

    cfg = {
        "base": (8, 256, 128, 512, 2, [(8, 64, True), (16, 64, False), (4, 256, False)], [(8, 64, True), (4, 64, False)]),
        # in/out not multiples of 64/256, remainder columns, uneven expert load
        "ragged": (5, 200, 300, 333, 3, [(8, 32, True), (4, 16, False)], [(4, 32, True), (8, 16, False)]),
        "bs12": (4, 384, 96, 300, 2, [(12, 64, True), (6, 32, False)], [(12, 32, True), (6, 32, False)]),
        "signs": (6, 128, 64, 256, 2, [(8, 32, True), (16, 32, False)], [(8, 32, True)]),
    }[case]
    E, H, I, T, k, sgu, sd = cfg
    seed = {"base": 101, "ragged": 202, "bs12": 303, "signs": 404}[case]
    ex, x, topi, topw = _prefill_case(E, H, I, T, k, sgu, sd, seed=seed, signs=(case == "signs"))
    assert ex._use_prefill(x, T * k, min(E, T * k))
    _lib.LAUNCHES.reset()
    _lib.LAUNCHES.enabled = True
    y_tc = ex(x, topi, topw)
    _lib.LAUNCHES.enabled = False
    assert _lib.LAUNCHES.calls.get("skcq_prefill_gemm_swiglu") == 1 and _lib.LAUNCHES.calls.get("skcq_prefill_gemm") == 1
    ex.prefill_min_rows = 1 << 30
    _lib.LAUNCHES.reset()
    _lib.LAUNCHES.enabled = True
    y_ref = ex(x, topi, topw)
    _lib.LAUNCHES.enabled = False
    assert "skcq_prefill_gemm" not in _lib.LAUNCHES.calls and "skcq_prefill_gemm_swiglu" not in _lib.LAUNCHES.calls
    a, b = y_tc.double(), y_ref.double()
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    assert cos >= 0.9999, cos
    assert (a - b).abs().max().item() <= 1e-2 * b.abs().max().item(), (a - b).abs().max().item()


def test_prefill_gemm_exact_on_bf16_operands():
    """With bf16-exact weights and inputs the GEMM result equals an fp64
    matmul of the same operands to fp32 accumulation accuracy."""
    from skcq_b200 import _lib
    from skcq_b200._lib import call, ptr, stream

    E, H, I, T, k = 4, 192, 320, 400, 2
    ex, x, topi, topw = _prefill_case(E, H, I, T, k, [(8, 16, False)], [(8, 16, False)], seed=77)
    P = T * k
    route = torch.empty(2 * P + 2 * (E + 1), dtype=torch.int32, device="cuda")
    perm, inv, seg, active = route[:P], route[P:2 * P], route[2 * P:2 * P + E + 1], route[2 * P + E + 1:]
    call("skcq_route_sort", ptr(topi.contiguous()), T, k, E, ptr(perm), ptr(seg), ptr(inv), ptr(active), None, 0,
         0, stream())
    max_tiles = -(-P // 128) + E
    tiles = torch.empty(1 + 3 * max_tiles, dtype=torch.int32, device="cuda")
    call("skcq_prefill_plan", ptr(seg), E, max_tiles, ptr(tiles), stream())
    A = torch.empty(max_tiles * 3 * 8192, dtype=torch.bfloat16, device="cuda")
    call("skcq_prefill_pack", 0, ptr(x), 1, x.stride(0), ptr(perm), T, None, 0, H, ptr(tiles), max_tiles, ptr(A),
         stream())
    y = ex.gate.prefill(A, tiles, max_tiles, active, E, P, H)
    _lib.poll_device_error()
    # reference: per row, its token's x (bf16) against the expert's decoded weight rounded to bf16
    seg_h = seg.cpu().tolist()
    perm_h = perm.cpu()
    for e in range(E):
        r0, r1 = seg_h[e], seg_h[e + 1]
        if r0 == r1:
            continue
        W = _dense_from_module(ex.gate, e).to(torch.bfloat16).double()  # (I, H)
        xs = x.cpu()[perm_h[r0:r1] % T].double()
        ref = xs @ W.t()
        got = y[r0:r1].double().cpu()
        assert torch.allclose(got, ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item()), e


def test_prefill_generic_activation_path():
    """A non-SiLU act_fn takes the unfused two-GEMM prefill route."""
    E, H, I, T, k = 4, 128, 96, 256, 2
    ex, x, topi, topw = _prefill_case(E, H, I, T, k, [(8, 32, True)], [(8, 32, True)], seed=505)
    ex.intermediate.act_fn = torch.nn.functional.gelu
    y_tc = ex(x, topi, topw).double()
    ex.prefill_min_rows = 1 << 30
    y_ref = ex(x, topi, topw).double()
    cos = torch.nn.functional.cosine_similarity(y_tc.flatten(), y_ref.flatten(), dim=0).item()
    assert cos >= 0.9999 and (y_tc - y_ref).abs().max().item() <= 1e-2 * y_ref.abs().max().item()


def test_graphed_decode_replays_eager_results():
    """GraphedExperts (CUDA-graph replay) gives bit-identical results to the
    eager forward for fresh inputs of the captured shape."""
    from skcq_b200.codebook_experts import CodebookExperts, GraphedExperts

    E, H, I, T, k = 16, 256, 128, 4, 4
    gate = _random_module(E, I, H, [(8, 64, True), (4, 256, False)], seed=61, dtype=torch.bfloat16)
    up = _random_module(E, I, H, [(8, 64, True), (4, 256, False)], seed=62, dtype=torch.bfloat16)
    down = _random_module(E, H, I, [(8, 64, True)], seed=63, dtype=torch.bfloat16)
    ex = CodebookExperts(gate, up, down, E, torch.nn.functional.silu)
    g = GraphedExperts(ex, T, k)
    gen = torch.Generator().manual_seed(64)
    for _ in range(3):
        x = torch.randn(T, H, generator=gen).to(torch.bfloat16).cuda()
        topi = torch.rand(T, E, generator=gen).argsort(-1)[:, :k].cuda()
        topw = torch.rand(T, k, generator=gen).cuda()
        y = g(x, topi, topw).clone()
        assert torch.equal(y, ex(x, topi, topw))


def test_route_sort_multi_cta_matches_one_cta():
    """Large batches sort over many CTAs (with scratch); the permutation,
    segments and active list equal the one-CTA sort's and the reference's
    stable expert order."""
    from skcq_b200 import _lib
    from skcq_b200._lib import call, ptr, stream

    for T, k, E in ((16384, 8, 128), (5000, 3, 7), (4097, 1, 256)):
        gen = torch.Generator().manual_seed(T + E)
        topi = torch.randint(0, E, (T, k), generator=gen).cuda()
        outs = []
        for use_scratch in (False, True):
            P = T * k
            perm = torch.full((P,), -1, dtype=torch.int32, device="cuda")
            inv = torch.full((P,), -1, dtype=torch.int32, device="cuda")
            seg = torch.empty(E + 1, dtype=torch.int32, device="cuda")
            active = torch.empty(E + 1, dtype=torch.int32, device="cuda")
            nbytes = int(_lib.load().skcq_route_sort_scratch_bytes(T, k, E)) if use_scratch else 0
            assert not use_scratch or nbytes > 0
            scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
            call("skcq_route_sort", ptr(topi), T, k, E, ptr(perm), ptr(seg), ptr(inv), ptr(active),
                 ptr(scratch) if use_scratch else None, nbytes, 0, stream())
            outs.append((perm.cpu(), inv.cpu(), seg.cpu(), active.cpu()))
        for a, b in zip(outs[0], outs[1]):
            assert torch.equal(a, b)
        perm, inv = outs[0][0].long(), outs[0][1].long()
        # stable by expert: the reference order of torch.where(expert_mask[e]) (pair = kpos * T + token)
        expert = topi.cpu().t().reshape(-1)
        ref = torch.sort(expert, stable=True).indices
        assert torch.equal(perm, ref)
        assert torch.equal(inv[perm], torch.arange(T * k))


def test_prefill_persistent_gemm_many_tiles():
    """More (row tile, output tile) items than SMs: every persistent CTA walks
    several items, alternating its two TMEM accumulators and carrying the
    stage ring across items; results agree with the fp32 gather path."""
    E, H, I, T, k = 8, 256, 512, 8192, 2
    ex, x, topi, topw = _prefill_case(E, H, I, T, k, [(8, 64, True), (4, 64, False)], [(8, 64, True)], seed=606)
    assert ex._use_prefill(x, T * k, E)
    y_tc = ex(x, topi, topw).double()
    ex.prefill_min_rows = 1 << 30
    y_ref = ex(x, topi, topw).double()
    cos = torch.nn.functional.cosine_similarity(y_tc.flatten(), y_ref.flatten(), dim=0).item()
    assert cos >= 0.9999, cos
    assert (y_tc - y_ref).abs().max().item() <= 1e-2 * y_ref.abs().max().item()


def _upcast_module(mod):
    """The same codebook module with its codebooks, scales and remainder
    upcast to f32 (exact), sign buffers and indices shared."""
    from skcq_b200.codebook_experts import CodebookModule, _CodebookLayer

    layers = []
    for lay in mod.layers:
        layers.append(_CodebookLayer(
            lay.codebook.detach().float(), lay.assignments, lay.n_blocks, lay.block_size, lay.out_dim, lay.k,
            remainder=lay.remainder.float() if lay.rem else None,
            signs=lay.signs,
            scales=lay.scales.detach().float() if lay.scales is not None else None,
        ))
    return CodebookModule(torch.nn.ModuleList(layers), len(layers), mod.out_dim).cuda()


@pytest.mark.parametrize("case", ["base", "ragged", "signs", "bench_shapes"])
def test_prefill_dequant_fast_path_is_bit_identical(case):
    """The register fast path of skcq_prefill_dequant (bf16 tables, block
    sizes 4 / 8 / 16) writes the same operand-image bits as the
    shared-memory decoder does for the same module in f32 (taken for f32
    tables): same scale * sign * centroid products and the same per-column
    order of layers, for whole 256-output images, for the gate/up interleaved
    halves and for an active-expert list."""
    E, out, inp, specs = {
        "base": (4, 512, 256, [(8, 64, True), (16, 64, False), (4, 256, False)]),
        # out not a multiple of 256, in not a multiple of 64, remainder columns
        "ragged": (3, 300, 200, [(8, 32, True), (16, 64, False), (4, 128, False)]),
        "signs": (3, 256, 128, [(8, 32, True), (16, 32, False)]),
        # the benchmark layer's codebooks (16-bit indices above 32767)
        "bench_shapes": (2, 768, 2048, [(8, 4096, True), (16, 4096, False), (4, 65536, False)]),
    }[case]
    mod = _random_module(E, out, inp, specs, seed=808, dtype=torch.bfloat16)
    if case == "signs":
        lay = mod.layers[0]
        g = torch.Generator().manual_seed(809)
        lay.signs = torch.where(torch.rand(E, out, lay.n_blocks * lay.block_size, generator=g) < 0.5, -1,
                                1).to(torch.int8).cuda()
        lay.sign_cov = lay.signs.shape[-1]
    ref = _upcast_module(mod)
    KC = -(-inp // 64)
    active = torch.tensor([E - 1, *range(E - 1, 0, -1)], dtype=torch.int32, device="cuda")  # all but expert 0
    for half, slots, act in ((-1, E, None), (0, E - 1, active), (1, E - 1, active)):
        NT = -(-out // (256 if half < 0 else 128))
        imgs = []
        for m in (mod, ref):
            W = torch.full((slots * NT * KC * 16384,), -7.0, dtype=torch.bfloat16, device="cuda")
            m.dequant_into(W, act, slots, inp, half)
            imgs.append(W.view(torch.int16))
        torch.cuda.synchronize()
        assert torch.equal(imgs[0], imgs[1]), (half, (imgs[0] != imgs[1]).sum().item())


@pytest.mark.parametrize("T", [1, 3, 8, 24])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_lookup_table_is_bit_identical(T, dtype):
    """The lookup-table decode (codebook_experts.py:57-60, matmul_gather) reads
    per-token block dots built with the same fused multiply-adds the gather
    path forms, so the MoE block's output is the same bits with the tables on
    every sign-free layer, on none, or where the automatic policy puts them;
    the last codebook carries a 13-column remainder."""
    from skcq_b200.codebook_experts import CodebookExperts

    E, H, I, k = 8, 2061, 96, 4
    specs = [(8, 256, True), (16, 512, False), (4, 1024, False)]
    ex = CodebookExperts(_random_module(E, I, H, specs, seed=11, dtype=dtype),
                         _random_module(E, I, H, specs, seed=12, dtype=dtype),
                         _random_module(E, H, I, [(8, 256, True), (4, 512, False)], seed=13, dtype=dtype), E,
                         torch.nn.functional.silu)
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, H, generator=g).to(dtype).cuda()
    topi = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).cuda()
    topw = torch.softmax(torch.randn(T, k, generator=g), -1).cuda()
    outs = {}
    for mode in ("off", "on", "auto"):
        ex.decode_lut = mode
        outs[mode] = ex(x, topi, topw)
    assert torch.equal(outs["on"], outs["off"])
    assert torch.equal(outs["auto"], outs["off"])
    ex.decode_lut = "on"
    assert ex._lut_layers(ex.gate, T, T * k) == [True, True, True]


def test_decode_lookup_table_skips_signed_layers():
    """A layer with SSVQ signs cannot use a table of plain dots (the reference
    switches such layers to gather_matmul, codebook_experts.py:50-51): the
    policy leaves it out, and the C ABI rejects a signed layer that carries
    one."""
    from skcq_b200 import _lib
    from skcq_b200._lib import ptr, stream
    from skcq_b200.codebook_experts import CodebookExperts, FwdLayer

    E, H, I = 4, 64, 32
    gate = _random_module(E, I, H, [(8, 64, True)], seed=21)
    gate.layers[0].signs = torch.where(torch.rand(E, I, H, generator=torch.Generator().manual_seed(2)) < 0.5, -1,
                                       1).to(torch.int8).cuda()
    ex = CodebookExperts(gate, _random_module(E, I, H, [(8, 64, True)], seed=22),
                         _random_module(E, H, I, [(8, 64, True)], seed=23), E, torch.nn.functional.silu)
    ex.decode_lut = "on"
    assert ex._lut_layers(ex.gate, 2, 8) is None
    d = gate.layers[0].descriptor(torch.device("cuda"), primary=True)
    lut = torch.zeros(8 * 64 * 2, device="cuda")
    d.lut, d.lut_tokens = ptr(lut), 2
    arr = (FwdLayer * 1)(d)
    x = torch.randn(2, H, device="cuda")
    seg = torch.tensor([0, 2], dtype=torch.int32, device="cuda")
    part = torch.empty(1, 2, I, device="cuda")
    rc = _lib.load().skcq_codebook_forward(_lib.C.cast(arr, _lib.C.c_void_p), 1, ptr(x), 0, x.stride(0), None, 2,
                                           ptr(seg), None, None, 1, 1, H, I, 1, 2, ptr(part), 2, stream())
    assert rc != 0 and "signs" in _lib.last_error()
