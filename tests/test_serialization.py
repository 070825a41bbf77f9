"""On-disk codebooks (build.py:30-106): the reference's directory layout and
files, the packed format's exact round trip, and replace_experts."""

from __future__ import annotations

import types

import torch

from skcq_b200 import codebook as cb
from skcq_b200.codebook.cwr import AQLMCWR, EuclideanCWR, SphericalCWR, SSVQCWR
from skcq_b200.codebook_experts import CodebookExperts, CodebookModule
from skcq_b200.serialization import (load_codebooks, load_packed, modules_from_results, replace_experts,
                                     save_codebooks, save_packed)

E, OUT, IN = 4, 8, 13  # in_dim 13: a remainder column after blocks of 4


def _result(seed: int, ssvq: bool):
    """A hand-made (AQLMCodebook, AQLMCWR) pair: spherical primary (optionally
    sign-split) bs=4 K=16 + euclidean residual bs=4 K=65536 (16-bit indices)."""
    g = torch.Generator().manual_seed(seed)
    rows, nb = E * OUT, IN // 4
    sph = cb.SphericalCodebook(cb.SphericalCodebookConfig(block_size=4, K=16))
    sph.directions = torch.randn(nb, 4, 16, generator=g).to(torch.bfloat16)
    euc = cb.EuclideanCodebook(cb.EuclideanCodebookConfig(block_size=4, K=65536))
    euc.centroids = torch.randn(nb, 4, 65536, generator=g).to(torch.bfloat16)
    prim_cwr = SphericalCWR(idxs=torch.randint(0, 16, (nb, rows), generator=g),
                            scales=torch.rand(rows, nb, generator=g),
                            remainder=torch.randn(rows, 1, generator=g).to(torch.bfloat16))
    res_cwr = EuclideanCWR(idxs=torch.randint(0, 65536, (nb, rows), generator=g),
                           remainder=torch.randn(rows, 1, generator=g).to(torch.bfloat16))
    primary = sph
    if ssvq:
        primary = cb.SSVQCodebook(sph)
        signs = torch.where(torch.rand(rows, IN, generator=g) < 0.5, -1, 1).to(torch.int8)
        prim_cwr = SSVQCWR(inner=prim_cwr, signs=signs[:, : nb * 4].contiguous())
    aqlm = cb.AQLMCodebook(primary, [euc], cb.AQLMCodebookConfig(out_dim=OUT, num_experts=E))
    return aqlm, AQLMCWR(primary=prim_cwr, residuals=[res_cwr])


def _same_state(a: CodebookModule, b: CodebookModule) -> None:
    sa, sb = a.state_dict(), b.state_dict()
    assert sa.keys() == sb.keys()
    for k in sa:
        assert sa[k].dtype == sb[k].dtype, k
        assert torch.equal(sa[k], sb[k]), k


def test_save_and_load_codebooks_layout(tmp_path):
    results = [{"gate": _result(1, True), "up": _result(2, False), "down": _result(3, False)},
               {"gate": _result(4, False), "up": _result(5, True), "down": _result(6, False)}]
    save_codebooks(results, tmp_path / "cb")
    for i in range(2):
        for name in ("gate", "up", "down"):
            data = torch.load(tmp_path / "cb" / f"layer_{i}" / f"{name}.pt", weights_only=True)
            assert set(data) == {"state_dict", "meta"}
            assert data["meta"]["num_experts"] == E and data["meta"]["out_dim"] == OUT
    loaded = load_codebooks(tmp_path / "cb", 2)
    built = modules_from_results(results)
    for i in range(2):
        for name in ("gate", "up", "down"):
            # the reference's load goes through empty() (bf16 floats), as here
            ref = built[i][name].to(torch.bfloat16)
            _same_state(loaded[i][name], ref)


def test_packed_round_trip_exact_and_smaller(tmp_path):
    aqlm, cwr = _result(7, True)
    mod = CodebookModule.from_cwr(aqlm, cwr, out_dim=OUT)
    save_packed(mod, tmp_path / "m.pkd")
    torch.save(mod.state_dict_with_meta(), tmp_path / "m.pt")
    back = load_packed(tmp_path / "m.pkd")
    _same_state(back, mod)
    assert back.layers[1].assignments.max().item() > 32767  # the 16-bit wrap is undone
    assert (tmp_path / "m.pkd").stat().st_size < (tmp_path / "m.pt").stat().st_size


def test_replace_experts_installs_codebook_experts():
    results = [{"gate": _result(11, False), "up": _result(12, False), "down": _result(13, False)}]
    mods = modules_from_results(results)
    act = torch.nn.functional.silu
    experts = torch.nn.Module()
    experts.w = torch.nn.Parameter(torch.zeros(1))
    experts.act_fn = act
    layer = types.SimpleNamespace(mlp=types.SimpleNamespace(experts=experts))
    model = types.SimpleNamespace(model=types.SimpleNamespace(layers=[layer]))
    replace_experts(model, mods, num_experts=E)
    new = layer.mlp.experts
    assert isinstance(new, CodebookExperts)
    assert new.gate is mods[0]["gate"] and new.down is mods[0]["down"] and new.num_experts == E
    assert new.intermediate.act_fn is act
