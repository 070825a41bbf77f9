"""Weight ingest (worker.py:62-134): shard map, row extraction (whole layer
and an expert range), farm assignment; a farm fit of a tiny model on the GPU."""

from __future__ import annotations

import json

import pytest
import torch
from safetensors.torch import save_file

from skcq_b200.ingest import build_layer_shard_map, extract_rows, farm_assignment, farm_layers

E, H, I, L = 4, 12, 8, 3


def _model_dir(tmp_path):
    g = torch.Generator().manual_seed(0)
    weights, wmap = {}, {}
    for layer in range(L):
        gu = torch.randn(E, 2 * I, H, generator=g).to(torch.bfloat16)
        dn = torch.randn(E, H, I, generator=g).to(torch.bfloat16)
        weights[layer] = (gu, dn)
        shard_a, shard_b = f"model-a-{layer % 2}.safetensors", "model-b.safetensors"
        wmap[f"model.language_model.layers.{layer}.mlp.experts.gate_up_proj"] = shard_a
        wmap[f"model.language_model.layers.{layer}.mlp.experts.down_proj"] = shard_b
    wmap["model.language_model.embed_tokens.weight"] = "model-b.safetensors"
    files: dict[str, dict[str, torch.Tensor]] = {}
    for key, shard in wmap.items():
        if "embed" in key:
            t = torch.zeros(2, 2)
        else:
            layer = int(key.split(".")[3])
            t = weights[layer][0] if "gate_up" in key else weights[layer][1]
        files.setdefault(shard, {})[key] = t.contiguous()
    for shard, tensors in files.items():
        save_file(tensors, str(tmp_path / shard))
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wmap}))
    return tmp_path, weights


def test_shard_map_and_rows(tmp_path):
    d, weights = _model_dir(tmp_path)
    shards = build_layer_shard_map(d)
    assert set(shards) == set(range(L))
    assert shards[1] == {"gate_up": "model-a-1.safetensors", "down": "model-b.safetensors"}
    rows = extract_rows(d, 1, shards, E, H, I)
    gu, dn = weights[1]
    assert torch.equal(rows["gate"], gu[:, :I, :].reshape(-1, H))
    assert torch.equal(rows["up"], gu[:, I:, :].reshape(-1, H))
    assert torch.equal(rows["down"], dn.reshape(-1, I))
    part = extract_rows(d, 1, shards, E, H, I, experts=(1, 3))
    assert torch.equal(part["gate"], rows["gate"][1 * I:3 * I])
    assert torch.equal(part["down"], rows["down"][1 * H:3 * H])
    with pytest.raises(ValueError):
        extract_rows(d, 1, shards, E, H, I, experts=(3, 5))


def test_farm_assignment_covers_layers_once():
    for n, w in ((48, 8), (5, 2), (3, 4)):
        got = sorted(x for r in range(w) for x in farm_assignment(n, w, r))
        assert got == list(range(n))


@pytest.mark.gpu
def test_farm_fits_tiny_model(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from skcq_b200.config import CodebookParams

    d, weights = _model_dir(tmp_path)
    params = CodebookParams(k_gate=16, k_up=16, k_down=16, n_blocks_gate_up=3, n_blocks_down=2, max_iters=5,
                            norm_threshold=1e-9, skip_zeros=False, residual_k=8)
    res = farm_layers(d, params, L, E, H, I, rank=1, world=2)
    assert sorted(res) == [1]
    aqlm, cwr = res[1]["down"]
    w = weights[1][1].reshape(-1, I).float()
    rel = (aqlm.reconstruct(cwr).cpu() - w).norm() / w.norm()
    assert rel < 0.6


class _FlakyCodebook:
    """Stand-in for an AQLM codebook whose fit fails with a device wait that
    ran out on the first ``fail`` attempts of each job (host-side injection:
    nothing runs on a GPU)."""

    attempts: dict[str, int] = {}
    fail = 1

    def __init__(self, name: str) -> None:
        self.name = name

    def fit(self, w):
        from skcq_b200.errors import DeviceTimeoutError

        n = _FlakyCodebook.attempts.get(self.name, 0) + 1
        _FlakyCodebook.attempts[self.name] = n
        if n <= _FlakyCodebook.fail:
            raise DeviceTimeoutError(f"{self.name}: device-side check failed (code 15)", 15)
        return ("cwr", self.name, n)


def _flaky_builder(*args, name="", **kw):
    return _FlakyCodebook(name)


def test_farm_retries_a_job_after_a_device_timeout(tmp_path, monkeypatch):
    """A (layer, projection) job whose fit raises DeviceTimeoutError is fitted
    again from a fresh codebook and the farm completes (worker.py:256-258
    reports such a job for another attempt)."""
    import skcq_b200.ingest as ingest
    from skcq_b200.config import CodebookParams

    d, _ = _model_dir(tmp_path)
    monkeypatch.setattr(ingest, "build_aqlm_codebook", _flaky_builder)
    _FlakyCodebook.attempts, _FlakyCodebook.fail = {}, 1
    res = farm_layers(d, CodebookParams(), L, E, H, I, rank=0, world=2, device="cpu", retries=2)
    assert sorted(res) == [0, 2]
    for layer in (0, 2):
        for proj in ("gate", "up", "down"):
            assert res[layer][proj][1] == ("cwr", f"L{layer}.{proj}", 2)
    assert all(n == 2 for n in _FlakyCodebook.attempts.values())


def test_farm_gives_up_after_the_retries_with_the_job_in_context(tmp_path, monkeypatch):
    import skcq_b200.ingest as ingest
    from skcq_b200.config import CodebookParams
    from skcq_b200.errors import InfrastructureError

    d, _ = _model_dir(tmp_path)
    monkeypatch.setattr(ingest, "build_aqlm_codebook", _flaky_builder)
    _FlakyCodebook.attempts, _FlakyCodebook.fail = {}, 5
    with pytest.raises(InfrastructureError) as ei:
        farm_layers(d, CodebookParams(), L, E, H, I, rank=0, world=1, device="cpu", retries=2)
    assert ei.value.context["layer"] == 0 and ei.value.context["projection"] == "gate"
    assert ei.value.context["attempts"] == 3 and ei.value.context["device_code"] == 15
    assert _FlakyCodebook.attempts == {"L0.gate": 3}


def test_farm_does_not_retry_bugs(tmp_path, monkeypatch):
    import skcq_b200.ingest as ingest
    from skcq_b200.config import CodebookParams

    calls = []

    class Broken:
        def __init__(self, name):
            self.name = name

        def fit(self, w):
            calls.append(self.name)
            raise RuntimeError("a bug")

    d, _ = _model_dir(tmp_path)
    monkeypatch.setattr(ingest, "build_aqlm_codebook", lambda *a, name="", **k: Broken(name))
    with pytest.raises(RuntimeError, match="a bug"):
        farm_layers(d, CodebookParams(), L, E, H, I, rank=0, world=1, device="cpu", retries=3)
    assert calls == ["L0.gate"]
