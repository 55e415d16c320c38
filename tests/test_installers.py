"""Layer installers (mirrors tests/test_fp8_metal.py:241-329; CPU only --
packing and module swaps need no kernel)."""

from types import SimpleNamespace

import torch

from glm53_flash_mlx_b200.fp8 import DirectFP8MoE
from glm53_flash_mlx_b200.grouped_fp8 import SortedGroupedFP8MoE
from glm53_flash_mlx_b200.loader import install_packed_decode_moe, install_packed_grouped_moe
from glm53_flash_mlx_b200.packed import PackedFP8MoE


class _Gate(torch.nn.Module):
    def forward(self, x):
        shape = (*x.shape[:-1], 2)
        return torch.zeros(shape, dtype=torch.int32), torch.ones(shape, dtype=x.dtype)


def _model(n_layers):
    config = SimpleNamespace(hidden_size=128, moe_intermediate_size=128, swiglu_limit=3.0, n_routed_experts=2,
                             num_experts_per_tok=2)
    layers = [SimpleNamespace(mlp=DirectFP8MoE(config, _Gate(), None), compile_ffn=True) for _ in range(n_layers)]
    return SimpleNamespace(language_model=SimpleNamespace(model=SimpleNamespace(layers=layers))), layers


def test_installer_replaces_every_direct_moe_layer_one_at_a_time():
    model, layers = _model(3)
    report = install_packed_grouped_moe(model)
    assert report["converted_layers"] == [0, 1, 2]
    assert report["converted_count"] == 3
    assert report["remaining_direct_layers"] == []
    assert report["all_old_expert_modules_detached"]
    assert report["layers"][0]["bank_bytes"] == 2 * (256 * 128 + 2 * 1 * 4 + 128 * 128 + 1 * 1 * 4)
    assert all(isinstance(layer.mlp, SortedGroupedFP8MoE) for layer in layers)
    assert all(not hasattr(layer.mlp, "experts") for layer in layers)
    assert all(not layer.compile_ffn for layer in layers)
    second = install_packed_grouped_moe(model)
    assert second["converted_count"] == 0
    assert second["remaining_direct_layers"] == []


def test_packed_decode_installer_never_installs_grouped_modules():
    model, layers = _model(2)
    report = install_packed_decode_moe(model)
    assert report["backend"] == "packed-decode"
    assert report["grouped_enabled"] is False
    assert report["converted_count"] == 2
    assert report["all_old_expert_modules_detached"]
    assert all(isinstance(layer.mlp, PackedFP8MoE) for layer in layers)
    assert all(not isinstance(layer.mlp, SortedGroupedFP8MoE) for layer in layers)
    assert model._glm53_moe_backend == "packed-decode"
    assert model._glm53_packed_decode_report is report
    assert install_packed_decode_moe(model)["converted_count"] == 0


def test_bank_pack_shapes_match_reference_known_answer():
    import json
    from pathlib import Path

    from glm53_flash_mlx_b200.packed import PackedFP8ExpertBank

    kat = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())["bank_shapes"]
    cfg = SimpleNamespace(hidden_size=kat["hidden_size"], moe_intermediate_size=kat["intermediate_size"],
                          swiglu_limit=3.0, n_routed_experts=kat["experts"], num_experts_per_tok=8)
    direct = DirectFP8MoE(cfg, _Gate(), None)
    g = torch.Generator().manual_seed(0)
    for e in direct.experts:
        for p in (e.gate_proj, e.up_proj, e.down_proj):
            p.weight = torch.randint(0, 247, p.weight.shape, generator=g, dtype=torch.int32).to(torch.uint8)
            p.weight_scale_inv = torch.rand(p.weight_scale_inv.shape, generator=g) * 0.002
    bank = PackedFP8ExpertBank.pack(direct.experts)
    for name, shape in kat["shapes"].items():
        assert list(getattr(bank, name).shape) == shape, name
    for i, e in enumerate(direct.experts):
        v = bank.expert(i, limit=3.0)
        assert torch.equal(v.gate_proj.weight, e.gate_proj.weight)
        assert torch.equal(v.up_proj.weight, e.up_proj.weight)
        assert torch.equal(v.down_proj.weight, e.down_proj.weight)
        assert torch.equal(v.gate_proj.weight_scale_inv, e.gate_proj.weight_scale_inv)
        assert torch.equal(v.up_proj.weight_scale_inv, e.up_proj.weight_scale_inv)
        assert torch.equal(v.down_proj.weight_scale_inv, e.down_proj.weight_scale_inv)
    import pytest

    with pytest.raises(IndexError):
        bank.expert(8, limit=3.0)
