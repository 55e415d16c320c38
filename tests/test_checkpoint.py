"""Checkpoint loading into the packed bank (CPU): a synthetic two-shard HF
safetensors checkpoint in the GLM-5 key layout, read back bit for bit."""

import json
import math

import pytest
import torch

from glm53_flash_mlx_b200 import checkpoint as C
from glm53_flash_mlx_b200 import synthetic as S

PREFIX = "model.language_model"
F8 = torch.float8_e4m3fn


def _codes(rows, cols, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 256, (rows, cols), generator=g, dtype=torch.uint8)


def _scales(rows, cols, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.rand((math.ceil(rows / 128), math.ceil(cols / 128)), generator=g) * 0.01


def _write_checkpoint(root, *, layers=(1, 3), E=5, H=256, I=128, Is=128, router_dtype=torch.bfloat16,
                      shards=2, mutate=None):
    """Returns the expected tensors {key: tensor} and writes the shards."""
    from safetensors.torch import save_file

    tensors = {}
    for L in layers:
        base = f"{PREFIX}.layers.{L}.mlp"
        for e in range(E):
            for proj, (r, c) in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
                seed = 1000 * L + 10 * e + len(proj)
                tensors[f"{base}.experts.{e}.{proj}.weight"] = _codes(r, c, seed).view(F8)
                tensors[f"{base}.experts.{e}.{proj}.weight_scale_inv"] = _scales(r, c, seed + 1)
        for proj, (r, c) in (("gate_proj", (Is, H)), ("up_proj", (Is, H)), ("down_proj", (H, Is))):
            tensors[f"{base}.shared_experts.{proj}.weight"] = _codes(r, c, 7 * L + len(proj)).view(F8)
            tensors[f"{base}.shared_experts.{proj}.weight_scale_inv"] = _scales(r, c, 7 * L + 3)
        g = torch.Generator().manual_seed(L)
        tensors[f"{base}.gate.weight"] = (torch.randn((E, H), generator=g) * 0.01).to(router_dtype)
        tensors[f"{base}.gate.e_score_correction_bias"] = torch.randn((E,), generator=g) * 0.1
    tensors["model.language_model.embed_tokens.weight"] = torch.zeros((8, H), dtype=torch.bfloat16)
    if mutate:
        mutate(tensors)
    keys = sorted(tensors)
    weight_map = {}
    for s in range(shards):
        name = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        part = {k: tensors[k].contiguous() for k in keys[s::shards]}
        save_file(part, str(root / name))
        weight_map.update({k: name for k in part})
    (root / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    return tensors


def test_bank_router_and_shared_expert_read_back_exactly(tmp_path):
    E, H, I = 5, 256, 128
    t = _write_checkpoint(tmp_path, E=E, H=H, I=I)
    idx = C.CheckpointIndex(tmp_path)
    assert idx.prefix() == PREFIX
    assert idx.moe_layers() == [1, 3]
    for L in (1, 3):
        bank = C.load_packed_bank(idx, L, device="cpu")
        assert (bank.expert_count, bank.hidden_size, bank.intermediate_size) == (E, H, I)
        base = f"{PREFIX}.layers.{L}.mlp.experts"
        for e in range(E):
            gu = bank.gate_up_weight[e]
            assert torch.equal(gu[:I], t[f"{base}.{e}.gate_proj.weight"].view(torch.uint8))
            assert torch.equal(gu[I:], t[f"{base}.{e}.up_proj.weight"].view(torch.uint8))
            assert torch.equal(bank.down_weight[e], t[f"{base}.{e}.down_proj.weight"].view(torch.uint8))
            assert torch.equal(bank.gate_up_scale_inv[e, :1], t[f"{base}.{e}.gate_proj.weight_scale_inv"])
            assert torch.equal(bank.gate_up_scale_inv[e, 1:], t[f"{base}.{e}.up_proj.weight_scale_inv"])
            assert torch.equal(bank.down_scale_inv[e], t[f"{base}.{e}.down_proj.weight_scale_inv"])
        cfg = S.moe_config(H, I, E, 2, 7.0)
        gate = C.load_router(idx, L, cfg, device="cpu")
        assert gate.weight.dtype == torch.float32
        assert torch.equal(gate.weight, t[f"{PREFIX}.layers.{L}.mlp.gate.weight"].float())
        assert torch.equal(gate.e_score_correction_bias, t[f"{PREFIX}.layers.{L}.mlp.gate.e_score_correction_bias"])
        shared = C.load_shared_expert(idx, L, limit=7.0, device="cpu")
        sb = f"{PREFIX}.layers.{L}.mlp.shared_experts"
        for proj in ("gate_proj", "up_proj", "down_proj"):
            assert torch.equal(getattr(shared, proj).weight, t[f"{sb}.{proj}.weight"].view(torch.uint8))
            assert torch.equal(getattr(shared, proj).weight_scale_inv, t[f"{sb}.{proj}.weight_scale_inv"])
        moe = C.load_packed_moe(idx, L, cfg, device="cpu")
        assert moe.bank.expert_count == E and moe.shared_experts is not None


def test_single_file_checkpoint_without_index(tmp_path):
    from safetensors.torch import save_file

    t = _write_checkpoint(tmp_path, layers=(0,), E=2, shards=1)
    one = tmp_path / "one.safetensors"
    save_file({k: v.contiguous() for k, v in t.items()}, str(one))
    bank = C.load_packed_bank(one, 0, device="cpu")
    assert bank.expert_count == 2


@pytest.mark.parametrize(
    "mutate,match",
    [
        (lambda t: t.pop(f"{PREFIX}.layers.1.mlp.experts.2.up_proj.weight"), "missing"),
        (lambda t: t.__setitem__(f"{PREFIX}.layers.1.mlp.experts.1.down_proj.weight",
                                 torch.zeros((256, 128), dtype=torch.bfloat16)), "E4M3"),
        (lambda t: t.__setitem__(f"{PREFIX}.layers.1.mlp.experts.0.gate_proj.weight_scale_inv",
                                 torch.ones((2, 2))), "scale shape"),
        (lambda t: t.__setitem__(f"{PREFIX}.layers.1.mlp.experts.3.gate_proj.weight",
                                 torch.zeros((128, 128), dtype=torch.uint8)), "shape"),
        (lambda t: [t.pop(k) for k in list(t) if ".experts.4." in k and ".layers.1." in k] and
         [t.__setitem__(k.replace(".experts.3.", ".experts.6."), t.pop(k)) for k in list(t)
          if ".experts.3." in k and ".layers.1." in k], "not 0.."),
    ],
)
def test_bank_loading_fails_closed(tmp_path, mutate, match):
    _write_checkpoint(tmp_path, layers=(1,), mutate=mutate)
    with pytest.raises(ValueError, match=match):
        C.load_packed_bank(tmp_path, 1, device="cpu")


def test_router_shape_mismatch_and_missing_shared_expert(tmp_path):
    def drop_shared(t):
        for k in [k for k in t if ".shared_experts." in k]:
            t.pop(k)

    _write_checkpoint(tmp_path, layers=(2,), E=5, mutate=drop_shared)
    idx = C.CheckpointIndex(tmp_path)
    assert C.load_shared_expert(idx, 2, limit=7.0, device="cpu") is None
    with pytest.raises(ValueError, match="does not match the gate"):
        C.load_router(idx, 2, S.moe_config(256, 128, 6, 2, 7.0), device="cpu")


@pytest.mark.gpu
def test_loaded_layer_decodes_on_gpu_like_the_oracle(tmp_path, oracle):
    """A checkpoint layer loaded onto the GPU runs PackedFP8MoE's one-token decode;
    the result matches the oracle on the same (loaded) tensors."""
    import zlib

    import numpy as np

    from gpu_util import assert_layer_close, bank_host, bits, certify_packed_decode, shared_host
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    E, H, I = 8, 512, 256

    def realistic(t):  # quantised N(0, 0.02) codes instead of raw random bytes
        for k in list(t):
            if k.endswith("_proj.weight"):
                r, c = t[k].shape
                w, s = S.random_block_fp8(r, c, seed=zlib.crc32(k.encode()) % 10_000, tensor=1)
                t[k] = w.view(F8)
                t[k + "_scale_inv"] = s

    _write_checkpoint(tmp_path, layers=(0,), E=E, H=H, I=I, Is=I, router_dtype=torch.float32, mutate=realistic)
    cfg = S.moe_config(H, I, E, 8, 10.0)
    moe = C.load_packed_moe(tmp_path, 0, cfg, device="cuda")
    for t in range(3):
        x = S.random_bf16((1, 1, H), seed=50 + t, device="cuda")
        out = moe(x)  # one token: router + decode in one library call (the step's workspace)
        idx, sc = moe.gate(x)
        torch.cuda.synchronize()
        ids = idx.reshape(-1).cpu().numpy().astype(np.uint32)
        scs = sc.reshape(-1).cpu().numpy()
        hb, hs = bank_host(moe.bank), shared_host(shared_fp8_tensors(moe.shared_experts))
        ref = oracle.packed_decode_moe(bits(x.reshape(-1)), ids, scs, hb, hs, 10.0)
        cert = certify_packed_decode(bits(x.reshape(-1)), ids, scs, hb, hs, 10.0, bits(out.reshape(-1)),
                                     moe._workspace._buffers[(x.device, "step_decode")])
        assert_layer_close(bits(out.reshape(-1)), ref, certificate=cert)
