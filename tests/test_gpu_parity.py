"""CUDA path vs the CPU oracle on seeded inputs (needs a B200: -m gpu)."""

import ctypes
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from gpu_util import (MAX_ABS, assert_layer_close, bank_host, bits, certify_by_envelope, certify_expert_rows,
                      certify_grouped, certify_grouped_f8, certify_grouped_linear, certify_linear,
                      certify_packed_decode, check_grouped_route_plan, direct_combine, f32, from_bits,
                      router_logit_check, shared_host)

pytestmark = pytest.mark.gpu
KATS = json.loads((Path(__file__).resolve().parent / "golden" / "reference_kats.json").read_text())


@pytest.fixture(scope="module")
def G():
    import glm53_flash_mlx_b200 as G

    return G


@pytest.fixture(scope="module")
def N():
    from glm53_flash_mlx_b200 import _native as N

    N.lib()
    return N


@pytest.fixture(scope="module")
def S():
    from glm53_flash_mlx_b200 import synthetic as S

    return S


# ---------------------------------------------------------------------------
# BF16 SwiGLU sigmoid: the reference's all-BF16 sweep, bit for bit
# ---------------------------------------------------------------------------


def test_sigmoid_sweep_bit_exact_on_gpu(N, oracle):
    kat = KATS["sigmoid_sweep"]
    allbits = np.arange(1 << 16, dtype=np.uint16)
    vals = f32(allbits)
    dom = allbits[np.isfinite(vals) & (np.abs(vals) <= np.float32(10.0))]
    g = from_bits(dom)
    out = torch.empty_like(g)
    N.check(N.lib().glm53_sigmoid_bf16(g.data_ptr(), g.numel(), out.data_ptr(), N.stream()), "sigmoid")
    torch.cuda.synchronize()
    got = bits(out)
    assert hashlib.sha256(got.tobytes()).hexdigest() == kat["reference_sigmoid_sha256"]
    # and beyond the pinned domain (g < -10) GPU and oracle agree
    neg = allbits[np.isfinite(vals) & (vals < -10.0)]
    out2 = torch.empty(neg.size, dtype=torch.bfloat16, device="cuda")
    N.check(N.lib().glm53_sigmoid_bf16(from_bits(neg).data_ptr(), neg.size, out2.data_ptr(), N.stream()), "sigmoid")
    assert np.array_equal(bits(out2), oracle.sigmoid_bf16(neg))


# ---------------------------------------------------------------------------
# block_fp8_linear
# ---------------------------------------------------------------------------


@pytest.mark.parametrize(
    "M,N_,K",
    [(1, 129, 257), (2, 129, 257), (1, 256, 4096), (3, 384, 1024), (8, 512, 2048), (16, 256, 256),
     (17, 256, 512), (64, 256, 512), (200, 384, 1024), (1, 6144, 4096),
     # two tile groups per block (eight / five staged rows at K = 4096), an odd tile count
     (8, 6144, 4096), (5, 1040, 4096), (16, 4096, 4096)],
)
def test_block_linear_matches_oracle(G, S, oracle, M, N_, K):
    w, s = S.random_block_fp8(N_, K, seed=M * 1000 + N_, device="cuda")
    x = S.random_bf16((M, K), seed=K, device="cuda")
    y = G.block_fp8_linear(x, w, s)
    torch.cuda.synchronize()
    ref = oracle.block_fp8_linear(bits(x), w.cpu().numpy(), s.cpu().numpy())
    cert = certify_linear(bits(x), w.cpu().numpy(), s.cpu().numpy(), bits(y))
    stats = assert_layer_close(bits(y), ref, certificate=cert)
    assert stats["bit_identical"] >= 0.97, stats  # only summation-order rounding flips


def test_block_linear_reference_geometry_random_codes(G, oracle):
    """tests/test_fp8_metal.py:23-39: random codes 0..246 (includes 0x7F = 480)."""
    g = torch.Generator(device="cuda").manual_seed(5)
    codes = torch.randint(0, 247, (129, 257), generator=g, device="cuda", dtype=torch.int32).to(torch.uint8)
    scales = torch.rand((2, 3), generator=g, device="cuda") * 0.02
    x = torch.randn((2, 257), generator=g, device="cuda").to(torch.bfloat16)
    y = G.block_fp8_linear(x, codes, scales)
    lut = oracle.e4m3_table()
    dense = lut[codes.cpu().numpy()] * np.repeat(np.repeat(scales.cpu().numpy(), 128, 0), 128, 1)[:129, :257]
    expected = oracle.bf16_from_f32(f32(bits(x)) @ dense.T)
    assert np.abs(f32(bits(y)) - f32(expected)).max() <= 0.03125


def test_block_linear_fail_closed_checks(G):
    x = torch.zeros((1, 256), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((128, 256), dtype=torch.uint8, device="cuda")
    s = torch.ones((1, 2), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError, match="uint8"):
        G.block_fp8_linear(x, w.float(), s)
    with pytest.raises(ValueError, match="float32"):
        G.block_fp8_linear(x, w, s.double())
    with pytest.raises(ValueError, match="input width"):
        G.block_fp8_linear(x[:, :128], w, s)
    with pytest.raises(ValueError, match="block128"):
        G.block_fp8_linear(x, w, torch.ones((2, 2), device="cuda"))
    with pytest.raises(RuntimeError):
        G.block_fp8_linear(x.cpu(), w, s)
    y = G.block_fp8_linear(x[:0], w, s)
    assert y.shape == (0, 128)


# ---------------------------------------------------------------------------
# Router
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("T", [1, 2, 5, 8, 9, 16, 24, 32, 40, 64, 300])
def test_router_matches_oracle(G, S, oracle, T):
    E, H = 288, 4096
    w, b = S.make_router(E, H, seed=1, device="cuda", zipf_alpha=0.5 if T > 8 else 0.0)
    x = S.random_bf16((T, H), seed=T, device="cuda")
    idx, sc, logits = G.router_topk(x, w, b, top_k=8, return_logits=True)
    torch.cuda.synchronize()
    r_idx, r_sc, r_l64, margin = oracle.router(bits(x), w.cpu().numpy(), b.cpu().numpy(), top_k=8)
    stats = router_logit_check(logits.cpu().numpy(), r_l64, bits(x), w.cpu().numpy())
    print(f"[router T={T}] {stats}")
    if T <= 64:  # FP64 sums (per-expert CTAs up to 8 tokens, FP64 tensor-core tiles to 64): every logit
        # within 1e-6 relative of the FP64 oracle, none excepted
        assert stats["beyond_1e-6_relative_within_bound"] == 0, stats
    clear = margin > 1e-5
    assert clear.mean() > 0.9
    assert np.array_equal(idx.cpu().numpy()[clear].astype(np.uint32), r_idx[clear])
    np.testing.assert_allclose(sc.cpu().numpy()[clear], r_sc[clear], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("T,E,H", [(40, 16, 512), (100, 16, 256), (12, 16, 512), (70, 64, 1024)])
def test_router_small_width_matches_oracle(G, S, oracle, T, E, H):
    """Widths below the FP64 tensor-core tiles' 1024 and few expert tiles: the
    per-expert kernel up to 32 tokens, the BF16-split tcgen05 kernel above
    (its K ranges capped at one per 128-wide K block)."""
    w, b = S.make_router(E, H, seed=T + H, device="cuda")
    x = S.random_bf16((T, H), seed=T, device="cuda")
    idx, sc, logits = G.router_topk(x, w, b, top_k=8, return_logits=True)
    torch.cuda.synchronize()
    r_idx, r_sc, r_l64, margin = oracle.router(bits(x), w.cpu().numpy(), b.cpu().numpy(), top_k=8)
    stats = router_logit_check(logits.cpu().numpy(), r_l64, bits(x), w.cpu().numpy())
    assert stats["beyond_1e-6_relative_within_bound"] == 0 or T > 32, stats
    clear = margin > 1e-5
    assert np.array_equal(idx.cpu().numpy()[clear].astype(np.uint32), r_idx[clear])
    np.testing.assert_allclose(sc.cpu().numpy()[clear], r_sc[clear], rtol=1e-6, atol=1e-6)


def test_router_group_selection_matches_oracle(G, S, oracle):
    E, H, T = 64, 512, 16
    w, b = S.make_router(E, H, seed=3, device="cuda")
    x = S.random_bf16((T, H), seed=4, device="cuda")
    idx, sc = G.router_topk(x, w, b, top_k=6, n_group=8, topk_group=3, routed_scaling_factor=2.5)
    r_idx, r_sc, _, margin = oracle.router(bits(x), w.cpu().numpy(), b.cpu().numpy(), top_k=6, n_group=8,
                                           topk_group=3, routed_scaling_factor=2.5)
    clear = margin > 1e-5
    assert np.array_equal(idx.cpu().numpy()[clear].astype(np.uint32), r_idx[clear])
    np.testing.assert_allclose(sc.cpu().numpy()[clear], r_sc[clear], rtol=1e-6, atol=1e-6)


# ---------------------------------------------------------------------------
# Packed decode MoE
# ---------------------------------------------------------------------------


def _decode_case(S, E, H, I, seed, limit):
    bank = S.make_bank(E, H, I, seed=seed, device="cuda")
    shared = S.make_shared(H, I, seed=seed + 1, limit=limit, device="cuda")
    return bank, shared


@pytest.mark.parametrize("E,H,I,limit", [(8, 257, 129, 3.0), (8, 256, 128, 3.0), (16, 1024, 384, 10.0)])
def test_packed_decode_matches_oracle_small(G, S, oracle, E, H, I, limit):
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    bank, shared_mod = _decode_case(S, E, H, I, 11, limit)
    shared = shared_fp8_tensors(shared_mod)
    from glm53_flash_mlx_b200 import _native as N

    gen = np.random.default_rng(E + H)
    ws = N.Workspace()
    for trial in range(3):
        ids = gen.permutation(E)[:8].astype(np.int32)
        sc = gen.uniform(0.05, 0.3, 8).astype(np.float32)
        x = S.random_bf16((H,), seed=trial, device="cuda", std=2.0)
        out = G.packed_decode_moe(x, torch.from_numpy(ids).cuda(), torch.from_numpy(sc).cuda(), bank, shared,
                                  limit=limit, workspace=ws)
        torch.cuda.synchronize()
        ref = oracle.packed_decode_moe(bits(x), ids, sc, bank_host(bank), shared_host(shared), limit)
        cert = certify_packed_decode(bits(x), ids, sc, bank_host(bank), shared_host(shared), limit, bits(out),
                                     ws._buffers[(x.device, "decode")])
        stats = assert_layer_close(bits(out), ref, certificate=cert)
        assert stats["bit_identical"] >= 0.95, stats


def test_packed_decode_config2_full_size(G, S, oracle):
    """Config 2: H=4096, I=1536, 288 experts + shared, limit 10, routed by the
    FP32 router; oracle on the 8 touched experts."""
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    E, H, I = 288, 4096, 1536
    bank = S.make_bank(E, H, I, seed=1, device="cuda")
    shared = shared_fp8_tensors(S.make_shared(H, I, seed=2, device="cuda"))
    w, b = S.make_router(E, H, seed=3, device="cuda")
    from glm53_flash_mlx_b200 import _native as N

    ws = N.Workspace()
    for t in range(4):
        x = S.random_bf16((1, H), seed=100 + t, device="cuda")
        idx, sc = G.router_topk(x, w, b, top_k=8)
        out = G.packed_decode_moe(x[0], idx[0], sc[0], bank, shared, limit=10.0, workspace=ws)
        torch.cuda.synchronize()
        ids = idx[0].cpu().numpy()
        sub = bank_host(bank, ids)
        local = np.arange(8, dtype=np.uint32)
        ref = oracle.packed_decode_moe(bits(x[0]), local, sc[0].cpu().numpy(), sub, shared_host(shared), 10.0)
        cert = certify_packed_decode(bits(x[0]), local, sc[0].cpu().numpy(), sub, shared_host(shared), 10.0,
                                     bits(out), ws._buffers[(x.device, "decode")])
        stats = assert_layer_close(bits(out), ref, certificate=cert)
        print(f"[config2 token {t}] {stats} {cert}")
        assert stats["bit_identical"] >= 0.95, stats


def test_split_decode_matches_single_call_bitwise(G, S):
    """GLM53_FLAG_SHARED_ONLY on a side stream + GLM53_FLAG_SKIP_SHARED after
    the join give the bits of one glm53_packed_decode_moe call."""
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200.packed import packed_decode_moe, shared_fp8_tensors

    E, H, I = 16, 4096, 1536
    bank = S.make_bank(E, H, I, seed=71, device="cuda")
    shared = shared_fp8_tensors(S.make_shared(H, I, seed=72, device="cuda"))
    gen = torch.Generator().manual_seed(73)
    ws_full, ws_split = N.Workspace(), N.Workspace()
    side = torch.cuda.Stream()
    for t in range(3):
        x = S.random_bf16((H,), seed=74 + t, device="cuda")
        ids = torch.randperm(E, generator=gen)[:8].to(torch.int32).cuda()
        sc = (torch.rand(8, generator=gen) * 0.25 + 0.05).cuda()
        full = packed_decode_moe(x, ids, sc, bank, shared, limit=10.0, workspace=ws_full)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            packed_decode_moe(x, ids, sc, bank, shared, limit=10.0, workspace=ws_split, split="shared")
        torch.cuda.current_stream().wait_stream(side)
        part = packed_decode_moe(x, ids, sc, bank, shared, limit=10.0, workspace=ws_split, split="routed")
        torch.cuda.synchronize()
        assert torch.equal(full, part), t


@pytest.mark.parametrize("I", [1536, 2048])  # 12-warp and 16-warp overlapped gate/up CTAs
def test_decode_after_router_overlap_bitwise(G, S, I):
    """GLM53_FLAG_AFTER_ROUTER (gate/up launched as a programmatic dependent
    of the router, the shared expert streaming while the router runs) gives
    the bits of the serial launch: through the module (eager and as a CUDA
    graph of several layers back to back) and through the C-ABI."""
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200.packed import packed_decode_moe, shared_fp8_tensors
    from glm53_flash_mlx_b200.router import Float32Gate

    E, H = 64, 4096
    cfg = S.moe_config(H, I, E, 8, 10.0)
    mods = []
    for layer in range(3):
        gate = Float32Gate(cfg, device="cuda")
        w, b = S.make_router(E, H, seed=80 + layer, device="cuda")
        gate.weight.copy_(w)
        gate.e_score_correction_bias.copy_(b)
        mods.append(G.PackedFP8MoE(S.make_bank(E, H, I, seed=90 + layer, device="cuda"), cfg, gate,
                                   S.make_shared(H, I, seed=95 + layer, device="cuda")))

    def serial(m, x):
        idx, sc = m.gate(x)
        return packed_decode_moe(x.reshape(-1), idx.reshape(-1), sc.reshape(-1), m.bank,
                                 shared_fp8_tensors(m.shared_experts), limit=10.0, workspace=N.Workspace())

    xs = [S.random_bf16((1, 1, H), seed=100 + t, device="cuda") for t in range(6)]
    for t, x in enumerate(xs):  # module forward: the flag is set from the second call on
        for m in mods:
            got = m(x)
            assert torch.equal(got.reshape(-1), serial(m, x)), (t, "module")
    # raw C-ABI: router then decode with the flag, the same workspace every layer
    lib = N.lib()
    ws = N.Workspace()
    dws = ws.get(torch.device("cuda"), "d", lib.glm53_packed_decode_workspace_bytes(8, H, I, I))
    rws = ws.get(torch.device("cuda"), "r", lib.glm53_router_workspace_bytes(1, E))
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    idx = torch.empty(8, dtype=torch.int32, device="cuda")
    sc = torch.empty(8, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    for t, x in enumerate(xs):
        for m in mods:
            sh = shared_fp8_tensors(m.shared_experts)
            out = torch.empty(H, dtype=torch.bfloat16, device="cuda")
            N.check(lib.glm53_router_topk(x.data_ptr(), 1, H, m.gate.weight.data_ptr(), E,
                                          m.gate.e_score_correction_bias.data_ptr(), 8, 1, 1, 1, 1.0,
                                          idx.data_ptr(), sc.data_ptr(), None, rws.data_ptr(), rws.numel(), st), "r")
            N.check(lib.glm53_packed_decode_moe(
                x.data_ptr(), H, idx.data_ptr(), sc.data_ptr(), 8, m.bank.gate_up_weight.data_ptr(),
                m.bank.gate_up_scale_inv.data_ptr(), m.bank.down_weight.data_ptr(), m.bank.down_scale_inv.data_ptr(),
                E, I, *(p.data_ptr() for p in sh), I, 10.0, out.data_ptr(), dws.data_ptr(), dws.numel(),
                status.data_ptr(), N.FLAG_E4M3_FINITE | N.FLAG_AFTER_ROUTER, st), "d")
            assert torch.equal(out, serial(m, x)), (t, "c-abi")
    assert int(status.item()) == 0
    # CUDA graph: three layers chained, replayed over several inputs
    static_x = xs[0].clone()
    for m in mods:
        m(static_x)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        h = static_x
        outs = []
        for m in mods:
            outs.append(m(h))
    for t, x in enumerate(xs):
        static_x.copy_(x)
        g.replay()
        torch.cuda.synchronize()
        for m, o in zip(mods, outs):
            assert torch.equal(o.reshape(-1), serial(m, x)), (t, "graph")


def test_packed_moe_module_matches_direct_module_bitwise(G, S):
    """tests/test_fp8_metal.py:87-151: packed decode and 9-row prefill are
    bit-equal to the Direct module over the same expert tensors."""
    from types import SimpleNamespace

    routes = torch.tensor([[7, 1, 5, 0, 3, 6, 2, 4]], dtype=torch.int32, device="cuda")
    scores = torch.tensor([[0.24, 0.18, 0.15, 0.13, 0.11, 0.08, 0.06, 0.05]], device="cuda")

    class FixedGate(torch.nn.Module):
        def forward(self, x):
            shape = (*x.shape[:-1], 8)
            return routes.expand(shape), scores.expand(shape)

    config = SimpleNamespace(hidden_size=257, moe_intermediate_size=129, swiglu_limit=3.0, n_routed_experts=8,
                             num_experts_per_tok=8)
    direct = G.DirectFP8MoE(config, FixedGate(), None, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(7)
    for e in direct.experts:
        for p in (e.gate_proj, e.up_proj, e.down_proj):
            p.weight = torch.randint(0, 247, p.weight.shape, generator=g, device="cuda", dtype=torch.int32).to(
                torch.uint8)
            p.weight_scale_inv = torch.rand(p.weight_scale_inv.shape, generator=g, device="cuda") * 0.002
    bank = G.PackedFP8ExpertBank.pack(direct.experts)
    packed = G.PackedFP8MoE(bank, config, direct.gate, None)
    x = (torch.randn((1, 1, 257), generator=g, device="cuda") * 2).to(torch.bfloat16)
    assert torch.equal(packed(x), direct(x))
    xp = (torch.randn((1, 9, 257), generator=g, device="cuda") * 2).to(torch.bfloat16)
    assert torch.equal(packed(xp), direct(xp))


def test_packed_decode_flags_bad_expert_without_trapping(G, S):
    from glm53_flash_mlx_b200.packed import check_status

    bank, _ = _decode_case(S, 8, 256, 128, 5, 3.0)
    x = S.random_bf16((256,), seed=1, device="cuda")
    ids = torch.tensor([0, 1, 2, 3, 4, 5, 6, 99], dtype=torch.int32, device="cuda")
    sc = torch.full((8,), 0.125, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = G.packed_decode_moe(x, ids, sc, bank, None, limit=3.0, status=status)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    with pytest.raises(IndexError):
        check_status(status)
    with pytest.raises(ValueError):
        G.packed_decode_moe(x[:128], ids, sc, bank, None, limit=3.0)


# ---------------------------------------------------------------------------
# Route plan and grouped prefill
# ---------------------------------------------------------------------------


def _plan_gpu(ids, E, tile_rows, scores=None):
    from glm53_flash_mlx_b200.grouped_fp8 import _route_plan

    t = torch.from_numpy(ids.astype(np.int32)).cuda()
    s = None if scores is None else torch.from_numpy(scores).cuda()
    p = _route_plan(t, E, s, tile_rows)
    torch.cuda.synchronize()
    return {k: (v.cpu().numpy() if v is not None else None) for k, v in p.items()}


def test_route_plan_tile_descriptor_known_answer_on_gpu(G):
    kat = KATS["tile_descriptors"]
    se = torch.tensor([0] * 31 + [1] * 32 + [287] * 33, dtype=torch.int32, device="cuda")
    te, ts, tl, ro, to = (t.cpu().numpy() for t in G.build_grouped_tile_plan(se, 288))
    valid = ts < 96
    assert [list(map(int, t)) for t in zip(te[valid], ts[valid], tl[valid])] == kat["valid"]
    assert te.size == 3 + 288 and (te[~valid] == 0).all() and (ts[~valid] == 96).all() and (tl[~valid] == 0).all()


@pytest.mark.parametrize("R,E,tile_rows", [(96, 8, 32), (16384, 288, 32), (16384, 288, 128), (65536, 288, 128),
                                           (1000, 1024, 8), (1, 288, 128)])
def test_route_plan_bit_exact(oracle, R, E, tile_rows):
    rng = np.random.default_rng(R + E)
    ids = rng.integers(0, E, R).astype(np.uint32)
    if R > 10:
        ids[::37] = E + 5  # invalid ids, counted and placed last
    scores = rng.uniform(size=R).astype(np.float32)
    got = _plan_gpu(ids, E, tile_rows, scores)
    ref = oracle.route_plan(ids, E, scores)
    for k in ("order", "inverse", "sorted_experts", "sorted_scores"):
        assert np.array_equal(got[k].view(np.uint32), ref[k].view(np.uint32)), k
    assert np.array_equal(got["route_offsets"].view(np.uint32), ref["expert_offsets"])
    assert int(got["invalid_count"][0]) == ref["invalid"]
    te, ts, tl, ro, to = oracle.tile_plan(ref["sorted_experts"], E, tile_rows)
    assert np.array_equal(got["tile_experts"].view(np.uint32), te)
    assert np.array_equal(got["tile_starts"].view(np.uint32), ts)
    assert np.array_equal(got["tile_lengths"].view(np.uint32), tl)
    assert np.array_equal(got["tile_offsets"].view(np.uint32), to)
    assert int(got["descriptor_count"][0]) == int(to[-1])


def test_grouped_linear_and_pieces_match_oracle(G, S, oracle):
    E, H, I, T, k = 8, 256, 128, 32, 8
    bank = S.make_bank(E, H, I, seed=21, device="cuda")
    x = S.random_bf16((T, H), seed=22, device="cuda")
    gen = np.random.default_rng(3)
    idx = np.stack([gen.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    sc = gen.uniform(0.05, 0.3, (T, k)).astype(np.float32)
    it, st = torch.from_numpy(idx).cuda(), torch.from_numpy(sc).cuda()
    sorted_x, sorted_experts, sorted_scores, inverse = G.build_route_plan(x, it, st)
    plan = G.build_grouped_tile_plan(sorted_experts, E)
    gate_up = G.grouped_fp8_linear(sorted_x, plan, bank.gate_up_weight, bank.gate_up_scale_inv)
    hidden = G.activate_gate_up(gate_up, I, 3.0)
    down = G.grouped_fp8_linear(hidden, plan, bank.down_weight, bank.down_scale_inv)
    out = G.restore_and_reduce(down, sorted_scores, inverse, (T, H), k)
    torch.cuda.synchronize()
    rp = oracle.route_plan(idx.reshape(-1), E, sc.reshape(-1))
    assert np.array_equal(bits(sorted_x), bits(x)[rp["order"] // k])
    hb = bank_host(bank)
    r_gu = oracle.grouped_linear(bits(sorted_x), rp["sorted_experts"], hb[0], hb[1])
    assert_layer_close(bits(gate_up), r_gu, certificate=certify_grouped_linear(
        bits(sorted_x), rp["sorted_experts"], hb[0], hb[1], bits(gate_up)))
    r_hidden = oracle.activate_gate_up(bits(gate_up), I, 3.0)
    assert np.array_equal(bits(hidden), r_hidden)  # same inputs -> bit-exact elementwise
    r_down = oracle.grouped_linear(bits(hidden), rp["sorted_experts"], hb[2], hb[3])
    assert_layer_close(bits(down), r_down, certificate=certify_grouped_linear(
        bits(hidden), rp["sorted_experts"], hb[2], hb[3], bits(down)))
    r_out = oracle.restore_and_reduce(bits(down), rp["sorted_scores"], rp["inverse"], T, k)
    assert np.array_equal(bits(out), r_out)  # same inputs -> bit-exact combine


@pytest.mark.parametrize("T,E,H,I,Is", [(32, 8, 256, 128, 128), (200, 64, 1024, 384, 256)])
def test_grouped_moe_matches_oracle(G, S, oracle, T, E, H, I, Is):
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    bank = S.make_bank(E, H, I, seed=T, device="cuda")
    shared = shared_fp8_tensors(S.make_shared(H, Is, seed=T + 1, device="cuda"))
    w, b = S.make_router(E, H, seed=T + 2, device="cuda", zipf_alpha=0.5)
    x = S.random_bf16((T, H), seed=T + 3, device="cuda")
    idx, sc = G.router_topk(x, w, b, top_k=8)
    from glm53_flash_mlx_b200 import _native as N

    ws = N.Workspace()
    out = G.grouped_moe(x, idx, sc, bank, shared, limit=10.0, workspace=ws)
    torch.cuda.synchronize()
    hb, hs = bank_host(bank), shared_host(shared)
    ref = oracle.grouped_moe(bits(x), idx.cpu().numpy(), sc.cpu().numpy(), hb, hs, 10.0)
    cert = certify_grouped(bits(x), idx.cpu().numpy(), sc.cpu().numpy(), hb, hs, 10.0, bits(out),
                           ws._buffers[(x.device, "grouped")])
    assert_layer_close(bits(out), ref, certificate=cert)


def _spread_tokens(idx_np: np.ndarray, E: int, want: int) -> np.ndarray:
    """Tokens covering the most and the least loaded experts: experts are taken
    alternately from both ends of the load order, up to 8 of each expert's
    tokens, until `want` distinct tokens are chosen."""
    loads = np.bincount(idx_np.reshape(-1), minlength=E)
    order = np.argsort(-loads, kind="stable")
    order = order[loads[order] > 0]
    picks, seen = [], set()
    lo, hi = 0, len(order) - 1
    turn = 0
    while len(picks) < want and lo <= hi:
        e = order[lo] if turn == 0 else order[hi]
        if turn == 0:
            lo += 1
        else:
            hi -= 1
        turn ^= 1
        for t in np.nonzero((idx_np == e).any(axis=1))[0][:8]:
            if int(t) not in seen:
                seen.add(int(t))
                picks.append(int(t))
    return np.sort(np.array(picks[:want], dtype=np.int64))


def test_grouped_moe_config3_full_size_token_subset(G, S, oracle):
    """Config 3 at T=2048 (16,384 routes, Zipf-skewed bias): the whole layer
    on the GPU, checked against the oracle on 256 tokens that cover the most
    and the least loaded experts (a token's output depends only on its own
    routes), with the rounding certificate of every intermediate."""
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    E, H, I, T = 288, 4096, 1536, 2048
    bank = S.make_bank(E, H, I, seed=2, device="cuda")
    shared = shared_fp8_tensors(S.make_shared(H, I, seed=3, device="cuda"))
    w, b = S.make_router(E, H, seed=4, device="cuda", zipf_alpha=0.5)
    x = S.random_bf16((T, H), seed=5, device="cuda")
    idx, sc = G.router_topk(x, w, b, top_k=8)
    ws = N.Workspace()
    out = G.grouped_moe(x, idx, sc, bank, shared, limit=10.0, workspace=ws)
    torch.cuda.synchronize()
    idx_all = idx.cpu().numpy()
    sel = _spread_tokens(idx_all, E, 256)
    assert sel.size == 256
    idx_np = idx_all[sel]
    touched = np.unique(idx_np)
    remap = np.searchsorted(touched, idx_np).astype(np.uint32)
    hb, hs = bank_host(bank, touched), shared_host(shared)
    ref = oracle.grouped_moe(bits(x)[sel], remap, sc.cpu().numpy()[sel], hb, hs, 10.0)
    cert = certify_grouped(bits(x), idx_all, sc.cpu().numpy(), hb, hs, 10.0, bits(out),
                           ws._buffers[(x.device, "grouped")], tokens=sel, bank_experts=touched, expert_count=E)
    stats = assert_layer_close(bits(out)[sel], ref, certificate=cert)
    # 16,384 routes: the chunked (multi-block) route plan
    check_grouped_route_plan(ws._buffers[(x.device, "grouped")], idx_all, sc.cpu().numpy(), E, H, I, I)
    loads = np.bincount(idx_all.reshape(-1), minlength=E)
    print(f"[config3 T=2048, 256 tokens, {touched.size} experts, loads {loads[touched].min()}..{loads.max()}] "
          f"{stats} {cert}")


@pytest.mark.parametrize("T,E,H,I,Is", [(32, 8, 256, 128, 128), (200, 64, 1024, 384, 256)])
def test_grouped_moe_f8_matches_oracle(G, S, oracle, T, E, H, I, Is):
    """GLM53_FLAG_F8_MMA (tcgen05 kind::f8f6f4, hi + lo E4M3 activations):
    within the north-star bound of the oracle on the real BF16 input, with the
    F8 certificate (terms bit-exact against the oracle's split, every
    intermediate inside the rounding envelope of the represented problem, the
    combine bit for bit)."""
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    bank = S.make_bank(E, H, I, seed=T, device="cuda")
    shared = shared_fp8_tensors(S.make_shared(H, Is, seed=T + 1, device="cuda"))
    w, b = S.make_router(E, H, seed=T + 2, device="cuda", zipf_alpha=0.5)
    x = S.random_bf16((T, H), seed=T + 3, device="cuda")
    idx, sc = G.router_topk(x, w, b, top_k=8)
    ws = N.Workspace()
    out = G.grouped_moe(x, idx, sc, bank, shared, limit=10.0, workspace=ws, mma="f8")
    torch.cuda.synchronize()
    assert int(ws.get(x.device, "status", 4).view(torch.int32)[0].item()) == 0
    hb, hs = bank_host(bank), shared_host(shared)
    ref = oracle.grouped_moe(bits(x), idx.cpu().numpy(), sc.cpu().numpy(), hb, hs, 10.0)
    cert = certify_grouped_f8(bits(x), idx.cpu().numpy(), sc.cpu().numpy(), hb, hs, 10.0, bits(out),
                              ws._buffers[(x.device, "grouped")])
    stats = assert_layer_close(bits(out), ref, certificate=cert)
    print(f"[f8 T={T} H={H} I={I}] {stats} {cert}")


def test_grouped_moe_f8_config3_full_size_token_subset(G, S, oracle):
    """Config 3 at T=2048 on the FP8 tensor-core kernels, checked like the
    kind::f16 run: 256 tokens covering the most and the least loaded experts,
    the F8 certificate and the north-star bound against the oracle."""
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    E, H, I, T = 288, 4096, 1536, 2048
    bank = S.make_bank(E, H, I, seed=2, device="cuda")
    shared = shared_fp8_tensors(S.make_shared(H, I, seed=3, device="cuda"))
    w, b = S.make_router(E, H, seed=4, device="cuda", zipf_alpha=0.5)
    x = S.random_bf16((T, H), seed=5, device="cuda")
    idx, sc = G.router_topk(x, w, b, top_k=8)
    ws = N.Workspace()
    out = G.grouped_moe(x, idx, sc, bank, shared, limit=10.0, workspace=ws, mma="f8")
    torch.cuda.synchronize()
    assert int(ws.get(x.device, "status", 4).view(torch.int32)[0].item()) == 0
    idx_all = idx.cpu().numpy()
    sel = _spread_tokens(idx_all, E, 256)
    idx_np = idx_all[sel]
    touched = np.unique(idx_np)
    remap = np.searchsorted(touched, idx_np).astype(np.uint32)
    hb, hs = bank_host(bank, touched), shared_host(shared)
    ref = oracle.grouped_moe(bits(x)[sel], remap, sc.cpu().numpy()[sel], hb, hs, 10.0)
    cert = certify_grouped_f8(bits(x), idx_all, sc.cpu().numpy(), hb, hs, 10.0, bits(out),
                              ws._buffers[(x.device, "grouped")], tokens=sel, bank_experts=touched, expert_count=E)
    stats = assert_layer_close(bits(out)[sel], ref, certificate=cert)
    print(f"[f8 config3 T=2048, 256 tokens, {touched.size} experts] {stats} {cert}")


def test_e4m3_split_rows_matches_oracle(oracle):
    """glm53_e4m3_split_rows: terms and scales equal the oracle's split value
    for value (rows with tiny, zero, large and denormal-scale entries), and the
    in-place form writes the same bytes."""
    from glm53_flash_mlx_b200 import _native as N

    rng = np.random.default_rng(0)
    x = rng.standard_normal((64, 4096)).astype(np.float32)
    x[0, :100] *= 1e-5
    x[1] = 0
    x[2, 5] = 3e4
    x[3] *= 1e-30
    xb = oracle.bf16_from_f32(x)
    xt = from_bits(xb)
    terms = torch.empty((64, 2 * 4096), dtype=torch.uint8, device="cuda")
    scale = torch.empty(64, dtype=torch.float32, device="cuda")
    dev = xt.device
    N.check(N.lib().glm53_e4m3_split_rows(xt.data_ptr(), 64, 4096, terms.data_ptr(), scale.data_ptr(),
                                          N.stream(dev)), "glm53_e4m3_split_rows")
    torch.cuda.synchronize()
    tab = oracle.e4m3_table()
    t = terms.cpu().numpy()
    hi, lo, s = oracle.split_e4m3_rows(xb)
    assert np.array_equal(tab[t[:, :4096]], hi) and np.array_equal(tab[t[:, 4096:]], lo)
    assert np.array_equal(scale.cpu().numpy(), s)
    rep = (hi.astype(np.float64) + lo) * s[:, None]
    exact = np.abs(f32(xb)) >= np.abs(f32(xb)).max(axis=1, keepdims=True) * 2.0 ** -9
    assert np.array_equal(rep[exact], f32(xb)[exact])
    xt2 = xt.clone()
    N.check(N.lib().glm53_e4m3_split_rows(xt2.data_ptr(), 64, 4096, xt2.data_ptr(), scale.data_ptr(),
                                          N.stream(dev)), "glm53_e4m3_split_rows")
    torch.cuda.synchronize()
    assert torch.equal(xt2.view(torch.uint8).reshape(64, -1), terms)


def test_sorted_grouped_module_vs_direct_and_decode_fallback(G, S):
    """tests/test_fp8_metal.py:154-198: 32-token grouped prefill within
    0.02/0.02 of Direct; decode falls back and is bit-equal; min_routes 256."""
    from types import SimpleNamespace

    class DeterministicGate(torch.nn.Module):
        def forward(self, x):
            rows = x.reshape(-1, x.shape[-1]).shape[0]
            routes = torch.arange(rows * 8, dtype=torch.int32, device=x.device).reshape(rows, 8)
            indices = ((routes * 5 + 3) % 8).reshape(*x.shape[:-1], 8)
            return indices, torch.full(indices.shape, 0.125, dtype=torch.float32, device=x.device)

    config = SimpleNamespace(hidden_size=256, moe_intermediate_size=128, swiglu_limit=3.0, n_routed_experts=8,
                             num_experts_per_tok=8)
    direct = G.DirectFP8MoE(config, DeterministicGate(), None, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(9)
    for e in direct.experts:
        for p in (e.gate_proj, e.up_proj, e.down_proj):
            p.weight = torch.randint(0, 247, p.weight.shape, generator=g, device="cuda", dtype=torch.int32).to(
                torch.uint8)
            p.weight_scale_inv = torch.rand(p.weight_scale_inv.shape, generator=g, device="cuda") * 0.002
    bank = G.PackedFP8ExpertBank.pack(direct.experts)
    grouped = G.SortedGroupedFP8MoE(bank, config, direct.gate, None)
    assert grouped.min_routes == 256
    xp = torch.randn((1, 32, 256), generator=g, device="cuda").to(torch.bfloat16)
    assert torch.allclose(grouped(xp).float(), direct(xp).float(), rtol=0.02, atol=0.02)
    xd = torch.randn((1, 1, 256), generator=g, device="cuda").to(torch.bfloat16)
    assert torch.equal(grouped(xd), direct(xd))


# ---------------------------------------------------------------------------
# E4M3 decode modes
# ---------------------------------------------------------------------------


def test_e4m3_scan_detects_nan_codes(S):
    from glm53_flash_mlx_b200 import _native as N

    w, _ = S.random_block_fp8(256, 4096, seed=3, device="cuda")
    assert N.e4m3_finite(w)
    w2 = w.clone()
    w2[100, 1234] = 0x7F
    assert not N.e4m3_finite(w2)
    w3 = w.clone()
    w3[-1, -1] = 0xFF
    assert not N.e4m3_finite(w3)


@pytest.mark.parametrize("M,N_,K", [(1, 6144, 4096), (8, 512, 2048), (3, 384, 1536)])
def test_finite_decode_matches_exact_decode_bitwise(G, S, M, N_, K):
    """The hardware E4M3 decode (codes scaled by 1) and the exact bit decode
    (codes scaled by 1/256, scale x 256) give identical FP32 sums."""
    w, s = S.random_block_fp8(N_, K, seed=7, device="cuda")
    x = S.random_bf16((M, K), seed=8, device="cuda")
    a = G.block_fp8_linear(x, w, s, e4m3_finite=False)
    b = G.block_fp8_linear(x, w, s, e4m3_finite=True)
    assert torch.equal(a, b)


def test_exact_decode_handles_0x7f_as_480(G, oracle):
    """Codes 0x7F/0xFF decode to +-480 (the reference table) on the exact path."""
    codes = torch.full((16, 256), 0x38, dtype=torch.uint8, device="cuda")  # 1.0
    codes[:, 0] = 0x7F
    codes[:, 1] = 0xFF
    s = torch.ones((1, 2), dtype=torch.float32, device="cuda")
    x = torch.zeros((1, 256), dtype=torch.bfloat16, device="cuda")
    x[0, 0] = 1.0
    x[0, 1] = 0.5
    y = G.block_fp8_linear(x, codes, s)
    assert torch.all(y.float() == 480.0 - 240.0)


@pytest.mark.parametrize("E,H,I,with_shared", [(16, 1024, 256, True), (64, 4096, 1536, True),
                                                (16, 1024, 384, False)])
def test_captured_decode_matches_module_call(G, S, E, H, I, with_shared):
    """PackedFP8MoE.capture_decode() (one glm53_decode_step_host call per
    token: input copy kernel, router, packed decode writing a pinned output
    directly) gives the module's own bits for host and device rows."""
    from glm53_flash_mlx_b200.packed import PackedDecodeStep
    from glm53_flash_mlx_b200.router import Float32Gate

    cfg = S.moe_config(H, I, E, 8, 10.0)
    bank = S.make_bank(E, H, I, seed=81, device="cuda")
    shared = S.make_shared(H, I, seed=82, device="cuda") if with_shared else None
    gate = Float32Gate(cfg, device="cuda")
    w, b = S.make_router(E, H, seed=83, device="cuda")
    gate.weight.copy_(w)
    gate.e_score_correction_bias.copy_(b)
    mod = G.PackedFP8MoE(bank, cfg, gate, shared)
    cap = mod.capture_decode()
    assert isinstance(cap, PackedDecodeStep)
    y_pinned = torch.empty((1, 1, H), dtype=torch.bfloat16).pin_memory()
    for t in range(4):
        x = S.random_bf16((1, 1, H), seed=84 + t, device="cuda")
        want = mod(x).clone()
        got = cap(x.cpu().pin_memory()).clone()  # host in, device out
        torch.cuda.synchronize()
        assert torch.equal(got, want), t
        cap(x.cpu().pin_memory(), out=y_pinned)  # host in and out, output written by the decode kernel
        torch.cuda.synchronize()
        assert torch.equal(y_pinned, want.cpu()), t
        y_page = torch.empty((1, 1, H), dtype=torch.bfloat16)
        cap(x.cpu(), out=y_page)  # pageable host buffers
        torch.cuda.synchronize()
        assert torch.equal(y_page, want.cpu()), t
        assert torch.equal(cap(x).clone(), want), t  # device in
        y_dev = torch.empty((1, 1, H), dtype=torch.bfloat16, device="cuda")
        cap(x.cpu().pin_memory(), out=y_dev)  # host in, device out
        assert torch.equal(y_dev, want), t
    assert int(mod.status.view(torch.int32)[0].item()) == 0


def test_captured_graph_decode_host_buffers(G, S):
    """A layer whose gate is not the Float32Gate gets the CUDA-graph form of
    capture_decode (glm53_graph_step: copy kernels over pinned buffers around
    the replay, cudaMemcpyAsync for pageable ones); same bits as the module."""
    from glm53_flash_mlx_b200.packed import CapturedDecode

    E, H, I = 16, 1024, 256
    cfg = S.moe_config(H, I, E, 8, 10.0)
    bank = S.make_bank(E, H, I, seed=85, device="cuda")
    shared = S.make_shared(H, I, seed=86, device="cuda")
    routes = torch.tensor([[3, 9, 1, 14, 0, 7, 11, 5]], dtype=torch.int32, device="cuda")
    scores = torch.tensor([[0.2, 0.17, 0.15, 0.13, 0.11, 0.1, 0.08, 0.06]], device="cuda")

    class FixedGate(torch.nn.Module):
        def forward(self, x):
            shape = (*x.shape[:-1], 8)
            return routes.expand(shape), scores.expand(shape)

    mod = G.PackedFP8MoE(bank, cfg, FixedGate(), shared)
    cap = mod.capture_decode()
    assert isinstance(cap, CapturedDecode)
    y_pinned = torch.empty((1, 1, H), dtype=torch.bfloat16).pin_memory()
    for t in range(3):
        x = S.random_bf16((1, 1, H), seed=87 + t, device="cuda")
        want = mod(x).clone()
        cap(x.cpu().pin_memory(), out=y_pinned)
        torch.cuda.synchronize()
        assert torch.equal(y_pinned, want.cpu()), t
        y_page = torch.empty((1, 1, H), dtype=torch.bfloat16)
        cap(x.cpu(), out=y_page)
        torch.cuda.synchronize()
        assert torch.equal(y_page, want.cpu()), t


@pytest.mark.parametrize("M,N_,K", [(64, 576, 4096), (300, 1024, 1536), (2048, 4096, 4096)])
def test_block_linear_tensor_core_path_matches_oracle(G, S, oracle, M, N_, K):
    """M > 16 runs the tcgen05 GEMM through glm53_fp8_linear_ws (N = 576 cuts the
    last 128-row weight tile); the oracle checks a row subset at the largest M."""
    w, s = S.random_block_fp8(N_, K, seed=M, tensor=3, std=0.02, device="cuda")
    x = S.random_bf16((M, K), seed=M + 1, device="cuda", std=1.5)
    y = G.block_fp8_linear(x, w, s)
    torch.cuda.synchronize()
    rows = np.arange(M) if M <= 300 else np.random.default_rng(M).choice(M, 48, replace=False)
    ref = oracle.block_fp8_linear(bits(x)[rows], w.cpu().numpy(), s.cpu().numpy())
    cert = certify_linear(bits(x)[rows], w.cpu().numpy(), s.cpu().numpy(), bits(y)[rows])
    assert_layer_close(bits(y)[rows], ref, certificate=cert)


@pytest.mark.parametrize("T,E,H,I", [(2, 16, 1024, 256), (9, 32, 2048, 512), (16, 288, 4096, 1536),
                                     (24, 288, 4096, 1536), (64, 288, 4096, 1536)])
def test_batched_decode_matches_oracle_and_direct_loop(G, S, oracle, T, E, H, I):
    """Decode batches of 2..64 rows (below min_routes the reference runs
    Direct semantics, grouped_fp8.py:323-326): PackedFP8MoE's batched path
    (per-route decode + BF16 scatter-add in ascending expert id,
    glm53_flash_mlx/fp8.py:384-399) against the oracle of that order, with
    max-abs 2e-2 and cosine 0.9999.  An element beyond 2e-2 needs the staged
    certificate: the per-route rows (glm53_routes_decode, which the batched
    kernels reproduce bit for bit) have every hidden and down value inside the
    oracle's rounding envelope, and the batched output is the ascending-id BF16
    combine of those rows, bit for bit.  The Direct module's per-expert loop
    over the same bank is held to the same bar with the layer envelope."""
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200.ep import pack_shared_bank, routes_decode
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors
    from glm53_flash_mlx_b200.router import Float32Gate

    cfg = S.moe_config(H, I, E, 8, 10.0)
    bank = S.make_bank(E, H, I, seed=T + 7, device="cuda")
    shared = S.make_shared(H, I, seed=T + 8, device="cuda")
    gate = Float32Gate(cfg, device="cuda")
    w, b = S.make_router(E, H, seed=T + 9, device="cuda")
    gate.weight.copy_(w)
    gate.e_score_correction_bias.copy_(b)
    mod = G.PackedFP8MoE(bank, cfg, gate, shared)
    sh = shared_host(shared_fp8_tensors(shared))
    for trial in range(2):
        x = S.random_bf16((1, T, H), seed=100 * T + trial, device="cuda", std=1.5)
        got = mod(x)
        idx, sc = mod.gate(x)
        loop = mod._forward_routes(x, idx, sc)
        torch.cuda.synchronize()
        ids = idx.reshape(T, 8).cpu().numpy().astype(np.int64)
        scs = sc.reshape(T, 8).cpu().numpy()
        touched, local = np.unique(ids, return_inverse=True)  # ascending ids keep the loop order
        hb = bank_host(bank, touched)
        xb = bits(x.reshape(T, H))
        ref = oracle.direct_moe(xb, local.reshape(T, 8), scs, hb, sh, 10.0)
        # staged certificate of the batched output
        tensors = (bank.gate_up_weight, bank.gate_up_scale_inv, bank.down_weight, bank.down_scale_inv)
        wsr = N.Workspace()
        xr = x.reshape(T, H)
        rows = routes_decode(xr.repeat_interleave(8, dim=0), idx.reshape(-1), tensors, limit=10.0, workspace=wsr)
        hid = wsr._buffers[(xr.device, "routes")][:T * 8 * I * 2].view(torch.int16).reshape(T * 8, I)
        sh_tensors = pack_shared_bank(shared_fp8_tensors(shared))
        wss = N.Workspace()
        sh_rows = routes_decode(xr, torch.zeros(T, dtype=torch.int32, device="cuda"), sh_tensors, limit=10.0,
                                workspace=wss)
        sh_hid = wss._buffers[(xr.device, "routes")][:T * I * 2].view(torch.int16).reshape(T, I)
        torch.cuda.synchronize()
        rows_b, sh_b = bits(rows), bits(sh_rows)
        cert = certify_expert_rows(np.repeat(xb, 8, 0), local.reshape(-1).astype(np.uint32), hb, 10.0,
                                   f32(bits(hid)), rows_b, down_kind="bf16")
        cs = certify_expert_rows(xb, np.zeros(T, np.uint32), tuple(t.cpu().numpy() for t in sh_tensors), 10.0,
                                 f32(bits(sh_hid)), sh_b, down_kind="bf16")
        expect = direct_combine(f32(rows_b).reshape(T, 8, H), ids, scs, shared=f32(sh_b))
        assert np.array_equal(bits(got.reshape(T, H)), expect), "batched output != combine of certified rows"
        cert = {k: cert[k] + cs[k] for k in cert}
        cert["certified"] = True
        stats = assert_layer_close(bits(got.reshape(T, H)), ref, certificate=cert)
        print(f"[batched T={T}] {stats} {cert}")
        lo, hi = oracle.direct_envelope(xb, local.reshape(T, 8), scs, hb, sh, 10.0)
        loop_stats = assert_layer_close(bits(loop.reshape(T, H)), ref,
                                        certificate=certify_by_envelope(bits(loop.reshape(T, H)), lo, hi))
        assert stats["bit_identical"] >= 0.99, stats
        same = float((bits(got) == bits(loop)).mean())
        assert same >= 0.99, (same, loop_stats)


@pytest.mark.parametrize("T", [24, 31])
def test_short_prefill_rows_stay_on_the_device(G, S, T):
    """A batch below min_routes (T * 8 < 256: 17..31 rows) runs the batched
    device path with no host synchronisation at all: torch's sync debug mode
    turns any device->host read (a routing readback, .cpu(), .item()) into an
    error.  The result equals a plain call's."""
    from glm53_flash_mlx_b200.grouped_fp8 import SortedGroupedFP8MoE
    from glm53_flash_mlx_b200.router import Float32Gate

    E, H, I = 288, 4096, 1536
    cfg = S.moe_config(H, I, E, 8, 10.0)
    gate = Float32Gate(cfg, device="cuda")
    w, b = S.make_router(E, H, seed=T, device="cuda")
    gate.weight.copy_(w)
    gate.e_score_correction_bias.copy_(b)
    mod = SortedGroupedFP8MoE(S.make_bank(E, H, I, seed=T + 1, device="cuda"), cfg, gate,
                              S.make_shared(H, I, seed=T + 2, device="cuda"))
    x = S.random_bf16((1, T, H), seed=T + 3, device="cuda")
    want = mod(x).clone()  # first call: weight scans and workspaces
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        got = mod(x)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()
    mod.check_status()
    assert torch.equal(got, want)


@pytest.mark.parametrize("T,E,H,I", [(3, 8, 1024, 256), (16, 64, 2048, 768)])
def test_coalesced_batched_decode_equals_per_route_decode_bitwise(G, S, T, E, H, I):
    """glm53_batched_decode_moe (each expert's weights streamed once for all of
    its routes, the routes in the MMA's N columns) gives the bits of the
    per-route decode (glm53_routes_decode) followed by glm53_direct_combine."""
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200.ep import routes_decode
    from glm53_flash_mlx_b200.packed import batched_decode_moe

    bank = S.make_bank(E, H, I, seed=T + 21, device="cuda")
    gen = torch.Generator().manual_seed(T)
    # few experts, so several routes share one (and descriptors hold 1..4 routes)
    ids = torch.stack([torch.randperm(E, generator=gen)[:8] for _ in range(T)]).to(torch.int32).cuda()
    sc = (torch.rand((T, 8), generator=gen) * 0.25 + 0.05).cuda()
    x = S.random_bf16((T, H), seed=T + 22, device="cuda", std=1.5)
    got = batched_decode_moe(x, ids, sc, bank, None, limit=10.0)
    tensors = (bank.gate_up_weight, bank.gate_up_scale_inv, bank.down_weight, bank.down_scale_inv)
    rows = routes_decode(x.repeat_interleave(8, dim=0), ids.reshape(-1), tensors, limit=10.0)
    want = torch.empty_like(x)
    N.check(N.lib().glm53_direct_combine(rows.data_ptr(), ids.data_ptr(), sc.data_ptr(), T, 8, H, None,
                                         want.data_ptr(), N.stream()), "combine")
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("top_k,H", [(8, 4096), (9, 520), (32, 1024)])
def test_direct_combine_orders_slots_by_expert_then_slot(top_k, H):
    """glm53_direct_combine: per token, BF16(row * score) added in BF16 in
    ascending expert id -- repeated ids in slot order (a stable sort, as
    np.argsort(kind="stable") and the module's index_add order) -- then the
    shared row; widths that are not multiples of the CTA's 512 columns."""
    from glm53_flash_mlx_b200 import _native as N

    T = 5
    gen = torch.Generator().manual_seed(top_k * 7 + H)
    ids = torch.randint(0, 6, (T, top_k), generator=gen, dtype=torch.int32)  # repeats within a token
    sc = torch.rand((T, top_k), generator=gen) * 0.5 + 0.05
    rows = (torch.randn((T * top_k, H), generator=gen) * 3).to(torch.bfloat16)
    shared = (torch.randn((T, H), generator=gen)).to(torch.bfloat16)
    out = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    rd, idd, sd, shd = rows.cuda(), ids.cuda(), sc.cuda(), shared.cuda()
    N.check(N.lib().glm53_direct_combine(rd.data_ptr(), idd.data_ptr(), sd.data_ptr(), T, top_k, H, shd.data_ptr(),
                                         out.data_ptr(), N.stream()), "combine")
    torch.cuda.synchronize()
    expect = direct_combine(f32(bits(rows)).reshape(T, top_k, H), ids.numpy(), sc.numpy(), shared=f32(bits(shared)))
    assert np.array_equal(bits(out), expect)


def test_batched_decode_flags_bad_expert_without_trapping(G, S):
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200.packed import batched_decode_moe

    E, H, I = 8, 256, 128
    bank = S.make_bank(E, H, I, seed=5, device="cuda")
    ids = torch.tensor([[0, 1, 2, 3, 4, 5, 6, 7], [7, 6, 5, 4, 3, 2, 1, 99]], dtype=torch.int32, device="cuda")
    sc = torch.full((2, 8), 0.1, device="cuda")
    x = S.random_bf16((2, H), seed=6, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = batched_decode_moe(x, ids, sc, bank, None, limit=10.0, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & N.STATUS_BAD_EXPERT
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("T,E,H,I", [(3, 8, 1024, 256), (16, 288, 4096, 1536)])
def test_batched_shared_expert_route_equals_shared_rows_added_last(G, S, T, E, H, I):
    """glm53_batched_decode_moe_shared (the shared expert as one more route per
    token, weight 1.0) gives the bits of glm53_batched_decode_moe given the
    shared expert's per-route decode rows as `shared` (added after the routed
    experts); a bad routed id is flagged and skipped in both."""
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200.ep import routes_decode
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    bank = S.make_bank(E, H, I, seed=T + 31, device="cuda")
    sh = shared_fp8_tensors(S.make_shared(H, I, seed=T + 32, device="cuda"))
    gen = torch.Generator().manual_seed(T + 33)
    ids = torch.stack([torch.randperm(E, generator=gen)[:8] for _ in range(T)]).to(torch.int32)
    ids[T - 1, 7] = E + 5  # out of range: skipped and flagged
    ids = ids.cuda()
    sc = (torch.rand((T, 8), generator=gen) * 0.25 + 0.05).cuda()
    x = S.random_bf16((T, H), seed=T + 34, device="cuda", std=1.5)
    lib = N.lib()
    flags = N.decode_flags(bank.gate_up_weight, bank.down_weight, sh[0], sh[2], sh[4])
    # the shared expert as a one-expert bank: its per-route decode rows
    one = (torch.cat([sh[0], sh[2]]).unsqueeze(0).contiguous(), torch.cat([sh[1], sh[3]]).unsqueeze(0).contiguous(),
           sh[4].unsqueeze(0).contiguous(), sh[5].unsqueeze(0).contiguous())
    rows = routes_decode(x, torch.zeros(T, dtype=torch.int32, device="cuda"), one, limit=10.0, flags=flags)
    st_a = torch.zeros(1, dtype=torch.int32, device="cuda")
    st_b = torch.zeros(1, dtype=torch.int32, device="cuda")
    want = torch.empty_like(x)
    ws = torch.zeros(lib.glm53_batched_decode_workspace_bytes(T, 8, E, H, I), dtype=torch.uint8, device="cuda")
    N.check(lib.glm53_batched_decode_moe(
        x.data_ptr(), T, H, ids.data_ptr(), sc.data_ptr(), 8, bank.gate_up_weight.data_ptr(),
        bank.gate_up_scale_inv.data_ptr(), bank.down_weight.data_ptr(), bank.down_scale_inv.data_ptr(), E, I, 10.0,
        rows.data_ptr(), want.data_ptr(), ws.data_ptr(), ws.numel(), st_a.data_ptr(), flags, N.stream()), "old")
    got = torch.empty_like(x)
    ws2 = torch.zeros(lib.glm53_batched_decode_shared_workspace_bytes(T, 8, E, H, I), dtype=torch.uint8,
                      device="cuda")
    N.check(lib.glm53_batched_decode_moe_shared(
        x.data_ptr(), T, H, ids.data_ptr(), sc.data_ptr(), 8, bank.gate_up_weight.data_ptr(),
        bank.gate_up_scale_inv.data_ptr(), bank.down_weight.data_ptr(), bank.down_scale_inv.data_ptr(), E, I,
        *(t.data_ptr() for t in sh), 10.0, got.data_ptr(), ws2.data_ptr(), ws2.numel(), st_b.data_ptr(), flags,
        N.stream()), "shared")
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert int(st_a.item()) & N.STATUS_BAD_EXPERT and int(st_b.item()) & N.STATUS_BAD_EXPERT
