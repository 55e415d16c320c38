"""FFN boundary around the MoE: mHC collapse + post-attention RMSNorm before
the router, hc expand after the MoE.

CPU tests pin the oracle against an independent float64 numpy restatement and
known answers; GPU tests (-m gpu) compare the sm_100a kernels with the oracle.
Tolerances: the hc expand is bit-exact (same FMA chain, same inputs);
``post``/``comb`` within atol 1e-5 + rtol 1e-5 (FP32 mixing sums over 4H
terms in another order).  ``collapsed`` = BF16(sum_b pre[b] x[b]) within one
BF16 ulp plus 1e-5 * sum_b |x[b]| (a 1e-5 change of ``pre`` moves a sum that
cancels by that much, i.e. by several ulps of a small result); collapsed and
normalized also meet the layer bar (max(2e-2, 1 ulp), cosine >= 0.9999) with
at least 99% of elements bit-identical.
"""

import numpy as np
import pytest
import torch

from gpu_util import assert_layer_close, bf16_ulp, bits, f32, from_bits

H_CFG = 4096
N_BR = 4


def _inputs(T, H, seed):
    import oracle as O

    rng = np.random.default_rng(seed)
    K = N_BR * H
    state = O.bf16_from_f32(rng.standard_normal((T, N_BR, H)).astype(np.float32))
    fn = O.bf16_from_f32((rng.standard_normal((24, K)) / np.sqrt(K)).astype(np.float32))
    scale = np.array([1.0, 0.8, 1.5], np.float32)
    base = (rng.standard_normal(24) * 0.5).astype(np.float32)
    norm_w = O.bf16_from_f32((1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    return state, fn, scale, base, norm_w


def _f64_collapse(state_bits, fn_bits, scale, base, iters=20, eps=1e-6, norm_eps=1e-6):
    """Independent float64 restatement of the mHC collapse (no BF16 rounding)."""
    import oracle as O

    x = O.f32_from_bf16(state_bits).astype(np.float64)
    T, n, H = x.shape
    flat = x.reshape(T, n * H)
    r = 1.0 / np.sqrt((flat**2).mean(-1, keepdims=True) + norm_eps)
    m = flat @ O.f32_from_bf16(fn_bits).astype(np.float64).T * r
    sig = lambda z: 1.0 / (1.0 + np.exp(-z))  # noqa: E731
    pre = sig(m[:, :n] * scale[0] + base[:n]) + eps
    post = 2.0 * sig(m[:, n:2 * n] * scale[1] + base[n:2 * n])
    z = (m[:, 2 * n:] * scale[2] + base[2 * n:]).reshape(T, n, n)
    e = np.exp(z - z.max(-1, keepdims=True))
    c = e / e.sum(-1, keepdims=True) + eps
    c = c / (c.sum(-2, keepdims=True) + eps)
    for _ in range(iters - 1):
        c = c / (c.sum(-1, keepdims=True) + eps)
        c = c / (c.sum(-2, keepdims=True) + eps)
    y = (pre[:, :, None] * x).sum(1)
    return y, post, c


def _ulps(a_bits, b_bits):
    a = a_bits.astype(np.int32)
    b = b_bits.astype(np.int32)
    # BF16 bit patterns to a monotonic integer line
    a = np.where(a & 0x8000, 0x8000 - a, a)
    b = np.where(b & 0x8000, 0x8000 - b, b)
    return np.abs(a - b)


# ---------------------------------------------------------------------------
# CPU: the oracle
# ---------------------------------------------------------------------------


def test_oracle_collapse_matches_float64_restatement(oracle):
    state, fn, scale, base, norm_w = _inputs(6, 256, 11)
    col, nor, post, comb, _ = oracle.hc_collapse_norm(state, fn, scale, base, norm_w)
    y64, post64, comb64 = _f64_collapse(state, fn, scale, base)
    np.testing.assert_allclose(post, post64, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(comb, comb64, rtol=1e-5, atol=1e-6)
    assert _ulps(col, oracle.bf16_from_f32(y64.astype(np.float32))).max() <= 1
    # comb is (nearly) doubly stochastic: columns sum to 1 after the last step
    np.testing.assert_allclose(comb.sum(-2), 1.0, atol=1e-5)
    np.testing.assert_allclose(comb.sum(-1), 1.0, atol=1e-3)
    assert ((post > 0) & (post < 2)).all()


def test_oracle_rms_norm_matches_numpy(oracle):
    rng = np.random.default_rng(3)
    x = oracle.bf16_from_f32(rng.standard_normal((5, 512)).astype(np.float32) * 3)
    w = oracle.bf16_from_f32((1 + 0.2 * rng.standard_normal(512)).astype(np.float32))
    out = oracle.rms_norm(x, w, 1e-6)
    xf = oracle.f32_from_bf16(x).astype(np.float64)
    inv = 1.0 / np.sqrt((xf**2).mean(-1, keepdims=True) + 1e-6)
    ref = oracle.f32_from_bf16(w).astype(np.float64) * oracle.f32_from_bf16(
        oracle.bf16_from_f32((xf * inv).astype(np.float32))).astype(np.float64)
    assert _ulps(out, oracle.bf16_from_f32(ref.astype(np.float32))).max() <= 1
    # the fused collapse applies the same norm to its own collapsed rows
    state, fn, scale, base, norm_w = _inputs(4, 256, 5)
    col, nor, *_ = oracle.hc_collapse_norm(state, fn, scale, base, norm_w)
    np.testing.assert_array_equal(nor, oracle.rms_norm(col, norm_w, 1e-6))


def test_oracle_hc_expand_known_answers_and_float64(oracle):
    rng = np.random.default_rng(4)
    T, H = 3, 64
    moe = oracle.bf16_from_f32(rng.standard_normal((T, H)).astype(np.float32))
    res = oracle.bf16_from_f32(rng.standard_normal((T, N_BR, H)).astype(np.float32))
    eye = np.broadcast_to(np.eye(N_BR, dtype=np.float32), (T, N_BR, N_BR)).copy()
    zero_post = np.zeros((T, N_BR), np.float32)
    np.testing.assert_array_equal(oracle.hc_expand(moe, res, zero_post, eye), res)
    ones = np.ones((T, N_BR), np.float32)
    out = oracle.hc_expand(moe, res, ones, np.zeros_like(eye))
    np.testing.assert_array_equal(out, np.repeat(moe[:, None, :], N_BR, axis=1))
    post = rng.random((T, N_BR)).astype(np.float32) * 2
    comb = rng.random((T, N_BR, N_BR)).astype(np.float32)
    out = oracle.hc_expand(moe, res, post, comb)
    ref = post[:, :, None].astype(np.float64) * oracle.f32_from_bf16(moe)[:, None, :] + np.einsum(
        "tsb,tsd->tbd", comb.astype(np.float64), oracle.f32_from_bf16(res).astype(np.float64))
    assert _ulps(out, oracle.bf16_from_f32(ref.astype(np.float32))).max() <= 1


def test_hc_operators_fail_closed_without_cuda():
    import glm53_flash_mlx_b200 as G

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    hc = G.HyperConnection(64)
    with pytest.raises(RuntimeError, match="CUDA"):
        hc(torch.zeros((1, 4, 64), dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="CUDA"):
        G.hc_expand(torch.zeros((1, 64), dtype=torch.bfloat16), torch.zeros((1, 4, 64), dtype=torch.bfloat16),
                    torch.zeros((1, 4)), torch.zeros((1, 4, 4)))
    with pytest.raises(ValueError, match="branches"):
        G.HyperConnection(64, hc_mult=2)


def test_hc_workspace_query_is_host_only():
    from glm53_flash_mlx_b200 import _native as N

    lib = N.load_library()
    assert lib.glm53_hc_collapse_workspace_bytes(1, 4096) == 64 * 25 * 4
    assert lib.glm53_hc_collapse_workspace_bytes(2048, 4096) == 2048 * 8 * 25 * 4
    assert lib.glm53_hc_collapse_workspace_bytes(4, 4100) == 0  # H % 8 != 0
    assert lib.glm53_hc_collapse_workspace_bytes(4, 16384) == 0  # H > 8192


# ---------------------------------------------------------------------------
# GPU: kernels vs the oracle
# ---------------------------------------------------------------------------


def _module(G, fn, scale, base, H, dev):
    hc = G.HyperConnection(H, device=dev)
    hc.fn.copy_(from_bits(fn, dev))
    hc.scale.copy_(torch.from_numpy(scale))
    hc.base.copy_(torch.from_numpy(base))
    return hc


@pytest.mark.gpu
@pytest.mark.parametrize("T,H", [(1, H_CFG), (3, H_CFG), (16, H_CFG), (37, H_CFG), (256, H_CFG),
                                 (2048, H_CFG), (5, 256), (2, 8192)])
def test_hc_collapse_norm_matches_oracle(oracle, T, H):
    import glm53_flash_mlx_b200 as G

    dev = torch.device("cuda:0")
    state, fn, scale, base, norm_w = _inputs(T, H, 100 + T + H)
    col_o, nor_o, post_o, comb_o, _ = oracle.hc_collapse_norm(state, fn, scale, base, norm_w)
    hc = _module(G, fn, scale, base, H, dev)
    norm = G.RMSNorm(H, device=dev)
    norm.weight.copy_(from_bits(norm_w, dev))
    col, nor, post, comb = hc.collapse_norm(from_bits(state, dev), norm)
    torch.cuda.synchronize()
    np.testing.assert_allclose(post.cpu().numpy(), post_o, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(comb.cpu().numpy(), comb_o, rtol=1e-5, atol=1e-5)
    g, r = f32(bits(col)), f32(col_o)
    scale_x = np.abs(f32(state)).sum(1)
    # the collapse is one FP32 weighted sum over the 4 branches rounded to BF16:
    # with pre within 1e-5 of the oracle's (checked above), the GPU value is
    # within one BF16 ulp plus 1e-5 * sum |state| of the oracle's
    col_ok = bool((np.abs(g - r) <= bf16_ulp(r) + 1e-5 * scale_x).all())
    assert col_ok
    # the RMSNorm rounds twice after it (x * rsqrt, then * weight): an element
    # beyond max-abs 2e-2 is accepted when it is at most two BF16 ulps off (a
    # collapse flip carried through those two roundings)
    gn, rn = f32(bits(nor)), f32(nor_o)
    dn = np.abs(gn - rn)
    nor_ok = bool(((dn <= 2e-2) | (dn <= 2 * bf16_ulp(rn))).all())
    assert nor_ok
    for gpu_bits, ref_bits, ok, basis in ((bits(col), col_o, col_ok, "collapse: one BF16 rounding"),
                                          (bits(nor), nor_o, nor_ok, "norm: two BF16 roundings after it")):
        stats = assert_layer_close(gpu_bits, ref_bits, certificate={"certified": ok, "basis": basis})
        assert stats["bit_identical"] >= 0.99, stats
    # the module call without the norm returns the same collapse
    col2, post2, comb2 = hc(from_bits(state, dev))
    assert torch.equal(col2, col) and torch.equal(post2, post) and torch.equal(comb2, comb)


@pytest.mark.gpu
@pytest.mark.parametrize("T,H", [(1, H_CFG), (9, 1024), (300, H_CFG)])
def test_rms_norm_matches_oracle(oracle, T, H):
    import glm53_flash_mlx_b200 as G

    rng = np.random.default_rng(T + H)
    x = oracle.bf16_from_f32((rng.standard_normal((T, H)) * 2).astype(np.float32))
    w = oracle.bf16_from_f32((1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    dev = torch.device("cuda:0")
    out = G.rms_norm(from_bits(x, dev), from_bits(w, dev), 1e-6)
    assert _ulps(bits(out), oracle.rms_norm(x, w, 1e-6)).max() <= 1


@pytest.mark.gpu
@pytest.mark.parametrize("T,H", [(1, H_CFG), (7, H_CFG), (256, H_CFG), (2048, H_CFG), (3, 264)])
def test_hc_expand_bit_exact(oracle, T, H):
    import glm53_flash_mlx_b200 as G

    rng = np.random.default_rng(7 * T + H)
    moe = oracle.bf16_from_f32(rng.standard_normal((T, H)).astype(np.float32))
    res = oracle.bf16_from_f32(rng.standard_normal((T, N_BR, H)).astype(np.float32))
    post = (rng.random((T, N_BR)) * 2).astype(np.float32)
    comb = rng.random((T, N_BR, N_BR)).astype(np.float32)
    dev = torch.device("cuda:0")
    out = G.hc_expand(from_bits(moe, dev), from_bits(res, dev), torch.from_numpy(post).to(dev),
                      torch.from_numpy(comb).to(dev))
    np.testing.assert_array_equal(bits(out), oracle.hc_expand(moe, res, post, comb))


@pytest.mark.gpu
@pytest.mark.parametrize("T,E,H,I", [(1, 16, 256, 128), (1, 32, 4096, 1536), (3, 16, 256, 128)])
def test_ffn_boundary_composes_the_three_calls_bitwise(oracle, T, E, H, I):
    """FFNBoundary(state) == hc_expand(mlp(norm(collapse(state)))) through a
    PackedFP8MoE layer (one token: the expand runs inside the decode's final
    reduce, glm53_packed_decode_moe_hc; more tokens: the separate calls), and
    its collapse and expand agree with the oracle."""
    import glm53_flash_mlx_b200 as G
    from glm53_flash_mlx_b200 import synthetic as S

    dev = torch.device("cuda:0")
    config = S.moe_config(H=H, I=I, E=E)
    gate = G.Float32Gate(config, device=dev)
    w, b = S.make_router(E, H, seed=21, device=dev)
    gate.weight.copy_(w)
    gate.e_score_correction_bias.copy_(b)
    bank = S.make_bank(E, H, I, seed=21, device=dev)
    mlp = G.PackedFP8MoE(bank, config, gate, S.make_shared(H, I, seed=21, device=dev))
    state, fn, scale, base, norm_w = _inputs(T, H, 22)
    hc = _module(G, fn, scale, base, H, dev)
    norm = G.RMSNorm(H, device=dev)
    norm.weight.copy_(from_bits(norm_w, dev))
    block = G.FFNBoundary(hc, norm, mlp)
    st = from_bits(state, dev)
    out = block(st)
    _, nor, post, comb = hc.collapse_norm(st, norm)
    moe = mlp(nor)
    ref = G.hc_expand(moe, st, post, comb)
    assert torch.equal(out, ref)
    np.testing.assert_array_equal(bits(ref), oracle.hc_expand(bits(moe), state, post.cpu().numpy(),
                                                              comb.cpu().numpy()))


@pytest.mark.gpu
def test_hc_rejects_bad_geometry():
    import glm53_flash_mlx_b200 as G

    dev = torch.device("cuda:0")
    hc = G.HyperConnection(256, device=dev)
    with pytest.raises(ValueError, match="must end in"):
        hc(torch.zeros((2, 3, 256), dtype=torch.bfloat16, device=dev))
    with pytest.raises(ValueError, match="BF16"):
        hc(torch.zeros((2, 4, 256), dtype=torch.float32, device=dev))
    with pytest.raises(ValueError, match="residual shape"):
        G.hc_expand(torch.zeros((2, 256), dtype=torch.bfloat16, device=dev),
                    torch.zeros((2, 4, 128), dtype=torch.bfloat16, device=dev),
                    torch.zeros((2, 4), device=dev), torch.zeros((2, 4, 4), device=dev))
    big = G.HyperConnection(16384, device=dev)
    with pytest.raises(ValueError, match="not supported"):
        big(torch.zeros((1, 4, 16384), dtype=torch.bfloat16, device=dev))


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 2048])
def test_hc_calls_replay_bitwise_in_a_cuda_graph(T):
    """The collapse (mix kernel + its programmatic-dependent finish kernel) and
    the expand captured in one CUDA graph give the eager results bit for bit,
    on fresh inputs copied into the captured buffers."""
    import glm53_flash_mlx_b200 as G

    dev = torch.device("cuda:0")
    state, fn, scale, base, norm_w = _inputs(T, H_CFG, 300 + T)
    hc = _module(G, fn, scale, base, H_CFG, dev)
    norm = G.RMSNorm(H_CFG, device=dev)
    norm.weight.copy_(from_bits(norm_w, dev))
    st = from_bits(state, dev)
    moe = torch.randn((T, H_CFG), device=dev).to(torch.bfloat16)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        hc.collapse_norm(st, norm)  # eager call first: workspace allocation
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        _, g_nor, g_post, g_comb = hc.collapse_norm(st, norm)
        g_out = G.hc_expand(moe, st, g_post, g_comb)
    st2, _, _, _, _ = _inputs(T, H_CFG, 400 + T)
    st.copy_(from_bits(st2, dev))
    graph.replay()
    torch.cuda.synchronize()
    _, nor, post, comb = hc.collapse_norm(st, norm)
    out = G.hc_expand(moe, st, post, comb)
    torch.cuda.synchronize()
    assert torch.equal(g_nor, nor) and torch.equal(g_post, post) and torch.equal(g_comb, comb)
    assert torch.equal(g_out, out)
    del graph
