"""Pin the CPU oracle against the reference's own known answers (CPU only)."""

import hashlib
import json
from pathlib import Path

import ml_dtypes
import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
KATS = json.loads((GOLDEN / "reference_kats.json").read_text())


def _sigmoid_domain(O):
    bits = np.arange(1 << 16, dtype=np.uint16)
    vals = O.f32_from_bf16(bits)
    return bits[np.isfinite(vals) & (np.abs(vals) <= np.float32(10.0))]


def test_e4m3_table_matches_reference_table(oracle):
    ref = np.array(KATS["e4m3_table"]["values"], dtype=np.float32)
    lut = oracle.e4m3_table()
    assert np.array_equal(lut.view(np.uint32), ref.view(np.uint32))  # includes -0.0 at 0x80
    assert lut[0x7F] == 480.0 and lut[0xFF] == -480.0


def test_e4m3_table_differs_from_e4m3fn_only_at_0x7f_0xff(oracle):
    lut = oracle.e4m3_table()
    std = np.arange(256, dtype=np.uint8).view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    differ = [c for c in range(256) if not (lut[c] == std[c])]
    assert differ == [0x7F, 0xFF]
    assert np.isnan(std[0x7F]) and np.isnan(std[0xFF])


def test_sigmoid_sweep_reproduces_reference_hash(oracle):
    kat = KATS["sigmoid_sweep"]
    dom = _sigmoid_domain(oracle)
    assert dom.size == kat["domain_elements"]
    assert hashlib.sha256(dom.tobytes()).hexdigest() == kat["domain_bits_sha256"]
    sig = oracle.sigmoid_bf16(dom)
    assert hashlib.sha256(sig.tobytes()).hexdigest() == kat["reference_sigmoid_sha256"]


def test_standard_bf16_formula_matches_reference_standard_hash(oracle):
    """A numpy restatement of the standard per-op BF16 formula (correctly
    rounded exp) reproduces the reference's standard_bf16 hash, and differs
    from the reference sigmoid at exactly the one recorded element."""
    kat = KATS["sigmoid_sweep"]
    O = oracle
    dom = _sigmoid_domain(O)
    g = O.f32_from_bf16(dom)
    e = O.bf16_from_f32(np.exp(np.abs(g).astype(np.float64)).astype(np.float32))
    den = O.bf16_from_f32(np.float32(1) + O.f32_from_bf16(e))
    tail = O.bf16_from_f32(np.float32(1) / O.f32_from_bf16(den))
    sig = np.where(g < 0, tail, O.bf16_from_f32(np.float32(1) - O.f32_from_bf16(tail))).astype(np.uint16)
    assert hashlib.sha256(sig.tobytes()).hexdigest() == kat["standard_bf16_sha256"]
    pinned = O.sigmoid_bf16(dom)
    diff = np.flatnonzero(pinned != sig)
    first = kat["standard_bf16_first_difference"]
    assert diff.tolist() == [first["index"]]
    assert f"0x{int(sig[first['index']]):04x}" == first["actual_bits"]
    assert f"0x{int(pinned[first['index']]):04x}" == first["reference_bits"]


def test_tile_descriptor_known_answer(oracle):
    kat = KATS["tile_descriptors"]
    sorted_experts = np.array([0] * 31 + [1] * 32 + [287] * 33, dtype=np.uint32)
    te, ts, tl, ro, to = oracle.tile_plan(sorted_experts, kat["expert_count"], kat["tile_rows"])
    valid = ts < sorted_experts.size
    assert [list(map(int, t)) for t in zip(te[valid], ts[valid], tl[valid])] == kat["valid"]
    assert te.size == (96 + 31) // 32 + 288
    # sentinels: expert 0, start = routes, length 0
    assert set(te[~valid].tolist()) == {0} and set(ts[~valid].tolist()) == {96} and set(tl[~valid].tolist()) == {0}
    counts = np.diff(ro)
    assert int((counts > 0).sum()) == kat["unique_experts"]
    assert int((counts == 0).sum()) == kat["zero_route_experts"]
    covered = np.zeros(96, dtype=int)
    for s, n in zip(ts[valid], tl[valid]):
        covered[s : s + n] += 1
    assert (covered == 1).all()
    # no descriptor crosses an expert boundary
    for e, s, n in zip(te[valid], ts[valid], tl[valid]):
        assert (sorted_experts[s : s + n] == e).all()


def test_score_recompute_known_answer(oracle):
    kat = KATS["score_recompute"]
    O = oracle
    w = np.array(kat["weight"], dtype=np.float32)
    x = O.bf16_from_f32(np.array([kat["x"]], dtype=np.float32))
    # the recorded ids [2, 0] are kept; only their weights are recomputed
    idx, sc, logits, margin = O.router(x, w, np.zeros(3, np.float32), top_k=2,
                                       routed_scaling_factor=kat["routed_scaling_factor"])
    np.testing.assert_allclose(logits[0], [1.0, 2.0, 3.0])
    got = O.scores_for_indices(logits, np.array([kat["indices"]]),
                               routed_scaling_factor=kat["routed_scaling_factor"])
    np.testing.assert_allclose(got[0], kat["expected_scores"], rtol=kat["tolerance"], atol=kat["tolerance"])
    # the router's own selection is the top-2 by sigmoid(logit) + bias
    assert idx[0].tolist() == [2, 1]
    np.testing.assert_allclose(sc[0], O.scores_for_indices(logits, idx, routed_scaling_factor=2.0)[0], rtol=1e-6)


def test_block_linear_matches_dequantised_matmul(oracle):
    """tests/test_fp8_metal.py:23-39 restated: 129 x 257 crosses block edges."""
    O = oracle
    rng = np.random.default_rng(1)
    m, k = 129, 257
    codes = rng.integers(0, 247, (m, k)).astype(np.uint8)
    scales = (rng.uniform(size=(2, 3)) * 0.02).astype(np.float32)
    x = O.bf16_from_f32(rng.normal(size=(2, k)).astype(np.float32))
    y = O.block_fp8_linear(x, codes, scales)
    dense = O.e4m3_table()[codes] * np.repeat(np.repeat(scales, 128, 0), 128, 1)[:m, :k]
    expected = O.bf16_from_f32(O.f32_from_bf16(x) @ dense.T)
    assert np.abs(O.f32_from_bf16(y) - O.f32_from_bf16(expected)).max() <= 0.03125


def test_route_plan_is_stable_counting_sort(oracle):
    rng = np.random.default_rng(2)
    ids = rng.integers(0, 40, 997).astype(np.uint32)
    ids[::97] = 50  # out of range for E = 40
    plan = oracle.route_plan(ids, 40, rng.uniform(size=997).astype(np.float32))
    valid = ids < 40
    expected = np.concatenate([np.argsort(np.where(valid, ids, 40), kind="stable")])
    assert np.array_equal(plan["order"], expected)
    assert np.array_equal(plan["inverse"][plan["order"]], np.arange(997))
    assert plan["invalid"] == int((~valid).sum())
    assert np.array_equal(plan["expert_offsets"], np.concatenate([[0], np.cumsum(np.bincount(ids[valid], minlength=40))]))


def test_oracle_regression_fixtures(oracle):
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    fx = np.load(GOLDEN / "oracle_small.npz")
    inputs = mg.small_inputs()
    assert str(fx["inputs_sha256"]) == mg.inputs_digest(inputs), "seeded inputs changed"
    fresh = mg.oracle_small()
    for key in fx.files:
        if key == "inputs_sha256":
            continue
        assert np.array_equal(fresh[key], fx[key]), key


def test_packed_decode_oracle_equals_direct_composition(oracle):
    """The fused decode oracle equals the Direct composition (selected
    projections, BF16 SwiGLU, down, FP32 slot sum) -- the reference's
    packed == Direct bit-equality (tests/test_fp8_metal.py:140-145)."""
    O = oracle
    fx = np.load(GOLDEN / "oracle_small.npz")
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    d = mg.small_inputs()
    I = 129
    gate = np.stack([O.block_fp8_linear(d["dec_x"], d["dec_gu_w"][e, :I], d["dec_gu_s"][e, :2]) for e in d["dec_ids"]])
    up = np.stack([O.block_fp8_linear(d["dec_x"], d["dec_gu_w"][e, I:], d["dec_gu_s"][e, 2:]) for e in d["dec_ids"]])
    hidden = O.swiglu_bf16(gate, up, 3.0)
    assert np.array_equal(hidden.reshape(-1), fx["dec_hidden"][: 8 * I])
    down = np.stack([O.block_fp8_linear(hidden[j], d["dec_d_w"][e], d["dec_d_s"][e]) for j, e in enumerate(d["dec_ids"])])
    total = np.zeros(257, np.float32)
    for j in range(8):
        total = total + O.f32_from_bf16(down[j]) * d["dec_scores"][j]
    routed = O.bf16_from_f32(total)
    shared = O.shared_expert(d["dec_x"], tuple(d["dec_" + n] for n in ("sg_w", "sg_s", "su_w", "su_s", "sd_w", "sd_s")), 3.0)
    assert np.array_equal(O.bf16_add(routed, shared), fx["dec_y"])


@pytest.mark.parametrize("limit", [3.0, 10.0])
def test_swiglu_clamps(oracle, limit):
    O = oracle
    g = O.bf16_from_f32(np.array([50.0, -50.0, 0.0, limit], np.float32))
    u = O.bf16_from_f32(np.array([50.0, -50.0, 1.0, 1.0], np.float32))
    h = O.f32_from_bf16(O.swiglu_bf16(g, u, limit))
    expected = limit * limit / (1.0 + np.exp(-limit))  # silu(L) * L after both clamps
    assert abs(h[0] - expected) <= expected * 2 ** -6
    assert abs(h[1]) < 1e-3
    assert h[2] == 0.0


def test_e4m3_round_matches_ml_dtypes_and_the_table(oracle):
    """oracle.e4m3_round (the FP8 path's activation conversion) is the
    round-to-nearest-even E4M3 conversion: identity on every finite table
    value, equal to ml_dtypes' float8_e4m3fn cast inside the finite range,
    saturating at +-448 above it."""
    lut = oracle.e4m3_table()
    fin = np.abs(lut) <= 448
    assert np.array_equal(oracle.e4m3_round(lut[fin]), lut[fin])
    rng = np.random.default_rng(7)
    a = (rng.standard_normal(200_000) * np.exp2(rng.integers(-14, 9, 200_000))).astype(np.float32)
    a = a[np.abs(a) < 464]
    want = a.astype(ml_dtypes.float8_e4m3fn).astype(np.float32)
    assert np.array_equal(oracle.e4m3_round(a), want)
    assert oracle.e4m3_round(np.float32([500.0, -1e9]))[0] == 448.0
    assert oracle.e4m3_round(np.float32([-1e9]))[0] == -448.0


def test_split_e4m3_rows_is_exact_within_2e9_of_the_row_maximum(oracle):
    """(hi + lo) * scale reproduces every BF16 element within 2^9 of its row
    maximum, and misses a smaller one by at most 2^-10 * scale."""
    rng = np.random.default_rng(8)
    x = (rng.standard_normal((32, 1024)) * np.exp2(rng.integers(-20, 20, (32, 1)))).astype(np.float32)
    x[3, :50] *= 1e-6
    x[5] = 0
    xb = oracle.bf16_from_f32(x)
    xv = oracle.f32_from_bf16(xb).astype(np.float64)
    hi, lo, s = oracle.split_e4m3_rows(xb)
    rep = (hi.astype(np.float64) + lo) * s[:, None]
    m = np.abs(xv).max(axis=1, keepdims=True)
    exact = np.abs(xv) >= m * 2.0 ** -9
    assert np.array_equal(rep[exact], xv[exact])
    assert (np.abs(rep - xv) <= 2.0 ** -10 * s[:, None]).all()
    assert (np.abs(hi) <= 448).all() and (np.abs(hi).max(axis=1)[m[:, 0] > 0] >= 128).all()
    assert s[5] == 1.0 and not rep[5].any()

