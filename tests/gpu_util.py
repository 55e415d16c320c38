"""Helpers shared by the GPU parity tests."""

from __future__ import annotations

import ctypes

import numpy as np
import torch

# North-star tolerances for BF16 layer outputs against the reference path.
MAX_ABS = 2e-2
MIN_COSINE = 0.9999


def bits(t: torch.Tensor) -> np.ndarray:
    """BF16 tensor -> numpy uint16 bit patterns (host copy)."""
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def from_bits(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def f32(a_bits: np.ndarray) -> np.ndarray:
    return (np.asarray(a_bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))


def bf16_ulp(v: np.ndarray) -> np.ndarray:
    """Spacing of BF16 values at |v| (2^(e-7) for |v| in [2^e, 2^(e+1)))."""
    a = np.abs(np.asarray(v, dtype=np.float32))
    e = np.floor(np.log2(np.maximum(a, np.float32(2.0 ** -126))))
    return np.exp2(e - 7).astype(np.float32)


def assert_layer_close(gpu_bits: np.ndarray, ref_bits: np.ndarray, *, max_abs: float = MAX_ABS,
                       min_cos: float = MIN_COSINE, certificate: dict | None = None) -> dict:
    """North-star layer tolerance: every element within max-abs 2e-2 of the
    oracle and cosine >= 0.9999 over the tensor.  An element beyond 2e-2 is
    accepted only when ``certificate`` (from ``certify_*``) proves the whole
    output: every intermediate BF16 / FP16 / FP32 value of the kernels lies in
    the oracle's rounding envelope of its exact value (a flip at a BF16
    rounding midpoint within the stated FP32 evaluation bound) and the final
    combine reproduces the output bit for bit from them.  Such elements are
    counted, with their size in BF16 ulps of the oracle value."""
    g, r = f32(gpu_bits), f32(ref_bits)
    assert np.isfinite(g).all(), "non-finite GPU output"
    diff = np.abs(g - r)
    err = float(diff.max()) if g.size else 0.0
    cos = cosine(g, r)
    same = float((np.asarray(gpu_bits) == np.asarray(ref_bits)).mean()) if g.size else 1.0
    over = diff > max_abs
    n_over = int(over.sum())
    ulps_over = sorted(set((diff[over] / bf16_ulp(r[over])).round(3).tolist())) if n_over else []
    if n_over:
        assert certificate is not None and certificate.get("certified"), (
            f"{n_over} elements beyond max-abs {max_abs} (largest {err}) and no rounding certificate")
    assert cos >= min_cos, f"cosine {cos} < {min_cos}"
    out = {"max_abs": err, "cosine": cos, "bit_identical": same, "beyond_max_abs_certified": n_over,
           "beyond_ulps": ulps_over}
    if n_over:
        print(f"[parity] {n_over} element(s) beyond {max_abs}: certified rounding flips of {ulps_over} BF16 ulp")
    return out


# ---------------------------------------------------------------------------
# Rounding certificates: every intermediate of the kernels against the
# oracle's envelope of its exact value, and the final combine bit for bit
# ---------------------------------------------------------------------------


def _f32_down(a: np.ndarray) -> np.ndarray:
    """Largest FP32 <= each float64 value."""
    f = a.astype(np.float32)
    return np.where(f.astype(np.float64) > a, np.nextafter(f, np.float32(-np.inf)), f)


def _f32_up(a: np.ndarray) -> np.ndarray:
    f = a.astype(np.float32)
    return np.where(f.astype(np.float64) < a, np.nextafter(f, np.float32(np.inf)), f)


def bf16_round(a) -> np.ndarray:
    """FP32 values -> nearest-even BF16 values, as FP32."""
    import oracle as O

    return O.f32_from_bf16(O.bf16_from_f32(np.asarray(a, dtype=np.float32)))


def certify_expert_rows(x_rows_bits, ids, bank, limit, hidden, down, *, down_kind: str,
                        hidden_fp16: bool = False) -> dict:
    """Certificate of per-route expert rows computed by the GPU.

    hidden: the kernel's SwiGLU hidden rows [R, I] as FP32 values (stored as
    BF16, or as FP16 when ``hidden_fp16``); down: the kernel's down
    projections [R, H] -- FP32 values before rounding (``down_kind="f32"``)
    or BF16 bits (``"bf16"``).
      1. every hidden value is one of the BF16 values reachable from the exact
         gate / up dot products by an FP32 evaluation within the stated bound
         (``oracle.hidden_envelope``; for FP16 storage, the FP16 roundings of
         the envelope's ends);
      2. every down value lies in the interval of every FP32 evaluation of the
         down projection of the kernel's own hidden row
         (``oracle.down_interval``), or, for BF16 rows, between the BF16
         roundings of its ends.
    Returns counts of the values that sit on a rounding flip."""
    import oracle as O

    h_lo, h_hi = O.hidden_envelope(x_rows_bits, ids, bank, limit)
    if hidden_fp16:
        h_lo = h_lo.astype(np.float16).astype(np.float32)
        h_hi = h_hi.astype(np.float16).astype(np.float32)
    hidden = np.asarray(hidden, dtype=np.float32)
    bad = (hidden < h_lo) | (hidden > h_hi)
    assert not bad.any(), (f"{int(bad.sum())} hidden values outside their rounding envelope, e.g. "
                           f"{hidden[bad][:4]} vs [{h_lo[bad][:4]}, {h_hi[bad][:4]}]")
    lo, hi = O.down_interval(hidden, ids, bank[2], bank[3])
    if down_kind == "f32":
        d = np.asarray(down, dtype=np.float32)
        ok = (d >= _f32_down(lo)) & (d <= _f32_up(hi))
        straddle = bf16_round(_f32_down(lo)) != bf16_round(_f32_up(hi))
    else:
        d = f32(down)
        d_lo, d_hi = bf16_round(_f32_down(lo)), bf16_round(_f32_up(hi))
        ok = (d >= d_lo) & (d <= d_hi)
        straddle = d_lo != d_hi
    assert ok.all(), (f"{int((~ok).sum())} down values outside the FP32 evaluation interval of the kernel's "
                      f"own hidden rows")
    return {"hidden_values": int(hidden.size), "hidden_envelope_two_or_more": int((h_hi > h_lo).sum()),
            "down_values": int(d.size), "down_on_bf16_midpoint_band": int(straddle.sum())}


def slot_combine(down_f32_rows, scores, shared=None) -> np.ndarray:
    """The packed decode / grouped combine (packed.py:168-179,
    grouped_fp8.py:273-276): FP32 slot-ordered sum of BF16 rows times FP32
    scores -> BF16, then the BF16 shared add.  down_f32_rows [k, ..., H] BF16
    values as FP32; returns BF16 bits."""
    import oracle as O

    total = np.zeros(down_f32_rows.shape[1:], dtype=np.float32)
    for j in range(down_f32_rows.shape[0]):
        s = np.asarray(scores[j], dtype=np.float32)
        s = s[..., None] if s.ndim else s
        total = total + down_f32_rows[j] * s
    res = bf16_round(total)
    if shared is not None:
        res = res + np.asarray(shared, dtype=np.float32)
    return O.bf16_from_f32(res)


def direct_combine(rows_f32, ids, scores, shared=None) -> np.ndarray:
    """DirectFP8MoE's multi-row combine (fp8.py:384-397): per token,
    BF16(row * score) added in BF16 in ascending expert id, then + shared.
    rows_f32 [T, k, H]; returns BF16 bits [T, H]."""
    import oracle as O

    T, k, H = rows_f32.shape
    order = np.argsort(np.asarray(ids).reshape(T, k), axis=1, kind="stable")
    acc = np.zeros((T, H), dtype=np.float32)
    tt = np.arange(T)
    for q in range(k):
        j = order[:, q]
        w = bf16_round(rows_f32[tt, j] * np.asarray(scores, dtype=np.float32).reshape(T, k)[tt, j][:, None])
        acc = bf16_round(acc + w)
    if shared is not None:
        acc = bf16_round(acc + np.asarray(shared, dtype=np.float32))
    return O.bf16_from_f32(acc)


def bank_host(bank, ids=None):
    """Host copies of the bank tensors (optionally only the experts in ids,
    re-indexed 0..len(ids)-1)."""
    ts = (bank.gate_up_weight, bank.gate_up_scale_inv, bank.down_weight, bank.down_scale_inv)
    if ids is not None:
        sel = torch.as_tensor(np.asarray(ids, dtype=np.int64), device=bank.gate_up_weight.device)
        ts = tuple(t.index_select(0, sel) for t in ts)
    return tuple(t.cpu().numpy() for t in ts)


def shared_host(shared_tensors):
    return None if shared_tensors is None else tuple(t.cpu().numpy() for t in shared_tensors)


def _shared_bank(shared_host_tuple):
    gw, gs, uw, us, dw, ds = shared_host_tuple
    return (np.concatenate([gw, uw])[None], np.concatenate([gs, us])[None], dw[None], ds[None])


def workspace_view(buf: torch.Tensor, offset: int, dtype, count: int) -> np.ndarray:
    """count values of dtype at byte offset of a device workspace (host copy)."""
    nbytes = np.dtype(dtype).itemsize * count
    return buf[offset:offset + nbytes].cpu().numpy().view(dtype)


def certify_packed_decode(x_bits, ids, scores, bank, shared, limit, out_bits, workspace: torch.Tensor) -> dict:
    """Certificate of one glm53_packed_decode_moe call from the intermediates
    it leaves in its workspace (glm53_packed_decode_workspace_layout): the
    routed and shared hidden rows and FP32 down projections are certified by
    ``certify_expert_rows``, and the output is K8's slot-ordered combine of the
    rounded down rows plus the rounded shared row, bit for bit.  bank / shared
    are host tuples (bank_host / shared_host)."""
    from glm53_flash_mlx_b200 import _native as N

    ids = np.asarray(ids, dtype=np.uint32).reshape(-1)
    top_k = ids.size
    H = bank[0].shape[2]
    I = bank[0].shape[1] // 2
    Is = 0 if shared is None else shared[0].shape[0]
    offs = (ctypes.c_size_t * 2)()
    N.check(N.lib().glm53_packed_decode_workspace_layout(top_k, H, I, Is, offs), "layout")
    hidden = f32(workspace_view(workspace, offs[0], np.uint16, top_k * I + Is))
    partial = workspace_view(workspace, offs[1], np.float32, (top_k + 1) * H).reshape(top_k + 1, H)
    x = np.asarray(x_bits, dtype=np.uint16).reshape(1, H)
    sc = np.asarray(scores, dtype=np.float32).reshape(-1)
    tensor_core = H % 128 == 0 and I % 128 == 0 and Is % 128 == 0
    if tensor_core:  # the tensor-core kernels keep the FP32 down projections
        cert = certify_expert_rows(np.repeat(x, top_k, 0), ids, bank, limit, hidden[:top_k * I].reshape(top_k, I),
                                   partial[:top_k], down_kind="f32")
        shared_row = None
        if shared is not None:
            cs = certify_expert_rows(x, np.zeros(1, np.uint32), _shared_bank(shared), limit,
                                     hidden[top_k * I:].reshape(1, Is), partial[top_k:top_k + 1], down_kind="f32")
            cert = {k: cert[k] + cs[k] for k in cert}
            shared_row = bf16_round(partial[top_k])
        expect = slot_combine(bf16_round(partial[:top_k]), sc, shared=shared_row)
        same = np.asarray(out_bits).reshape(-1) == expect
        assert same.all(), f"{int((~same).sum())} outputs differ from the combine of the certified intermediates"
        cert["certified"] = True
        return cert
    # the generic kernels reduce in registers: the hidden rows are certified,
    # then the output must lie in the combine of the down intervals of those
    # hidden rows (every step of the combine is monotone in each row)
    import oracle as O

    h_lo, h_hi = O.hidden_envelope(np.repeat(x, top_k, 0), ids, bank, limit)
    hr = hidden[:top_k * I].reshape(top_k, I)
    assert ((hr >= h_lo) & (hr <= h_hi)).all(), "hidden values outside their rounding envelope"
    lo, hi = O.down_interval(hr, ids, bank[2], bank[3])
    d_lo, d_hi = bf16_round(_f32_down(lo)), bf16_round(_f32_up(hi))
    t_lo = np.zeros(H, np.float32)
    t_hi = np.zeros(H, np.float32)
    for j in range(top_k):
        a, b = d_lo[j] * sc[j], d_hi[j] * sc[j]
        t_lo, t_hi = t_lo + np.minimum(a, b), t_hi + np.maximum(a, b)
    o_lo, o_hi = bf16_round(t_lo), bf16_round(t_hi)
    if shared is not None:
        hs = hidden[top_k * I:].reshape(1, Is)
        s_lo, s_hi = O.hidden_envelope(x, np.zeros(1, np.uint32), _shared_bank(shared), limit)
        assert ((hs >= s_lo) & (hs <= s_hi)).all(), "shared hidden values outside their rounding envelope"
        sl, shh = O.down_interval(hs, np.zeros(1, np.uint32), shared[4][None], shared[5][None])
        o_lo = bf16_round(o_lo + bf16_round(_f32_down(sl))[0])
        o_hi = bf16_round(o_hi + bf16_round(_f32_up(shh))[0])
    g = f32(np.asarray(out_bits, dtype=np.uint16)).reshape(-1)
    ok = (g >= o_lo) & (g <= o_hi)
    assert ok.all(), f"{int((~ok).sum())} outputs outside the combine of the certified rows' intervals"
    return {"certified": True, "hidden_values": int(hidden.size), "path": "generic (register reduce)"}


def certify_linear(x_bits, weight, scale_inv, y_bits) -> dict:
    """Certificate of a block-FP8 linear: each output is one of the BF16
    roundings of an FP32 evaluation of its dot product within the stated
    bound (one rounding site)."""
    import oracle as O

    x = f32(np.asarray(x_bits, dtype=np.uint16))
    M, K = x.shape
    N_ = weight.shape[0]
    lo, hi = O.down_interval(x, np.zeros(M, np.uint32), np.asarray(weight)[None], np.asarray(scale_inv)[None])
    y = f32(np.asarray(y_bits, dtype=np.uint16)).reshape(M, N_)
    d_lo, d_hi = bf16_round(_f32_down(lo)), bf16_round(_f32_up(hi))
    ok = (y >= d_lo) & (y <= d_hi)
    assert ok.all(), f"{int((~ok).sum())} linear outputs outside the FP32 evaluation interval"
    return {"certified": True, "outputs_on_bf16_midpoint_band": int((d_lo != d_hi).sum())}


def certify_grouped(x_bits, indices, scores, bank, shared, limit, out_bits, workspace: torch.Tensor,
                    tokens=None, bank_experts=None, expert_count=None) -> dict:
    """Certificate of one glm53_grouped_moe call (tensor-core path) for the
    listed tokens, from the intermediates it leaves in its workspace
    (glm53_grouped_moe_workspace_layout): each route's FP16 hidden row and
    BF16 down row, and the shared expert's, are certified by
    ``certify_expert_rows``; each token's output is restore_and_reduce's
    slot-ordered combine of its down rows plus its shared row, bit for bit.
    x_bits / indices / scores / out_bits cover all T tokens; bank / shared are
    host tuples (with ``bank_experts``, the bank holds only those experts, in
    that order, of ``expert_count``)."""
    from glm53_flash_mlx_b200 import _native as N

    x = np.asarray(x_bits, dtype=np.uint16)
    T, H = x.shape
    idx = np.asarray(indices).reshape(T, -1).astype(np.uint32)
    sc = np.asarray(scores, dtype=np.float32).reshape(T, -1)
    k = idx.shape[1]
    E = bank[0].shape[0] if expert_count is None else int(expert_count)
    I = bank[0].shape[1] // 2
    Is = 0 if shared is None else shared[0].shape[0]
    R = T * k
    offs = (ctypes.c_size_t * 8)()
    N.check(N.lib().glm53_grouped_moe_workspace_layout(T, k, E, H, I, Is, offs), "layout")
    inverse = workspace_view(workspace, offs[1], np.uint32, R)
    sorted_scores = workspace_view(workspace, offs[3], np.float32, R)
    tok = np.arange(T) if tokens is None else np.asarray(tokens)
    pos = inverse.reshape(T, k)[tok].reshape(-1).astype(np.int64)
    assert np.array_equal(sorted_scores[pos], sc[tok].reshape(-1)), "sorted scores do not match the routes"
    hid_all = workspace[offs[4]:offs[4] + R * I * 2].view(torch.float16).reshape(R, I)
    dn_all = workspace[offs[5]:offs[5] + R * H * 2].view(torch.int16).reshape(R, H)
    pos_t = torch.from_numpy(pos).to(workspace.device)
    hidden = hid_all.index_select(0, pos_t).float().cpu().numpy()
    down = dn_all.index_select(0, pos_t).cpu().numpy().view(np.uint16)
    # bank restricted to the touched experts (the certificate reads only those)
    ids = idx[tok].reshape(-1)
    if bank_experts is None:
        touched, local = np.unique(ids, return_inverse=True)
        sub = tuple(b[touched] for b in bank)
    else:
        be = np.asarray(bank_experts)
        local = np.searchsorted(be, ids)
        assert np.array_equal(be[local], ids), "bank_experts must hold every routed expert (sorted)"
        sub = bank
    cert = certify_expert_rows(np.repeat(x[tok], k, 0), local.astype(np.uint32), sub, limit, hidden, down,
                               down_kind="bf16", hidden_fp16=True)
    shared_rows = None
    if shared is not None:
        sh_h = workspace[offs[6]:offs[6] + T * Is * 2].view(torch.float16).reshape(T, Is)
        sh_o = workspace[offs[7]:offs[7] + T * H * 2].view(torch.int16).reshape(T, H)
        t_t = torch.from_numpy(tok.astype(np.int64)).to(workspace.device)
        sh_hidden = sh_h.index_select(0, t_t).float().cpu().numpy()
        sh_out = sh_o.index_select(0, t_t).cpu().numpy().view(np.uint16)
        cs = certify_expert_rows(x[tok], np.zeros(tok.size, np.uint32), _shared_bank(shared), limit, sh_hidden,
                                 sh_out, down_kind="bf16", hidden_fp16=True)
        cert = {key: cert[key] + cs[key] for key in cert}
        shared_rows = f32(sh_out)
    rows = f32(down).reshape(tok.size, k, H).transpose(1, 0, 2)
    expect = slot_combine(rows, sc[tok].T, shared=shared_rows)
    got = np.asarray(out_bits, dtype=np.uint16).reshape(T, H)[tok]
    same = got == expect
    assert same.all(), f"{int((~same).sum())} outputs differ from the combine of the certified intermediates"
    cert["certified"] = True
    return cert


def certify_grouped_linear(x_rows_bits, experts, weight, scale_inv, out_bits) -> dict:
    """Certificate of a grouped projection: row r of the output is one of the
    BF16 roundings of an FP32 evaluation of x[r] @ dequant(weight[experts[r]])^T
    within the stated bound."""
    import oracle as O

    x = f32(np.asarray(x_rows_bits, dtype=np.uint16))
    lo, hi = O.down_interval(x, np.asarray(experts, dtype=np.uint32), weight, scale_inv)
    y = f32(np.asarray(out_bits, dtype=np.uint16)).reshape(lo.shape)
    d_lo, d_hi = bf16_round(_f32_down(lo)), bf16_round(_f32_up(hi))
    ok = (y >= d_lo) & (y <= d_hi)
    assert ok.all(), f"{int((~ok).sum())} grouped outputs outside the FP32 evaluation interval"
    return {"certified": True, "outputs_on_bf16_midpoint_band": int((d_lo != d_hi).sum())}


def certify_by_envelope(gpu_bits, lo, hi) -> dict:
    """Output-level certificate: every GPU value inside the oracle's rounding
    envelope of the whole layer (``oracle.*_envelope``; wider than the staged
    certificates, used where the kernels' intermediates are not kept)."""
    g = f32(np.asarray(gpu_bits, dtype=np.uint16)).reshape(lo.shape)
    ok = (g >= lo) & (g <= hi)
    assert ok.all(), f"{int((~ok).sum())} outputs outside the layer's rounding envelope"
    return {"certified": True, "envelope": "layer"}


def router_logit_check(gpu_logits, ref64, x_bits, weight) -> dict:
    """FP32 router logits within 1e-6 relative of the FP64 oracle.  A logit
    whose relative error exceeds 1e-6 is accepted only when its absolute error
    is within the FP32 evaluation bound of the GPU router kernels,
    gamma(32) * sum_k |x_k w_k| (at most 32 FP32 roundings on a term's path:
    the small-batch kernel's 16 FMAs per thread, a 5-level warp sum and 8 warp
    partials; the tensor-core kernel's exact BF16 split with one rounding per
    MMA slice summed in double-FP32 stays far inside it): the logits near zero,
    where a relative error is ill-conditioned.  Returns their count."""
    g = np.asarray(gpu_logits, dtype=np.float64)
    r = np.asarray(ref64, dtype=np.float64)
    x = np.abs(f32(np.asarray(x_bits, dtype=np.uint16)).astype(np.float64)).reshape(g.shape[0], -1)
    absum = x @ np.abs(np.asarray(weight, dtype=np.float64)).T
    err = np.abs(g - r)
    rel_ok = err <= 1e-6 * np.abs(r)
    u = 2.0 ** -24
    bound_ok = err <= (32 * u / (1 - 32 * u)) * absum
    assert (rel_ok | bound_ok).all(), (
        f"{int((~(rel_ok | bound_ok)).sum())} logits beyond 1e-6 relative and the stated bound; worst rel "
        f"{float((err / np.maximum(np.abs(r), 1e-300)).max())}")
    return {"logits": int(g.size), "beyond_1e-6_relative_within_bound": int((~rel_ok).sum()),
            "max_rel": float((err / np.maximum(np.abs(r), 1e-30)).max())}


# ---------------------------------------------------------------------------
# FP8 tensor-core path (GLM53_FLAG_F8_MMA): activations as E4M3 term pairs
# ---------------------------------------------------------------------------


def term_rows(workspace: torch.Tensor, offset: int, rows, K: int):
    """hi, lo (FP32 values) of the E4M3 term rows [.., 2K bytes] at a byte
    offset of a device workspace, rows selected by index."""
    import oracle as O

    rows = np.asarray(rows, dtype=np.int64)
    n = int(rows.max()) + 1 if rows.size else 0
    buf = workspace[offset:offset + n * 2 * K].view(torch.uint8).reshape(n, 2 * K)
    t = buf.index_select(0, torch.from_numpy(rows).to(workspace.device)).cpu().numpy()
    tab = O.e4m3_table()
    return tab[t[:, :K]].astype(np.float32), tab[t[:, K:]].astype(np.float32)


def split_value(v, scale) -> np.ndarray:
    """The activation the FP8 kernel multiplies for value v of a row whose
    split scale is `scale`: (E4M3(v/s) + E4M3(v/s - E4M3(v/s))) * s.  Monotone
    in v, so it maps an envelope [lo, hi] onto [split(lo), split(hi)]."""
    import oracle as O

    s = np.asarray(scale, dtype=np.float32)
    vs = (np.asarray(v, dtype=np.float32) / s).astype(np.float32)
    hi = O.e4m3_round(vs)
    lo = O.e4m3_round((vs - hi).astype(np.float32))
    return ((hi.astype(np.float64) + lo) * s).astype(np.float32)


def _check_terms(hi, lo, scale, x_rows_bits, what: str) -> np.ndarray:
    """Kernel term rows against the oracle's split of the same BF16 rows,
    value for value; returns the represented rows as BF16 bits."""
    import oracle as O

    ohi, olo, osc = O.split_e4m3_rows(x_rows_bits)
    assert np.array_equal(scale, osc), f"{what}: split scales differ from the oracle's"
    assert np.array_equal(hi, ohi) and np.array_equal(lo, olo), f"{what}: E4M3 terms differ from the oracle's split"
    rep = ((hi.astype(np.float64) + lo) * scale[:, None]).astype(np.float32)
    rep_bits = O.bf16_from_f32(rep)
    assert np.array_equal(f32(rep_bits), rep), f"{what}: a represented activation is not a BF16 value"
    return rep_bits


def _certify_f8_rows(x_rep_bits, ids, bank, limit, h_hi, h_lo, h_scale, down_bits) -> dict:
    """Hidden terms and BF16 down rows of one F8 gate/up + down pair.

    The kernel's BF16 hidden value h (replaced in place by its terms) must lie
    in the hidden envelope of the represented input; its terms are the split
    of h at the row's scale, so (hi + lo) * scale lies in
    [split(env lo), split(env hi)].  The row scale must be the split scale of
    the row's largest term value (the maximum itself is exact).  The down row
    must be a BF16 rounding of an FP32 evaluation of the down projection of the
    represented hidden row."""
    import oracle as O

    e_lo, e_hi = O.hidden_envelope(x_rep_bits, ids, bank, limit)
    rep = ((h_hi.astype(np.float64) + h_lo) * h_scale[:, None]).astype(np.float32)
    m = np.abs(rep).max(axis=1)
    ex = np.frexp(m)[1]
    want = np.where(m > 0, np.ldexp(np.float32(1.0), np.maximum(ex - 8, -126)), np.float32(1.0))
    assert np.array_equal(h_scale, want.astype(np.float32)), "hidden split scales do not match the rows' maxima"
    q_lo, q_hi = split_value(e_lo, h_scale[:, None]), split_value(e_hi, h_scale[:, None])
    bad = (rep < q_lo) | (rep > q_hi)
    assert not bad.any(), (f"{int(bad.sum())} hidden terms outside the split of their rounding envelope, e.g. "
                           f"{rep[bad][:4]} vs [{q_lo[bad][:4]}, {q_hi[bad][:4]}]")
    lo, hi = O.down_interval(rep, ids, bank[2], bank[3])
    d = f32(down_bits)
    d_lo, d_hi = bf16_round(_f32_down(lo)), bf16_round(_f32_up(hi))
    ok = (d >= d_lo) & (d <= d_hi)
    assert ok.all(), f"{int((~ok).sum())} down values outside the FP32 evaluation interval of the represented rows"
    return {"hidden_values": int(rep.size), "hidden_envelope_two_or_more": int((e_hi > e_lo).sum()),
            "down_values": int(d.size), "down_on_bf16_midpoint_band": int((d_lo != d_hi).sum())}


def shared_down_splits(T: int, H: int, Is: int) -> int:
    """Split count the grouped composition gives the shared down projection
    (grouped_tc_splits over 128x128 output tiles); the FP8 shared pair runs
    only unsplit."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    tiles = ((T + 127) // 128) * ((H + 127) // 128)
    if Is <= 0 or Is % 128 or tiles * 2 > sms:
        return 1
    return max(1, min(sms // tiles, (Is // 128) // 4))


def certify_grouped_f8(x_bits, indices, scores, bank, shared, limit, out_bits, workspace: torch.Tensor,
                       tokens=None, bank_experts=None, expert_count=None) -> dict:
    """Certificate of one GLM53_FLAG_F8_MMA glm53_grouped_moe call for the
    listed tokens, from the intermediates it leaves in its workspace
    (glm53_grouped_moe_workspace_layout, glm53_grouped_moe_term_layout):

      1. every route's input terms and scale equal the oracle's split of its
         token row (``oracle.split_e4m3_rows``), value for value;
      2. hidden terms and down rows of the routed and the shared pair are
         certified against the represented input (``_certify_f8_rows``);
      3. each token's output is restore_and_reduce's slot-ordered combine of
         its down rows plus its shared row, bit for bit.

    The certificate proves the kernels' arithmetic on the represented
    activations; the representation itself (exact within 2^9 of each row's
    maximum) is counted in ``inexact_inputs`` / ``inexact_hidden``."""
    from glm53_flash_mlx_b200 import _native as N

    x = np.asarray(x_bits, dtype=np.uint16)
    T, H = x.shape
    idx = np.asarray(indices).reshape(T, -1).astype(np.uint32)
    sc = np.asarray(scores, dtype=np.float32).reshape(T, -1)
    k = idx.shape[1]
    E = bank[0].shape[0] if expert_count is None else int(expert_count)
    I = bank[0].shape[1] // 2
    Is = 0 if shared is None else shared[0].shape[0]
    R = T * k
    offs = (ctypes.c_size_t * 8)()
    N.check(N.lib().glm53_grouped_moe_workspace_layout(T, k, E, H, I, Is, offs), "layout")
    toffs = (ctypes.c_size_t * 6)()
    N.check(N.lib().glm53_grouped_moe_term_layout(T, k, E, H, I, Is, toffs), "term layout")
    inverse = workspace_view(workspace, offs[1], np.uint32, R)
    sorted_scores = workspace_view(workspace, offs[3], np.float32, R)
    tok = np.arange(T) if tokens is None else np.asarray(tokens)
    pos = inverse.reshape(T, k)[tok].reshape(-1).astype(np.int64)
    assert np.array_equal(sorted_scores[pos], sc[tok].reshape(-1)), "sorted scores do not match the routes"
    ids = idx[tok].reshape(-1)
    if bank_experts is None:
        touched, local = np.unique(ids, return_inverse=True)
        sub = tuple(b[touched] for b in bank)
    else:
        be = np.asarray(bank_experts)
        local = np.searchsorted(be, ids)
        assert np.array_equal(be[local], ids), "bank_experts must hold every routed expert (sorted)"
        sub = bank
    x_rows = np.repeat(x[tok], k, 0)
    hi, lo = term_rows(workspace, toffs[0], pos, H)
    xs = workspace_view(workspace, toffs[1], np.float32, R)[pos]
    x_rep = _check_terms(hi, lo, xs, x_rows, "routed input")
    hh, hl = term_rows(workspace, offs[4], pos, I)
    hs = workspace_view(workspace, toffs[2], np.float32, R)[pos]
    dn_all = workspace[offs[5]:offs[5] + R * H * 2].view(torch.int16).reshape(R, H)
    down = dn_all.index_select(0, torch.from_numpy(pos).to(workspace.device)).cpu().numpy().view(np.uint16)
    cert = _certify_f8_rows(x_rep, local.astype(np.uint32), sub, limit, hh, hl, hs, down)
    cert["inexact_inputs"] = int((x_rep != x_rows).sum())
    shared_rows = None
    if shared is not None:
        t_t = torch.from_numpy(tok.astype(np.int64)).to(workspace.device)
        sh_o = workspace[offs[7]:offs[7] + T * H * 2].view(torch.int16).reshape(T, H)
        sh_out = sh_o.index_select(0, t_t).cpu().numpy().view(np.uint16)
        if shared_down_splits(T, H, Is) == 1:
            shi, slo = term_rows(workspace, toffs[3], tok, H)
            ssc = workspace_view(workspace, toffs[4], np.float32, T)[tok]
            s_rep = _check_terms(shi, slo, ssc, x[tok], "shared input")
            sh, sl = term_rows(workspace, offs[6], tok, Is)
            shs = workspace_view(workspace, toffs[5], np.float32, T)[tok]
            cs = _certify_f8_rows(s_rep, np.zeros(tok.size, np.uint32), _shared_bank(shared), limit, sh, sl, shs,
                                  sh_out)
        else:  # a split shared down projection runs the shared pair on the kind::f16 kernels
            sh_h = workspace[offs[6]:offs[6] + T * Is * 2].view(torch.float16).reshape(T, Is)
            cs = certify_expert_rows(x[tok], np.zeros(tok.size, np.uint32), _shared_bank(shared), limit,
                                     sh_h.index_select(0, t_t).float().cpu().numpy(), sh_out, down_kind="bf16",
                                     hidden_fp16=True)
        cert = {key: cert[key] + cs[key] if key in cs else cert[key] for key in cert}
        shared_rows = f32(sh_out)
    rows = f32(down).reshape(tok.size, k, H).transpose(1, 0, 2)
    expect = slot_combine(rows, sc[tok].T, shared=shared_rows)
    got = np.asarray(out_bits, dtype=np.uint16).reshape(T, H)[tok]
    same = got == expect
    assert same.all(), f"{int((~same).sum())} outputs differ from the combine of the certified intermediates"
    cert["certified"] = True
    return cert


def check_grouped_route_plan(workspace: torch.Tensor, indices, scores, E: int, H: int, I: int, Is: int) -> None:
    """The route plan a glm53_grouped_moe call leaves in its workspace (order,
    inverse, sorted expert ids and scores) equals the oracle's stable expert
    sort of the same routes, element for element."""
    import oracle as O
    from glm53_flash_mlx_b200 import _native as N

    idx = np.asarray(indices)
    T, k = idx.shape
    R = T * k
    offs = (ctypes.c_size_t * 8)()
    N.check(N.lib().glm53_grouped_moe_workspace_layout(T, k, E, H, I, Is, offs), "layout")
    rp = O.route_plan(idx.reshape(-1).astype(np.uint32), E, np.asarray(scores, dtype=np.float32).reshape(-1))
    for name, off, dt in (("order", 0, np.uint32), ("inverse", 1, np.uint32), ("sorted_experts", 2, np.uint32),
                          ("sorted_scores", 3, np.float32)):
        got = workspace_view(workspace, offs[off], dt, R)
        assert np.array_equal(got, rp[name]), f"route plan {name} differs from the oracle's stable sort"
