"""numpy/ctypes front end of the C oracle -- TEST INFRASTRUCTURE ONLY.

BF16 tensors are numpy ``uint16`` bit patterns, E4M3 weights ``uint8`` codes,
scales ``float32``.  Each function names the reference flow it restates; the
scalar arithmetic is in ``oracle.c``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import numpy as np

__all__ = [
    "oracle_lib",
    "e4m3_table",
    "bf16_from_f32",
    "f32_from_bf16",
    "sigmoid_bf16",
    "swiglu_bf16",
    "block_fp8_linear",
    "packed_decode_moe",
    "router",
    "scores_for_indices",
    "route_plan",
    "tile_plan",
    "grouped_linear",
    "activate_gate_up",
    "restore_and_reduce",
    "bf16_add",
    "shared_expert",
    "direct_moe",
    "grouped_moe",
    "default_threads",
    "hc_collapse_norm",
    "rms_norm",
    "hc_expand",
    "head_major_to_rows",
    "envelope_depth",
    "rows_envelope",
    "packed_decode_envelope",
    "grouped_envelope",
    "direct_envelope",
    "hidden_envelope",
    "down_interval",
    "e4m3_round",
    "split_e4m3_rows",
]

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_lock = threading.Lock()
_lib = None

_u8 = ctypes.POINTER(ctypes.c_uint8)
_u16 = ctypes.POINTER(ctypes.c_uint16)
_u32 = ctypes.POINTER(ctypes.c_uint32)
_f32 = ctypes.POINTER(ctypes.c_float)
_f64 = ctypes.POINTER(ctypes.c_double)
_i64 = ctypes.c_int64


def default_threads() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:  # pragma: no cover
        return max(1, os.cpu_count() or 1)


def build_oracle() -> Path:
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def oracle_lib():
    global _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                build_oracle()
            lib = ctypes.CDLL(str(_LIB_PATH))
            sig = {
                "orc_e4m3_table": (None, [_f32]),
                "orc_sigmoid_bf16_vec": (None, [_u16, _i64, _u16]),
                "orc_swiglu_bf16_vec": (None, [_u16, _u16, _i64, ctypes.c_float, _u16]),
                "orc_block_fp8_linear": (ctypes.c_int, [_u16, _i64, _i64, _u8, _i64, _f32, _u16, ctypes.c_int]),
                "orc_packed_decode_moe": (
                    ctypes.c_int,
                    [_u16, _i64, _u32, _f32, ctypes.c_int, _u8, _f32, _u8, _f32, _i64, _i64,
                     _u8, _f32, _u8, _f32, _u8, _f32, _i64, ctypes.c_float, _u16, _u16, ctypes.c_int],
                ),
                "orc_router": (
                    ctypes.c_int,
                    [_u16, _i64, _i64, _f32, _i64, _f32, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                     ctypes.c_int, ctypes.c_float, _u32, _f32, _f64, _f32, _f32, ctypes.c_int],
                ),
                "orc_route_plan": (ctypes.c_int, [_u32, _i64, _i64, _f32, _u32, _u32, _u32, _f32, _u32, _u32]),
                "orc_tile_plan": (ctypes.c_int, [_u32, _i64, _i64, _i64, _u32, _u32, _u32, _u32, _u32, _u32]),
                "orc_grouped_linear": (ctypes.c_int, [_u16, _i64, _i64, _u32, _u8, _i64, _i64, _f32, _u16, ctypes.c_int]),
                "orc_activate_gate_up": (None, [_u16, _i64, _i64, ctypes.c_float, _u16]),
                "orc_restore_and_reduce": (None, [_u16, _f32, _u32, _i64, ctypes.c_int, _i64, _u16]),
                "orc_bf16_add": (None, [_u16, _u16, _i64, _u16]),
                "orc_hc_collapse_norm": (
                    ctypes.c_int,
                    [_u16, _i64, _i64, ctypes.c_int, _u16, _f32, _f32, ctypes.c_int, ctypes.c_float,
                     ctypes.c_float, _u16, ctypes.c_float, _u16, _u16, _f32, _f32, _f32, ctypes.c_int],
                ),
                "orc_rms_norm_bf16": (None, [_u16, _i64, _i64, _u16, ctypes.c_float, _u16]),
                "orc_hc_expand": (None, [_u16, _u16, _f32, _f32, _i64, _i64, _u16]),
                "orc_down_interval": (
                    ctypes.c_int,
                    [_f32, _i64, _i64, _u32, _u8, _f32, _i64, _i64, ctypes.c_int, _f64, _f64, ctypes.c_int],
                ),
                "orc_rows_envelope": (
                    ctypes.c_int64,
                    [_u16, _i64, _i64, _u32, _u8, _f32, _u8, _f32, _i64, _i64, ctypes.c_float, ctypes.c_int,
                     ctypes.c_int, _f32, _f32, _f32, _f32, ctypes.c_int],
                ),
            }
            for name, (res, args) in sig.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def _p(a: np.ndarray | None, ptype):
    if a is None:
        return ctypes.cast(None, ptype)
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ptype)


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=dtype))


# ----------------------------------------------------------------------------
# scalar helpers
# ----------------------------------------------------------------------------


def e4m3_table() -> np.ndarray:
    out = np.empty(256, dtype=np.float32)
    oracle_lib().orc_e4m3_table(_p(out, _f32))
    return out


def bf16_from_f32(a) -> np.ndarray:
    """Round-to-nearest-even FP32 -> BF16 bit patterns."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    b = a.view(np.uint32).astype(np.uint64)
    out = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = ((a.view(np.uint32)[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def f32_from_bf16(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def sigmoid_bf16(g_bits) -> np.ndarray:
    g = _c(g_bits, np.uint16).reshape(-1)
    out = np.empty_like(g)
    oracle_lib().orc_sigmoid_bf16_vec(_p(g, _u16), g.size, _p(out, _u16))
    return out


def swiglu_bf16(gate_bits, up_bits, limit: float) -> np.ndarray:
    g = _c(gate_bits, np.uint16)
    u = _c(up_bits, np.uint16)
    assert g.shape == u.shape
    out = np.empty_like(g)
    oracle_lib().orc_swiglu_bf16_vec(_p(g, _u16), _p(u, _u16), g.size, float(limit), _p(out, _u16))
    return out


def bf16_add(a, b) -> np.ndarray:
    a = _c(a, np.uint16)
    b = _c(b, np.uint16)
    out = np.empty_like(a)
    oracle_lib().orc_bf16_add(_p(a, _u16), _p(b, _u16), a.size, _p(out, _u16))
    return out


# ----------------------------------------------------------------------------
# K1/K2 block linear, packed decode
# ----------------------------------------------------------------------------


def block_fp8_linear(x_bits, weight, scale_inv, *, threads: int | None = None) -> np.ndarray:
    """glm53_flash_mlx/fp8.py:254-299 over [..., K] BF16 inputs."""
    x = _c(x_bits, np.uint16)
    w = _c(weight, np.uint8)
    s = _c(scale_inv, np.float32)
    n, k = w.shape
    flat = x.reshape(-1, k)
    out = np.empty((flat.shape[0], n), dtype=np.uint16)
    if flat.shape[0]:
        rc = oracle_lib().orc_block_fp8_linear(
            _p(flat, _u16), flat.shape[0], k, _p(w, _u8), n, _p(s, _f32), _p(out, _u16),
            threads or default_threads(),
        )
        assert rc == 0
    return out.reshape(*x.shape[:-1], n)


def packed_decode_moe(x_bits, ids, scores, bank, shared, limit: float, *,
                      threads: int | None = None, return_hidden: bool = False):
    """PackedFP8MoE.__call__ for one token (glm53_flash_mlx/packed.py:896-923).

    ``bank`` = (gate_up_w [E,2I,H], gate_up_s, down_w [E,H,I], down_s);
    ``shared`` = None or (gate_w, gate_s, up_w, up_s, down_w, down_s)."""
    x = _c(x_bits, np.uint16).reshape(-1)
    ids = _c(ids, np.uint32).reshape(-1)
    scores = _c(scores, np.float32).reshape(-1)
    gu_w, gu_s, d_w, d_s = (_c(bank[0], np.uint8), _c(bank[1], np.float32),
                            _c(bank[2], np.uint8), _c(bank[3], np.float32))
    E, two_i, H = gu_w.shape
    I = two_i // 2
    top_k = ids.size
    if shared is not None:
        sg_w, sg_s, su_w, su_s, sd_w, sd_s = (
            _c(shared[0], np.uint8), _c(shared[1], np.float32), _c(shared[2], np.uint8),
            _c(shared[3], np.float32), _c(shared[4], np.uint8), _c(shared[5], np.float32))
        Is = sg_w.shape[0]
    else:
        sg_w = sg_s = su_w = su_s = sd_w = sd_s = None
        Is = 0
    out = np.empty(H, dtype=np.uint16)
    hidden = np.empty(top_k * I + Is, dtype=np.uint16)
    rc = oracle_lib().orc_packed_decode_moe(
        _p(x, _u16), H, _p(ids, _u32), _p(scores, _f32), top_k,
        _p(gu_w, _u8), _p(gu_s, _f32), _p(d_w, _u8), _p(d_s, _f32), E, I,
        _p(sg_w, _u8), _p(sg_s, _f32), _p(su_w, _u8), _p(su_s, _f32), _p(sd_w, _u8), _p(sd_s, _f32), Is,
        float(limit), _p(out, _u16), _p(hidden, _u16), threads or default_threads(),
    )
    if rc == 3:
        raise IndexError("expert id out of range")
    assert rc == 0
    return (out, hidden) if return_hidden else out


# ----------------------------------------------------------------------------
# Router
# ----------------------------------------------------------------------------


def router(x_bits, weight, bias, *, top_k: int = 8, n_group: int = 1, topk_group: int = 1,
           norm_topk_prob: bool = True, routed_scaling_factor: float = 1.0,
           threads: int | None = None):
    """Float32Gate + group_expert_select (glm53_flash_mlx/patch.py:131-142).

    Returns (indices u32 [T,k], scores f32 [T,k], logits f64 [T,E],
    margin f32 [T]) where margin = choice[k-th] - choice[(k+1)-th best]."""
    x = _c(x_bits, np.uint16)
    w = _c(weight, np.float32)
    b = _c(bias, np.float32)
    E, H = w.shape
    flat = x.reshape(-1, H)
    T = flat.shape[0]
    idx = np.empty((T, top_k), dtype=np.uint32)
    sc = np.empty((T, top_k), dtype=np.float32)
    l64 = np.empty((T, E), dtype=np.float64)
    margin = np.empty(T, dtype=np.float32)
    rc = oracle_lib().orc_router(
        _p(flat, _u16), T, H, _p(w, _f32), E, _p(b, _f32), int(top_k), int(n_group),
        int(topk_group), int(bool(norm_topk_prob)), float(routed_scaling_factor),
        _p(idx, _u32), _p(sc, _f32), _p(l64, _f64), None, _p(margin, _f32),
        threads or default_threads(),
    )
    if rc != 0:
        raise ValueError("invalid router geometry")
    return idx, sc, l64, margin


def scores_for_indices(logits, indices, *, norm_topk_prob: bool = True, routed_scaling_factor: float = 1.0):
    """Route weights for given expert ids: sigmoid(logits) taken at the ids,
    normalised over the slots, times the scaling factor (the indices-only gate
    of scripts/localize_grouped_fp8_divergence.py, restated)."""
    lg = np.asarray(logits, dtype=np.float64)
    idx = np.asarray(indices, dtype=np.int64)
    sc = np.take_along_axis(1.0 / (1.0 + np.exp(-lg)), idx, axis=-1)
    if idx.shape[-1] > 1 and norm_topk_prob:
        sc = sc / sc.sum(axis=-1, keepdims=True)
    return (sc * routed_scaling_factor).astype(np.float32)


# ----------------------------------------------------------------------------
# Route plan / tile plan / grouped linear
# ----------------------------------------------------------------------------


def route_plan(ids, expert_count: int, scores=None):
    """Stable expert sort (glm53_flash_mlx/grouped_fp8.py:157-170)."""
    ids = _c(ids, np.uint32).reshape(-1)
    R = ids.size
    sc = None if scores is None else _c(scores, np.float32).reshape(-1)
    order = np.empty(R, np.uint32)
    inverse = np.empty(R, np.uint32)
    sorted_experts = np.empty(R, np.uint32)
    sorted_scores = np.empty(R, np.float32)
    offsets = np.empty(expert_count + 1, np.uint32)
    invalid = np.zeros(1, np.uint32)
    oracle_lib().orc_route_plan(
        _p(ids, _u32), R, expert_count, _p(sc, _f32), _p(order, _u32), _p(inverse, _u32),
        _p(sorted_experts, _u32), _p(sorted_scores, _f32), _p(offsets, _u32), _p(invalid, _u32),
    )
    return {
        "order": order,
        "inverse": inverse,
        "sorted_experts": sorted_experts,
        "sorted_scores": sorted_scores if sc is not None else None,
        "expert_offsets": offsets,
        "invalid": int(invalid[0]),
    }


def tile_plan(sorted_experts, expert_count: int, tile_rows: int = 32):
    """build_grouped_tile_plan (glm53_flash_mlx/grouped_fp8.py:173-203):
    (tile_experts, tile_starts, tile_lengths, route_offsets, tile_offsets)."""
    se = _c(sorted_experts, np.uint32).reshape(-1)
    R = se.size
    cap = (R + tile_rows - 1) // tile_rows + expert_count
    te = np.empty(cap, np.uint32)
    ts = np.empty(cap, np.uint32)
    tl = np.empty(cap, np.uint32)
    ro = np.empty(expert_count + 1, np.uint32)
    to = np.empty(expert_count + 1, np.uint32)
    cnt = np.zeros(1, np.uint32)
    oracle_lib().orc_tile_plan(
        _p(se, _u32), R, expert_count, tile_rows, _p(te, _u32), _p(ts, _u32), _p(tl, _u32),
        _p(ro, _u32), _p(to, _u32), _p(cnt, _u32),
    )
    return te, ts, tl, ro, to


def grouped_linear(x_sorted_bits, sorted_experts, weight, scale_inv, *,
                   threads: int | None = None) -> np.ndarray:
    """K12 semantics (glm53_flash_mlx/grouped_fp8.py:30-154, 206-262)."""
    x = _c(x_sorted_bits, np.uint16)
    se = _c(sorted_experts, np.uint32).reshape(-1)
    w = _c(weight, np.uint8)
    s = _c(scale_inv, np.float32)
    E, N, K = w.shape
    R = x.shape[0]
    out = np.zeros((R, N), dtype=np.uint16)
    oracle_lib().orc_grouped_linear(
        _p(x, _u16), R, K, _p(se, _u32), _p(w, _u8), E, N, _p(s, _f32), _p(out, _u16),
        threads or default_threads(),
    )
    return out


def activate_gate_up(gate_up_bits, intermediate_size: int, limit: float) -> np.ndarray:
    g = _c(gate_up_bits, np.uint16)
    R = g.shape[0]
    out = np.empty((R, intermediate_size), dtype=np.uint16)
    oracle_lib().orc_activate_gate_up(_p(g, _u16), R, intermediate_size, float(limit), _p(out, _u16))
    return out


def restore_and_reduce(sorted_out_bits, sorted_scores, inverse, tokens: int, top_k: int) -> np.ndarray:
    so = _c(sorted_out_bits, np.uint16)
    ss = _c(sorted_scores, np.float32)
    inv = _c(inverse, np.uint32)
    H = so.shape[1]
    out = np.empty((tokens, H), dtype=np.uint16)
    oracle_lib().orc_restore_and_reduce(_p(so, _u16), _p(ss, _f32), _p(inv, _u32), tokens, top_k, H, _p(out, _u16))
    return out


# ----------------------------------------------------------------------------
# Module-level flows
# ----------------------------------------------------------------------------


def shared_expert(x_bits, shared, limit: float, *, threads: int | None = None) -> np.ndarray:
    """ClampedMLP / DirectFP8Expert over BlockFP8Linear projections
    (glm53_flash_mlx/fp8.py:329-340): down(silu(min(gate, L)) * clip(up))."""
    gate = block_fp8_linear(x_bits, shared[0], shared[1], threads=threads)
    up = block_fp8_linear(x_bits, shared[2], shared[3], threads=threads)
    hidden = swiglu_bf16(gate, up, limit)
    return block_fp8_linear(hidden, shared[4], shared[5], threads=threads)


def _bank_expert(bank, e: int):
    gu_w, gu_s, d_w, d_s = bank
    I = gu_w.shape[1] // 2
    half = gu_s.shape[1] // 2
    return (gu_w[e, :I], gu_s[e, :half], gu_w[e, I:], gu_s[e, half:], d_w[e], d_s[e])


def direct_moe(x_bits, indices, scores, bank, shared, limit: float, *,
               threads: int | None = None) -> np.ndarray:
    """DirectFP8MoE prefill semantics (glm53_flash_mlx/fp8.py:384-397):
    ascending expert id, BF16 scatter-add of expert_out * score, + shared."""
    x = _c(x_bits, np.uint16)
    H = x.shape[-1]
    flat = x.reshape(-1, H)
    routes = _c(indices, np.int64).reshape(flat.shape[0], -1)
    sc = _c(scores, np.float32).reshape(flat.shape[0], -1)
    result = np.zeros(flat.shape, dtype=np.uint16)
    for e in np.unique(routes):
        rows, slots = np.nonzero(routes == e)
        expert = _bank_expert(bank, int(e))
        out = shared_expert(flat[rows], expert, limit, threads=threads)
        weighted = f32_from_bf16(out) * sc[rows, slots][:, None]
        upd = bf16_from_f32(weighted)
        result[rows] = bf16_add(result[rows], upd)
    if shared is not None:
        result = bf16_add(result, shared_expert(flat, shared, limit, threads=threads))
    return result.reshape(x.shape)


def grouped_moe(x_bits, indices, scores, bank, shared, limit: float, *,
                threads: int | None = None) -> np.ndarray:
    """SortedGroupedFP8MoE.grouped_from_routes (glm53_flash_mlx/grouped_fp8.py:294-321)."""
    x = _c(x_bits, np.uint16)
    H = x.shape[-1]
    flat = x.reshape(-1, H)
    T = flat.shape[0]
    idx = _c(indices, np.uint32).reshape(T, -1)
    top_k = idx.shape[1]
    plan = route_plan(idx.reshape(-1), bank[0].shape[0], _c(scores, np.float32).reshape(-1))
    sorted_x = flat[plan["order"] // top_k]
    I = bank[0].shape[1] // 2
    gate_up = grouped_linear(sorted_x, plan["sorted_experts"], bank[0], bank[1], threads=threads)
    hidden = activate_gate_up(gate_up, I, limit)
    down = grouped_linear(hidden, plan["sorted_experts"], bank[2], bank[3], threads=threads)
    result = restore_and_reduce(down, plan["sorted_scores"], plan["inverse"], T, top_k)
    if shared is not None:
        result = bf16_add(result, shared_expert(flat, shared, limit, threads=threads))
    return result.reshape(x.shape)


# ----------------------------------------------------------------------------
# FFN boundary: mHC collapse + RMSNorm (before the router), hc expand (after)
# ----------------------------------------------------------------------------

def hc_collapse_norm(state_bits, fn_bits, scale, base, norm_weight_bits=None, *,
                     sinkhorn_iters: int = 20, eps: float = 1e-6, norm_eps: float = 1e-6,
                     rms_eps: float = 1e-6, threads: int | None = None):
    """mHC collapse of ``state`` [T, 4, H] and the post-attention RMSNorm
    (the ``layer.ffn_hc`` -> ``layer.post_attention_layernorm`` sequence of
    scripts/profile_native_prefill_ffn_entry_seam.py:79-81).  Returns
    ``(collapsed [T,H] u16, normalized [T,H] u16 or None, post [T,4] f32,
    comb [T,4,4] f32, mixes [T,24] f32)``.  Parity of the collapse itself is
    unpinned (mlx-vlm's module is absent); see ``orc_hc_collapse_norm``."""
    state = _c(state_bits, np.uint16)
    T, n, H = state.shape
    fn = _c(fn_bits, np.uint16)
    if fn.shape != ((2 + n) * n, n * H):
        raise ValueError(f"hc fn shape {fn.shape} != {((2 + n) * n, n * H)}")
    scale = _c(scale, np.float32)
    base = _c(base, np.float32)
    w = None if norm_weight_bits is None else _c(norm_weight_bits, np.uint16)
    collapsed = np.zeros((T, H), np.uint16)
    normalized = None if w is None else np.zeros((T, H), np.uint16)
    post = np.zeros((T, n), np.float32)
    comb = np.zeros((T, n, n), np.float32)
    mixes = np.zeros((T, (2 + n) * n), np.float32)
    rc = oracle_lib().orc_hc_collapse_norm(
        _p(state, _u16), T, H, n, _p(fn, _u16), _p(scale, _f32), _p(base, _f32), sinkhorn_iters,
        eps, norm_eps, _p(w, _u16), rms_eps, _p(collapsed, _u16), _p(normalized, _u16),
        _p(post, _f32), _p(comb, _f32), _p(mixes, _f32), threads or default_threads())
    if rc:
        raise ValueError("oracle hc_collapse_norm: unsupported geometry")
    return collapsed, normalized, post, comb, mixes


def rms_norm(x_bits, weight_bits, eps: float = 1e-6) -> np.ndarray:
    """MLX fast RMSNorm over BF16 rows: BF16(w * BF16(x * rsqrt(mean(x^2)+eps)))."""
    x = _c(x_bits, np.uint16)
    T, H = x.reshape(-1, x.shape[-1]).shape
    w = _c(weight_bits, np.uint16)
    out = np.zeros_like(x)
    oracle_lib().orc_rms_norm_bf16(_p(x, _u16), T, H, _p(w, _u16), eps, _p(out, _u16))
    return out


def hc_expand(moe_bits, residual_bits, post, comb) -> np.ndarray:
    """hc expand of the MoE output into the 4-branch state
    (native_execution/native_indexer_plan.metal:2362-2389)."""
    moe = _c(moe_bits, np.uint16)
    residual = _c(residual_bits, np.uint16)
    T, n, H = residual.shape
    post = _c(post, np.float32)
    comb = _c(comb, np.float32)
    out = np.zeros((T, n, H), np.uint16)
    oracle_lib().orc_hc_expand(_p(moe, _u16), _p(residual, _u16), _p(post, _f32), _p(comb, _f32),
                               T, H, _p(out, _u16))
    return out


def head_major_to_rows(head_major_bits) -> np.ndarray:
    """[heads, rows, dim] -> [rows, heads * dim]: the index map of
    glm53_native_prefill_dsa_head_to_row_bfloat16
    (native_execution/native_indexer_plan.metal:2290-2304), position
    (head, row, d) -> row_major[(row * heads + head) * dim + d]."""
    hm = np.asarray(head_major_bits)
    heads, rows, dim = hm.shape
    out = np.empty(rows * heads * dim, dtype=hm.dtype)
    for head in range(heads):
        for row in range(rows):
            start = (row * heads + head) * dim
            out[start:start + dim] = hm[head, row]
    return out.reshape(rows, heads * dim)


# ----------------------------------------------------------------------------
# Rounding envelopes: the tolerance certificates of the parity tests
# ----------------------------------------------------------------------------

# FP32 roundings on any term's path through one projection of length K in
# the CUDA kernels (orc_rows_envelope states the model): two per MMA and
# eight MMAs per 128-K block (16), the block-scale product (1), one per block
# of the FP32 sum over blocks (ceil(K / 128)) and up to eight for a
# cross-warp or split-K reduction tree.
def envelope_depth(K: int) -> int:
    return 25 + (int(K) + 127) // 128


ENVELOPE_DEPTH = None  # per projection: envelope_depth(K)


def _bf16_round_f32(a) -> np.ndarray:
    """f32 values -> nearest BF16 values (as f32)."""
    return f32_from_bf16(bf16_from_f32(np.asarray(a, dtype=np.float32)))


def rows_envelope(x_rows_bits, ids, bank, limit: float, *, depth: int | None = None,
                  threads: int | None = None):
    """Envelope [lo, hi] (f32 arrays [R, H] of BF16 values) of the BF16 down
    row of expert ids[r] applied to x_rows[r], over every FP32 evaluation
    order of its dot products (orc_rows_envelope)."""
    x = _c(x_rows_bits, np.uint16)
    ids = _c(ids, np.uint32).reshape(-1)
    gu_w, gu_s, d_w, d_s = (_c(bank[0], np.uint8), _c(bank[1], np.float32),
                            _c(bank[2], np.uint8), _c(bank[3], np.float32))
    E, two_i, H = gu_w.shape
    R = ids.size
    x = x.reshape(R, H)
    lo = np.empty((R, H), dtype=np.float32)
    hi = np.empty((R, H), dtype=np.float32)
    if R:
        cut = oracle_lib().orc_rows_envelope(
            _p(x, _u16), R, H, _p(ids, _u32), _p(gu_w, _u8), _p(gu_s, _f32), _p(d_w, _u8), _p(d_s, _f32), E,
            two_i // 2, float(limit), depth or envelope_depth(H), depth or envelope_depth(two_i // 2),
            _p(lo, _f32), _p(hi, _f32), _p(None, _f32), _p(None, _f32), threads or default_threads())
        if cut < 0:
            raise IndexError("expert id out of range")
        assert cut == 0, f"{cut} candidate sets were cut: the envelope is incomplete"
    return lo, hi


def _shared_as_bank(shared):
    gw, gs, uw, us, dw, ds = (np.asarray(t) for t in shared)
    return (np.concatenate([gw, uw])[None], np.concatenate([gs, us])[None], dw[None], ds[None])


def _shared_envelope(x_rows_bits, shared, limit, threads):
    if shared is None:
        return None
    R = x_rows_bits.shape[0]
    return rows_envelope(x_rows_bits, np.zeros(R, np.uint32), _shared_as_bank(shared), limit, threads=threads)


def _slot_sum_envelope(d_lo, d_hi, scores):
    """FP32 slot-ordered weighted sum (packed.py:168-179 / grouped_fp8.py:273-276)
    at both envelope ends; every step is monotone in each term."""
    lo = np.zeros(d_lo.shape[1:], dtype=np.float32)
    hi = np.zeros(d_lo.shape[1:], dtype=np.float32)
    for j in range(d_lo.shape[0]):
        s = np.float32(scores[j])
        a, b = d_lo[j] * s, d_hi[j] * s
        lo = lo + np.minimum(a, b)
        hi = hi + np.maximum(a, b)
    return lo, hi


def packed_decode_envelope(x_bits, ids, scores, bank, shared, limit: float, *, threads: int | None = None):
    """Envelope of PackedFP8MoE's one-token decode output: K8's FP32
    slot-ordered sum -> BF16, then the BF16 shared add, applied to the ends
    of the routed and shared rows' envelopes.  Returns (lo, hi, pre_lo,
    pre_hi): the output ends and the FP32 range of the final rounding's
    argument."""
    x = _c(x_bits, np.uint16).reshape(1, -1)
    ids = _c(ids, np.uint32).reshape(-1)
    sc = _c(scores, np.float32).reshape(-1)
    d_lo, d_hi = rows_envelope(np.repeat(x, ids.size, 0), ids, bank, limit, threads=threads)
    t_lo, t_hi = _slot_sum_envelope(d_lo, d_hi, sc)
    r_lo, r_hi = _bf16_round_f32(t_lo), _bf16_round_f32(t_hi)
    sh = _shared_envelope(x, shared, limit, threads)
    if sh is None:
        return r_lo, r_hi, t_lo, t_hi
    p_lo, p_hi = r_lo + sh[0][0], r_hi + sh[1][0]
    return _bf16_round_f32(p_lo), _bf16_round_f32(p_hi), p_lo, p_hi


def grouped_envelope(x_bits, indices, scores, bank, shared, limit: float, *, tokens=None,
                     threads: int | None = None):
    """Envelope of SortedGroupedFP8MoE's output rows (restore_and_reduce's FP32
    slot sum -> BF16, + BF16 shared) for the listed tokens (default all).
    Returns (lo, hi) [len(tokens), H]."""
    x = _c(x_bits, np.uint16)
    H = x.shape[-1]
    flat = x.reshape(-1, H)
    idx = _c(indices, np.uint32).reshape(flat.shape[0], -1)
    sc = _c(scores, np.float32).reshape(flat.shape[0], -1)
    tok = np.arange(flat.shape[0]) if tokens is None else np.asarray(tokens)
    k = idx.shape[1]
    rows = np.repeat(flat[tok], k, 0)
    d_lo, d_hi = rows_envelope(rows, idx[tok].reshape(-1), bank, limit, threads=threads)
    d_lo = d_lo.reshape(tok.size, k, H)
    d_hi = d_hi.reshape(tok.size, k, H)
    lo = np.zeros((tok.size, H), dtype=np.float32)
    hi = np.zeros((tok.size, H), dtype=np.float32)
    for j in range(k):
        s = sc[tok, j][:, None]
        a, b = d_lo[:, j] * s, d_hi[:, j] * s
        lo = lo + np.minimum(a, b)
        hi = hi + np.maximum(a, b)
    lo, hi = _bf16_round_f32(lo), _bf16_round_f32(hi)
    sh = _shared_envelope(flat[tok], shared, limit, threads)
    if sh is not None:
        lo, hi = _bf16_round_f32(lo + sh[0]), _bf16_round_f32(hi + sh[1])
    return lo, hi


def direct_envelope(x_bits, indices, scores, bank, shared, limit: float, *, threads: int | None = None):
    """Envelope of DirectFP8MoE's multi-row output (fp8.py:384-397): per token,
    BF16(row * score) added in BF16 in ascending expert id, then the BF16
    shared output added.  Returns (lo, hi) [T, H]."""
    x = _c(x_bits, np.uint16)
    H = x.shape[-1]
    flat = x.reshape(-1, H)
    T = flat.shape[0]
    idx = _c(indices, np.int64).reshape(T, -1)
    sc = _c(scores, np.float32).reshape(T, -1)
    k = idx.shape[1]
    d_lo, d_hi = rows_envelope(np.repeat(flat, k, 0), idx.reshape(-1), bank, limit, threads=threads)
    d_lo = d_lo.reshape(T, k, H)
    d_hi = d_hi.reshape(T, k, H)
    lo = np.zeros((T, H), dtype=np.float32)
    hi = np.zeros((T, H), dtype=np.float32)
    order = np.argsort(idx, axis=1, kind="stable")
    tt = np.arange(T)
    for q in range(k):
        j = order[:, q]
        s = sc[tt, j][:, None]
        a = _bf16_round_f32(d_lo[tt, j] * s)
        b = _bf16_round_f32(d_hi[tt, j] * s)
        lo = _bf16_round_f32(lo + np.minimum(a, b))
        hi = _bf16_round_f32(hi + np.maximum(a, b))
    sh = _shared_envelope(flat, shared, limit, threads)
    if sh is not None:
        lo, hi = _bf16_round_f32(lo + sh[0]), _bf16_round_f32(hi + sh[1])
    return lo, hi


def hidden_envelope(x_rows_bits, ids, bank, limit: float, *, depth: int | None = None,
                    threads: int | None = None):
    """Envelope [lo, hi] (f32 [R, I], BF16 values) of the SwiGLU hidden row of
    expert ids[r] applied to x_rows[r]: the BF16 values that any FP32
    evaluation order of the gate / up dot products can lead to."""
    x = _c(x_rows_bits, np.uint16)
    ids = _c(ids, np.uint32).reshape(-1)
    gu_w, gu_s = _c(bank[0], np.uint8), _c(bank[1], np.float32)
    E, two_i, H = gu_w.shape
    I = two_i // 2
    R = ids.size
    x = x.reshape(R, H)
    lo = np.empty((R, I), dtype=np.float32)
    hi = np.empty((R, I), dtype=np.float32)
    if R:
        dummy_w = np.zeros((1, 1, 1), np.uint8)
        cut = oracle_lib().orc_rows_envelope(
            _p(x, _u16), R, H, _p(ids, _u32), _p(gu_w, _u8), _p(gu_s, _f32), _p(dummy_w, _u8),
            _p(np.zeros(1, np.float32), _f32), E, I, float(limit), depth or envelope_depth(H), 1, _p(None, _f32),
            _p(None, _f32), _p(lo, _f32), _p(hi, _f32), threads or default_threads())
        if cut < 0:
            raise IndexError("expert id out of range")
        assert cut == 0, f"{cut} candidate sets were cut: the envelope is incomplete"
    return lo, hi


def down_interval(hidden_f32, ids, down_w, down_s, *, depth: int | None = None, threads: int | None = None):
    """Real interval (f64 [R, H] lo, hi) containing every FP32 evaluation of
    the down projection of the given hidden rows (orc_down_interval)."""
    h = _c(hidden_f32, np.float32)
    ids = _c(ids, np.uint32).reshape(-1)
    d_w, d_s = _c(down_w, np.uint8), _c(down_s, np.float32)
    E, H, I = d_w.shape
    R = ids.size
    h = h.reshape(R, I)
    lo = np.empty((R, H), dtype=np.float64)
    hi = np.empty((R, H), dtype=np.float64)
    if R:
        rc = oracle_lib().orc_down_interval(_p(h, _f32), R, I, _p(ids, _u32), _p(d_w, _u8), _p(d_s, _f32), E, H,
                                            depth or envelope_depth(I), _p(lo, _f64), _p(hi, _f64),
                                            threads or default_threads())
        if rc == 3:
            raise IndexError("expert id out of range")
        assert rc == 0
    return lo, hi


def e4m3_round(a) -> np.ndarray:
    """Nearest E4M3 value of each FP32 value (ties to even, saturating at
    +-448, NaN kept): the conversion the kind::f8f6f4 activation split uses
    (PTX cvt.rn.satfinite.e4m3x2.f32).  E4M3 has 3 fraction bits, normals
    from 2^-6, subnormals spaced 2^-9."""
    a = np.asarray(a, dtype=np.float64)
    m = np.abs(a)
    e = np.floor(np.log2(np.maximum(m, 2.0 ** -6)))
    q = np.exp2(e - 3)
    r = np.minimum(np.rint(m / q) * q, 448.0)
    return np.copysign(r, a).astype(np.float32)


def split_e4m3_rows(x_bits):
    """hi, lo (FP32 values of E4M3 codes, [R, K]) and scale ([R]) of the
    activation split of the kind::f8f6f4 path: e = frexp(max |x|) - 8
    (at least -126; 0 for an all-zero row) puts the row maximum in
    [128, 256); hi = E4M3(x 2^-e), lo = E4M3(x 2^-e - hi), scale = 2^e.
    (hi + lo) * scale is the activation the tensor cores multiply; it equals
    x for every element within 2^9 of the row maximum."""
    x = f32_from_bf16(np.asarray(x_bits, dtype=np.uint16)).astype(np.float32)
    x = x.reshape(-1, x.shape[-1]) if x.ndim > 1 else x.reshape(1, -1)
    m = np.abs(x).max(axis=1) if x.size else np.zeros(x.shape[0], np.float32)
    ex = np.frexp(m)[1].astype(np.int64)
    e = np.where((m > 0) & np.isfinite(m), np.maximum(ex - 8, -126), 0)
    xs = (x * np.ldexp(np.float32(1.0), -e)[:, None].astype(np.float32)).astype(np.float32)
    hi = e4m3_round(xs)
    lo = e4m3_round((xs - hi).astype(np.float32))
    scale = np.ldexp(np.float32(1.0), e).astype(np.float32)
    scale = np.where(np.isinf(m), np.float32(np.nan), scale).astype(np.float32)
    return hi, lo, scale
