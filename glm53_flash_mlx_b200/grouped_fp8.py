"""Sorted-route grouped block-FP8 prefill MoE on B200.

Counterpart of glm53_flash_mlx/grouped_fp8.py: ``build_route_plan``
(:157-170), ``build_grouped_tile_plan`` (:173-203), ``grouped_fp8_linear``
(:206-262), ``activate_gate_up`` (:265-270), ``restore_and_reduce``
(:273-276) and ``SortedGroupedFP8MoE`` (:279-328).  Every step runs on the
device without a host synchronisation; ``SortedGroupedFP8MoE`` runs the whole
layer through one C-ABI call (route plan, grouped gate/up with a fused SwiGLU
epilogue, grouped down, slot-ordered combine, shared expert, BF16 add).
"""

from __future__ import annotations

import torch

from . import _native as N
from .abi import GROUPED_KERNEL_ABI, GROUPED_MEASURED_CROSSOVER_ROUTES, GROUPED_MIN_ROUTES  # noqa: F401
from .fp8 import BLOCK_SIZE
from .packed import PackedFP8MoE, check_status, shared_fp8_tensors, _SYNC_STATUS

GROUPED_TILE_ROWS = 32
GROUPED_OUTPUT_COLS = 32
GROUPED_K_TILE = 32
# Route rows per tensor-core tile of the B200 grouped kernel.
DEVICE_TILE_ROWS = 128
# Largest expert count of the device route plan (csrc/route_plan.cu).
ROUTE_PLAN_MAX_EXPERTS = 1024


def _route_plan(expert_ids: torch.Tensor, expert_count: int, scores: torch.Tensor | None, tile_rows: int):
    dev = N.require_cuda(expert_ids)
    ids = expert_ids.reshape(-1).to(torch.int32).contiguous()
    R = ids.numel()
    cap = (R + tile_rows - 1) // tile_rows + expert_count
    u32 = torch.int32
    order = torch.empty(R, dtype=u32, device=dev)
    inverse = torch.empty(R, dtype=u32, device=dev)
    sorted_experts = torch.empty(R, dtype=u32, device=dev)
    sc = None if scores is None else scores.reshape(-1).to(torch.float32).contiguous()
    sorted_scores = None if sc is None else torch.empty(R, dtype=torch.float32, device=dev)
    route_offsets = torch.empty(expert_count + 1, dtype=u32, device=dev)
    tile_offsets = torch.empty(expert_count + 1, dtype=u32, device=dev)
    te = torch.empty(cap, dtype=u32, device=dev)
    ts = torch.empty(cap, dtype=u32, device=dev)
    tl = torch.empty(cap, dtype=u32, device=dev)
    counts = torch.zeros(2, dtype=u32, device=dev)
    N.check(
        N.lib().glm53_route_plan(
            ids.data_ptr(), R, expert_count, tile_rows, N.ptr(sc), order.data_ptr(), inverse.data_ptr(),
            sorted_experts.data_ptr(), N.ptr(sorted_scores), route_offsets.data_ptr(), te.data_ptr(),
            ts.data_ptr(), tl.data_ptr(), tile_offsets.data_ptr(), counts.data_ptr(), counts[1:].data_ptr(),
            N.stream(dev),
        ),
        "glm53_route_plan",
    )
    return {
        "order": order,
        "inverse": inverse,
        "sorted_experts": sorted_experts,
        "sorted_scores": sorted_scores,
        "route_offsets": route_offsets,
        "tile_offsets": tile_offsets,
        "tile_experts": te,
        "tile_starts": ts,
        "tile_lengths": tl,
        "descriptor_count": counts[0:1],
        "invalid_count": counts[1:2],
    }


def build_route_plan(x, topk_indices, topk_scores):
    """Return a fully device-resident expert-sorted route plan:
    (sorted_x, sorted_experts, sorted_scores, inverse_order).  Routes are
    ordered by expert id, ties by route index (stable)."""
    flat_x = x.reshape(-1, x.shape[-1]).contiguous()
    top_k = topk_indices.shape[-1]
    # No host read of the largest id: the device histogram spans every id the
    # route plan supports (ROUTE_PLAN_MAX_EXPERTS); larger ids sort last.
    plan = _route_plan(topk_indices, ROUTE_PLAN_MAX_EXPERTS, topk_scores, GROUPED_TILE_ROWS)
    R = plan["order"].numel()
    sorted_x = torch.empty((R, flat_x.shape[1]), dtype=flat_x.dtype, device=flat_x.device)
    if R:
        N.check(
            N.lib().glm53_gather_rows(flat_x.data_ptr(), flat_x.shape[1], plan["order"].data_ptr(), R, top_k,
                                      sorted_x.data_ptr(), N.stream(flat_x.device)),
            "glm53_gather_rows",
        )
    return sorted_x, plan["sorted_experts"], plan["sorted_scores"], plan["inverse"]


def build_grouped_tile_plan(sorted_experts, expert_count: int, *, tile_rows: int = GROUPED_TILE_ROWS):
    """Expert-aligned fixed-capacity tile descriptors, built on the device:
    (tile_experts, tile_starts, tile_lengths, route_offsets, tile_offsets).
    capacity = ceil(routes / tile_rows) + expert_count; unused slots are the
    sentinel (expert 0, start = routes, length 0)."""
    plan = _route_plan(sorted_experts, expert_count, None, tile_rows)
    return (plan["tile_experts"], plan["tile_starts"], plan["tile_lengths"], plan["route_offsets"],
            plan["tile_offsets"])


_LINEAR_WS = N.Workspace()
_LINEAR_STATUS: dict = {}


def grouped_fp8_linear(x, tile_plan, weight, scale_inv, *, tile_rows: int = GROUPED_TILE_ROWS):
    """Project sorted route rows from a packed block-FP8 expert bank.

    Runs the tcgen05 grouped GEMM (exact FP16 weights, FP32 accumulation with
    per-128-K promotion) over the plan's descriptors; ``tile_rows`` is the
    longest descriptor the plan may hold (``build_grouped_tile_plan``'s
    ``tile_rows``).  A longer descriptor, or an expert id out of range, sets a
    device status bit that raises at the next call (``RuntimeError`` /
    ``IndexError``)."""
    if weight.dtype != torch.uint8 or weight.dim() != 3:
        raise ValueError("grouped weight must be [experts, out, in] uint8 E4M3")
    if scale_inv.dtype != torch.float32 or scale_inv.dim() != 3:
        raise ValueError("grouped scale must be [experts, out_blocks, in_blocks] FP32")
    routes, in_features = x.shape
    experts, out_features, weight_in = weight.shape
    if (out_features % BLOCK_SIZE != 0 or in_features % BLOCK_SIZE != 0
            or out_features % GROUPED_OUTPUT_COLS != 0 or in_features % GROUPED_K_TILE != 0):
        raise ValueError(
            "grouped probe requires block-aligned projection dimensions; "
            f"got out={out_features}, in={in_features}"
        )
    expected_scales = (experts, (out_features + BLOCK_SIZE - 1) // BLOCK_SIZE,
                       (in_features + BLOCK_SIZE - 1) // BLOCK_SIZE)
    if weight_in != in_features or tuple(scale_inv.shape) != expected_scales:
        raise ValueError(
            f"incompatible grouped shapes x={tuple(x.shape)}, weight={tuple(weight.shape)}, "
            f"scale={tuple(scale_inv.shape)}, expected_scale={expected_scales}"
        )
    if x.dtype != torch.bfloat16:
        raise ValueError(f"grouped_fp8_linear computes on BF16 activations, got {x.dtype}")
    tile_experts, tile_starts, tile_lengths = (t.contiguous() for t in tile_plan[:3])
    dev = N.require_cuda(x, weight, scale_inv, tile_experts)
    x = x.contiguous()
    weight = weight.contiguous()
    out = torch.empty((routes, out_features), dtype=x.dtype, device=dev)
    if routes:
        from .packed import StatusWord

        sw = _LINEAR_STATUS.get(dev)
        if sw is None:
            sw = _LINEAR_STATUS[dev] = StatusWord(dev)
        sw.raise_pending()
        stream = N.stream(dev)
        ws = _LINEAR_WS.get(dev, f"rows:{stream}", N.lib().glm53_grouped_fp8_linear_workspace_bytes(routes, in_features))
        N.check(
            N.lib().glm53_grouped_fp8_linear_ws(
                x.data_ptr(), routes, in_features, tile_experts.data_ptr(), tile_starts.data_ptr(),
                tile_lengths.data_ptr(), tile_experts.numel(), int(tile_rows), weight.data_ptr(), experts,
                out_features, scale_inv.contiguous().data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(),
                sw.word.data_ptr(), N.decode_flags(weight), stream,
            ),
            "glm53_grouped_fp8_linear_ws",
        )
        sw.publish()
        if _SYNC_STATUS:
            sw.check()
    return out


def activate_gate_up(gate_up, intermediate_size: int, limit: float):
    if intermediate_size % BLOCK_SIZE != 0:
        raise ValueError("gate/up split must align to the block-128 scale boundary")
    dev = N.require_cuda(gate_up)
    g = gate_up.contiguous()
    R = g.shape[0]
    hidden = torch.empty((R, intermediate_size), dtype=torch.bfloat16, device=dev)
    if R:
        N.check(N.lib().glm53_activate_gate_up(g.data_ptr(), R, intermediate_size, float(limit), hidden.data_ptr(),
                                               N.stream(dev)), "glm53_activate_gate_up")
    return hidden


def restore_and_reduce(sorted_output, sorted_scores, inverse_order, shape, top_k, shared=None):
    """FP32 weighted restore of the sorted rows and slot-ordered sum -> BF16,
    plus an optional BF16 shared-expert add."""
    dev = N.require_cuda(sorted_output, sorted_scores, inverse_order)
    H = shape[-1]
    T = inverse_order.numel() // top_k
    out = torch.empty((T, H), dtype=sorted_output.dtype, device=dev)
    sh = None if shared is None else shared.reshape(T, H).contiguous()
    if T:
        N.check(
            N.lib().glm53_restore_and_reduce(
                sorted_output.contiguous().data_ptr(), sorted_scores.contiguous().data_ptr(),
                inverse_order.to(torch.int32).contiguous().data_ptr(), T, top_k, H, N.ptr(sh), out.data_ptr(),
                N.stream(dev),
            ),
            "glm53_restore_and_reduce",
        )
    return out.reshape(shape)


def grouped_moe(x, indices, scores, bank, shared, *, limit: float, workspace: N.Workspace | None = None,
                status: torch.Tensor | None = None, mma: str = "f16"):
    """Whole grouped prefill layer from given routes (one C-ABI call).

    mma="f8" runs the grouped GEMMs on the FP8 tensor-core kernel
    (GLM53_FLAG_F8_MMA: E4M3 weights straight into tcgen05 kind::f8f6f4,
    activations as hi + lo E4M3 terms, exact within 2^9 of each row's
    maximum) when the bank has no 0x7F/0xFF codes; otherwise, and with "f16",
    the kind::f16 kernel."""
    if mma not in ("f16", "f8"):
        raise ValueError(f"mma must be 'f16' or 'f8', got {mma!r}")
    dev = N.require_cuda(x, indices, scores, bank.gate_up_weight)
    H = bank.hidden_size
    I = bank.intermediate_size
    flat = x.reshape(-1, H).contiguous()
    if flat.dtype != torch.bfloat16:
        raise ValueError(f"grouped MoE computes on BF16 activations, got {flat.dtype}")
    T = flat.shape[0]
    top_k = indices.shape[-1]
    idx = indices.reshape(-1).to(torch.int32).contiguous()
    sc = scores.reshape(-1).to(torch.float32).contiguous()
    if shared is not None:
        sg_w, sg_s, su_w, su_s, sd_w, sd_s = shared
        Is = sg_w.shape[0]
    else:
        sg_w = sg_s = su_w = su_s = sd_w = sd_s = None
        Is = 0
    flags = N.decode_flags(bank.gate_up_weight, bank.down_weight, *(() if shared is None else (sg_w, su_w, sd_w)))
    if mma == "f8":
        flags |= N.FLAG_F8_MMA
    wsp = workspace or N.Workspace()
    nbytes = N.lib().glm53_grouped_moe_workspace_bytes(T, top_k, bank.expert_count, H, I, Is)
    ws = wsp.get(dev, "grouped", nbytes)
    if status is None:
        status = wsp.get(dev, "status", 4)
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    if T:
        N.check(
            N.lib().glm53_grouped_moe(
                flat.data_ptr(), T, H, idx.data_ptr(), sc.data_ptr(), top_k,
                bank.gate_up_weight.data_ptr(), bank.gate_up_scale_inv.data_ptr(), bank.down_weight.data_ptr(),
                bank.down_scale_inv.data_ptr(), bank.expert_count, I, N.ptr(sg_w), N.ptr(sg_s), N.ptr(su_w),
                N.ptr(su_s), N.ptr(sd_w), N.ptr(sd_s), Is, float(limit), out.data_ptr(), ws.data_ptr(),
                ws.numel(), status.data_ptr(), flags, N.stream(dev),
            ),
            "glm53_grouped_moe",
        )
    if _SYNC_STATUS:
        check_status(status)
    return out.reshape(x.shape)


class SortedGroupedFP8MoE(PackedFP8MoE):
    """Prefill-only grouped path with the existing packed/decode fallback."""

    def __init__(self, bank, config, gate, shared_experts, *, min_routes: int = GROUPED_MIN_ROUTES):
        super().__init__(bank, config, gate, shared_experts)
        self.min_routes = int(min_routes)

    def grouped_from_routes(self, x, indices, scores):
        shared = shared_fp8_tensors(self.shared_experts)
        sw = self.status_word(x.device)
        sw.raise_pending()
        result = grouped_moe(x, indices, scores, self.bank, shared, limit=self.config.swiglu_limit,
                             workspace=self._workspace, status=sw.word)
        if shared is None and self.shared_experts is not None:
            result = result + self.shared_experts(x)
        sw.publish()
        return result

    def forward(self, x):
        routes = x.reshape(-1, x.shape[-1]).shape[0] * self.config.num_experts_per_tok
        if routes < self.min_routes:
            return super().forward(x)
        indices, scores = self.gate(x)
        return self.grouped_from_routes(x, indices, scores)
