"""Direct E4M3 block-FP8 operators on B200 (sm_100a).

Counterpart of glm53_flash_mlx/fp8.py: ``block_fp8_linear`` (fp8.py:254-299),
``BlockFP8Linear`` (fp8.py:302-326), ``DirectFP8Expert`` (fp8.py:329-340) and
``DirectFP8MoE`` (fp8.py:343-400) with the same argument meaning, the same
fail-closed checks and the same exceptions.  Weights stay uint8 E4M3 codes with
FP32 ``weight_scale_inv`` on the 128x128 grid; they are decoded only in
registers or shared memory inside the CUDA kernels.
"""

from __future__ import annotations

import torch
from torch import nn

from . import _native as N
from .abi import KERNEL_ABI_VERSION  # noqa: F401  (re-exported like the reference)

BLOCK_SIZE = 128
THREADS = 256
DECODE_TOP_K = 8
PREFILL_TILE_ROWS = 8


def _scale_shape(out_features: int, in_features: int) -> tuple[int, int]:
    return ((out_features + BLOCK_SIZE - 1) // BLOCK_SIZE, (in_features + BLOCK_SIZE - 1) // BLOCK_SIZE)


# Rows handled by the bandwidth GEMV (kGemvMaxRows in csrc/kernels.cuh); more
# rows go to the tcgen05 GEMM through glm53_fp8_linear_ws.
_GEMV_MAX_ROWS = 16
_LINEAR_WS = N.Workspace()


def block_fp8_linear(x: torch.Tensor, weight: torch.Tensor, scale_inv: torch.Tensor, *,
                     e4m3_finite: bool = False) -> torch.Tensor:
    """Compute ``x @ dequant(weight, scale_inv).T`` without expanding weight.

    x: BF16 [..., in] on a CUDA device; weight: uint8 E4M3 [out, in];
    scale_inv: float32 [ceil(out/128), ceil(in/128)].  Returns BF16 [..., out].
    ``e4m3_finite=True`` certifies that ``weight`` holds no code 0x7F/0xFF
    (see ``_native.e4m3_finite``) and enables the hardware E4M3 decode.
    """
    if not (isinstance(x, torch.Tensor) and x.is_cuda):
        raise RuntimeError("direct GLM-5.3 FP8 execution requires the CUDA backend")
    N.lib()
    if weight.dtype != torch.uint8 or weight.dim() != 2:
        raise ValueError(f"expected 2-D uint8 E4M3 weight, got {tuple(weight.shape)} {weight.dtype}")
    if scale_inv.dtype != torch.float32 or scale_inv.dim() != 2:
        raise ValueError("weight_scale_inv must be a 2-D float32 block table")
    out_features, in_features = weight.shape
    if x.shape[-1] != in_features:
        raise ValueError(f"input width {x.shape[-1]} != weight width {in_features}")
    expected = _scale_shape(out_features, in_features)
    if tuple(scale_inv.shape) != expected:
        raise ValueError(f"scale shape {tuple(scale_inv.shape)} != block128 shape {expected}")
    if x.dtype != torch.bfloat16:
        raise ValueError(f"block_fp8_linear computes on BF16 activations, got {x.dtype}")
    N.require_cuda(x, weight, scale_inv)
    original_shape = x.shape
    flat = x.reshape(-1, in_features).contiguous()
    weight = weight.contiguous()
    scale_inv = scale_inv.contiguous()
    out = torch.empty((flat.shape[0], out_features), dtype=x.dtype, device=x.device)
    M = flat.shape[0]
    flags = N.FLAG_E4M3_FINITE if e4m3_finite else 0
    if M > _GEMV_MAX_ROWS:
        # tensor-core GEMM: scratch for the FP16 activation rows, one per device and stream
        stream = N.stream(x.device)
        ws = _LINEAR_WS.get(x.device, f"rows:{stream}",
                            N.lib().glm53_fp8_linear_splitk_workspace_bytes(M, in_features, out_features))
        status = _LINEAR_WS.get(x.device, "status", 4)
        N.check(
            N.lib().glm53_fp8_linear_ws(
                flat.data_ptr(), M, in_features, weight.data_ptr(), out_features, scale_inv.data_ptr(),
                out.data_ptr(), ws.data_ptr(), ws.numel(), status.data_ptr(), flags, stream,
            ),
            "glm53_fp8_linear_ws",
        )
    elif M:
        N.check(
            N.lib().glm53_fp8_linear(
                flat.data_ptr(), M, in_features, weight.data_ptr(), out_features,
                scale_inv.data_ptr(), out.data_ptr(), flags, N.stream(x.device),
            ),
            "glm53_fp8_linear",
        )
    return out.reshape(*original_shape[:-1], out_features)


class BlockFP8Linear(nn.Module):
    """``nn.Linear`` ABI backed by canonical block-128 E4M3 tensors."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, device=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("weight", torch.zeros((out_features, in_features), dtype=torch.uint8, device=device))
        self.register_buffer(
            "weight_scale_inv",
            torch.ones(_scale_shape(out_features, in_features), dtype=torch.float32, device=device),
        )
        if bias:
            self.register_buffer("bias", torch.zeros((out_features,), dtype=torch.float32, device=device))
        else:
            self.bias = None

    @classmethod
    def from_linear(cls, linear: nn.Module) -> "BlockFP8Linear":
        out_features, in_features = linear.weight.shape
        return cls(in_features, out_features, bias=getattr(linear, "bias", None) is not None,
                   device=linear.weight.device)

    def forward(self, x):
        finite = self.weight.is_cuda and N.e4m3_finite(self.weight)
        y = block_fp8_linear(x, self.weight, self.weight_scale_inv, e4m3_finite=finite)
        return (y + self.bias).to(y.dtype) if self.bias is not None else y


def swiglu_pair(gate: torch.Tensor, up: torch.Tensor, limit: float) -> torch.Tensor:
    """silu(min(gate, L)) * clip(up, -L, L) on BF16 tensors with the reference's
    per-op BF16 rounding (the MLX ops of glm53_flash_mlx/fp8.py:337-340)."""
    inter = gate.shape[-1]
    fused = torch.cat([gate.reshape(-1, inter), up.reshape(-1, inter)], dim=-1).contiguous()
    hidden = torch.empty((fused.shape[0], inter), dtype=torch.bfloat16, device=gate.device)
    if fused.shape[0]:
        N.check(
            N.lib().glm53_activate_gate_up(fused.data_ptr(), fused.shape[0], inter, float(limit),
                                           hidden.data_ptr(), N.stream(gate.device)),
            "glm53_activate_gate_up",
        )
    return hidden.reshape(gate.shape)


class DirectFP8Expert(nn.Module):
    def __init__(self, hidden_size: int, intermediate_size: int, limit: float, device=None):
        super().__init__()
        self.gate_proj = BlockFP8Linear(hidden_size, intermediate_size, device=device)
        self.up_proj = BlockFP8Linear(hidden_size, intermediate_size, device=device)
        self.down_proj = BlockFP8Linear(intermediate_size, hidden_size, device=device)
        self.limit = float(limit)

    def forward(self, x):
        return self.down_proj(swiglu_pair(self.gate_proj(x), self.up_proj(x), self.limit))


class DirectFP8MoE(nn.Module):
    """Bucketed top-k MoE over separate canonical expert tensors
    (glm53_flash_mlx/fp8.py:343-400): selected top-8 decode for one row,
    ascending-expert BF16 scatter-add for more rows, plus the shared expert."""

    def __init__(self, config, gate, shared_experts, device=None):
        super().__init__()
        self.config = config
        self.gate = gate
        self.shared_experts = shared_experts
        self.experts = nn.ModuleList(
            [
                DirectFP8Expert(config.hidden_size, config.moe_intermediate_size, config.swiglu_limit, device=device)
                for _ in range(config.n_routed_experts)
            ]
        )

    def forward(self, x):
        indices, scores = self.gate(x)
        return self._forward_routes(x, indices, scores)

    def _forward_routes(self, x, indices, scores):
        # Routing is a phase boundary: one readback gives the host the expert
        # buckets (glm53_flash_mlx/fp8.py:366-369).
        routes = indices.reshape(-1, self.config.num_experts_per_tok).to(torch.int64).cpu()
        flat_x = x.reshape(-1, x.shape[-1])
        flat_scores = scores.reshape(-1, self.config.num_experts_per_tok)
        limit = self.config.swiglu_limit
        if flat_x.shape[0] == 1 and routes.shape == (1, DECODE_TOP_K):
            selected = [self._expert(int(e)) for e in routes[0].tolist()]
            return selected_decode_moe(flat_x[0], flat_scores[0], selected, self.shared_experts,
                                       limit=limit, workspace=self._decode_workspace()).reshape(x.shape)
        result = torch.zeros_like(flat_x)
        for expert_id in torch.unique(routes).tolist():
            rows_cpu, slots_cpu = torch.nonzero(routes == expert_id, as_tuple=True)
            rows = rows_cpu.to(flat_x.device)
            slots = slots_cpu.to(flat_x.device)
            expert_out = self._expert(int(expert_id))(flat_x[rows])
            route_weight = flat_scores[rows, slots][..., None]
            weighted = (expert_out.float() * route_weight.float()).to(flat_x.dtype)
            result.index_add_(0, rows, weighted)
        result = result.reshape(x.shape)
        if self.shared_experts is not None:
            result = result + self.shared_experts(x)
        return result

    def _expert(self, expert_id: int):
        return self.experts[expert_id]

    def _decode_workspace(self):
        ws = self.__dict__.get("_ws")
        if ws is None:
            ws = self.__dict__["_ws"] = N.Workspace()
        return ws


def _shared_parts(shared):
    from .packed import shared_fp8_tensors

    return shared_fp8_tensors(shared)


def selected_decode_moe(x: torch.Tensor, scores: torch.Tensor, experts, shared, *, limit: float,
                        workspace: N.Workspace | None = None) -> torch.Tensor:
    """Top-k decode over separately allocated experts (the Direct module's
    selected top-8 path, glm53_flash_mlx/fp8.py:372-383) with the packed
    decode kernels: bit-identical to PackedFP8MoE over the same tensors."""
    import ctypes

    dev = N.require_cuda(x, scores)
    H = x.numel()
    top_k = len(experts)
    I = experts[0].gate_proj.weight.shape[0]
    x = x.reshape(H).contiguous()
    sc = scores.reshape(-1).to(torch.float32).contiguous()
    tensors = []
    tables = {name: (ctypes.c_void_p * top_k)() for name in ("gw", "gs", "uw", "us", "dw", "ds")}
    for j, e in enumerate(experts):
        parts = (e.gate_proj.weight, e.gate_proj.weight_scale_inv, e.up_proj.weight, e.up_proj.weight_scale_inv,
                 e.down_proj.weight, e.down_proj.weight_scale_inv)
        parts = tuple(t.contiguous() for t in parts)
        tensors.append(parts)
        for name, t in zip(("gw", "gs", "uw", "us", "dw", "ds"), parts):
            tables[name][j] = t.data_ptr()
    sh = _shared_parts(shared)
    Is = sh[0].shape[0] if sh is not None else 0
    weights = [t for p in tensors for t in (p[0], p[2], p[4])] + ([sh[0], sh[2], sh[4]] if sh else [])
    flags = N.decode_flags(*weights)
    wsp = workspace or N.Workspace()
    ws = wsp.get(dev, "decode", N.lib().glm53_packed_decode_workspace_bytes(top_k, H, I, Is))
    status = wsp.get(dev, "status", 4)
    out = torch.empty(H, dtype=torch.bfloat16, device=dev)
    p = (lambda i: None if sh is None else sh[i].data_ptr())
    N.check(
        N.lib().glm53_selected_decode_moe(
            x.data_ptr(), H, sc.data_ptr(), top_k, tables["gw"], tables["gs"], tables["uw"], tables["us"],
            tables["dw"], tables["ds"], I, p(0), p(1), p(2), p(3), p(4), p(5), Is, float(limit), out.data_ptr(),
            ws.data_ptr(), ws.numel(), status.data_ptr(), flags, N.stream(dev),
        ),
        "glm53_selected_decode_moe",
    )
    if sh is None and shared is not None:
        out = (out.reshape(1, H) + shared(x.reshape(1, H))).reshape(H)
    return out
