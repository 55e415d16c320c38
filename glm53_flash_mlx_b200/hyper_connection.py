"""FFN boundary of a GLM-5.3 layer around the MoE, on B200.

The reference runs, per layer (scripts/trace_grouped_fp8_route_amplification.py:
178-214; scripts/profile_native_prefill_ffn_entry_seam.py:79-87):

    collapsed, post, comb = layer.ffn_hc(state)          # mHC collapse
    normalized = layer.post_attention_layernorm(collapsed)
    moe = layer.mlp(normalized)                          # router + MoE
    state = hc_expand(moe, state, post, comb)

``layer.ffn_hc`` is mlx-vlm's deepseek_v4 hyper-connection module (mlx-vlm
0.6.17 @ e82d557, not vendored by the reference).  ``HyperConnection`` here
restates the published mHC collapse (DeepSeek-V4 ``hc_pre`` with
``hc_split_sinkhorn``) with the parameter dtypes the reference loads: ``fn``
BF16 (cast with the model), ``scale`` and ``base`` FP32
(glm53_flash_mlx/patch.py:296-318).  ``hc_expand`` restates the reference's
own kernel ``glm53_native_prefill_post_attention_hc_expand``
(native_execution/native_indexer_plan.metal:2362-2389).  ``RMSNorm`` is MLX's
fast RMSNorm.  All three run the sm_100a kernels of ``csrc/hc.cu``; there is
no other path.
"""

from __future__ import annotations

import torch
from torch import nn

from . import _native as N

HC_BRANCHES = 4


def _bf16_rows(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be BF16, got {t.dtype}")
    return t.contiguous()


class RMSNorm(nn.Module):
    """``post_attention_layernorm``: out = BF16(w * BF16(x * rsqrt(mean(x^2) + eps)))
    over the last axis (MLX ``fast.rms_norm`` rounding)."""

    def __init__(self, hidden_size: int, eps: float = 1e-6, device=None):
        super().__init__()
        self.eps = float(eps)
        self.register_buffer("weight", torch.ones((hidden_size,), dtype=torch.bfloat16, device=device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    dev = N.require_cuda(x, weight)
    x = _bf16_rows(x, "rms_norm input")
    H = x.shape[-1]
    if weight.shape != (H,):
        raise ValueError(f"rms_norm weight shape {tuple(weight.shape)} != ({H},)")
    weight = _bf16_rows(weight, "rms_norm weight")
    out = torch.empty_like(x)
    T = x.numel() // H if H else 0
    N.check(N.lib().glm53_rms_norm(x.data_ptr(), T, H, weight.data_ptr(), float(eps), out.data_ptr(),
                                   N.stream(dev)), "glm53_rms_norm")
    return out


class HyperConnection(nn.Module):
    """mHC collapse of the 4-branch residual state (``layer.ffn_hc``).

    ``hc(state)`` with state BF16 [..., 4, H] returns
    ``(collapsed BF16 [..., H], post FP32 [..., 4], comb FP32 [..., 4, 4])``;
    ``hc.collapse_norm(state, norm)`` also applies ``norm`` (an ``RMSNorm``)
    in the same pass and returns ``(collapsed, normalized, post, comb)``.
    """

    def __init__(self, hidden_size: int, hc_mult: int = HC_BRANCHES, *, sinkhorn_iters: int = 20,
                 eps: float = 1e-6, norm_eps: float = 1e-6, device=None):
        super().__init__()
        if hc_mult != HC_BRANCHES:
            raise ValueError(f"hc_mult {hc_mult}: the kernels are built for {HC_BRANCHES} branches")
        self.hidden_size = int(hidden_size)
        self.hc_mult = int(hc_mult)
        self.sinkhorn_iters = int(sinkhorn_iters)
        self.eps = float(eps)
        self.norm_eps = float(norm_eps)
        mix = (2 + hc_mult) * hc_mult
        self.register_buffer("fn", torch.zeros((mix, hc_mult * hidden_size), dtype=torch.bfloat16, device=device))
        self.register_buffer("scale", torch.ones((3,), dtype=torch.float32, device=device))
        self.register_buffer("base", torch.zeros((mix,), dtype=torch.float32, device=device))
        self._workspace = N.Workspace()

    def forward(self, state: torch.Tensor):
        collapsed, _, post, comb = self._run(state, None)
        return collapsed, post, comb

    def collapse_norm(self, state: torch.Tensor, norm: RMSNorm):
        return self._run(state, norm)

    def _run(self, state: torch.Tensor, norm: RMSNorm | None):
        dev = N.require_cuda(state, self.fn, self.scale, self.base, None if norm is None else norm.weight)
        state = _bf16_rows(state, "hc state")
        n, H = self.hc_mult, self.hidden_size
        if state.dim() < 2 or tuple(state.shape[-2:]) != (n, H):
            raise ValueError(f"hc state shape {tuple(state.shape)} must end in ({n}, {H})")
        mix = (2 + n) * n
        if self.fn.shape != (mix, n * H) or self.fn.dtype != torch.bfloat16:
            raise ValueError(f"hc fn must be BF16 [{mix}, {n * H}]")
        if self.scale.shape != (3,) or self.scale.dtype != torch.float32:
            raise ValueError("hc scale must be float32 [3]")
        if self.base.shape != (mix,) or self.base.dtype != torch.float32:
            raise ValueError(f"hc base must be float32 [{mix}]")
        lead = state.shape[:-2]
        T = state.numel() // (n * H)
        collapsed = torch.empty((*lead, H), dtype=torch.bfloat16, device=dev)
        post = torch.empty((*lead, n), dtype=torch.float32, device=dev)
        comb = torch.empty((*lead, n, n), dtype=torch.float32, device=dev)
        normalized = None
        w = None
        rms_eps = 0.0
        if norm is not None:
            if norm.weight.shape != (H,):
                raise ValueError(f"norm weight shape {tuple(norm.weight.shape)} != ({H},)")
            w = _bf16_rows(norm.weight, "norm weight")
            rms_eps = norm.eps
            normalized = torch.empty_like(collapsed)
        ws_bytes = N.lib().glm53_hc_collapse_workspace_bytes(T, H)
        if T and ws_bytes == 0:
            raise ValueError(f"hidden size {H} is not supported by the hc kernels")
        ws = self._workspace.get(dev, "hc", ws_bytes)
        N.check(
            N.lib().glm53_hc_collapse_norm(
                state.data_ptr(), T, H, n, self.fn.contiguous().data_ptr(), self.scale.contiguous().data_ptr(),
                self.base.contiguous().data_ptr(), self.sinkhorn_iters, self.eps, self.norm_eps, N.ptr(w),
                float(rms_eps), collapsed.data_ptr(), N.ptr(normalized), post.data_ptr(), comb.data_ptr(),
                ws.data_ptr(), ws.numel(), N.stream(dev),
            ),
            "glm53_hc_collapse_norm",
        )
        return collapsed, normalized, post, comb


def hc_expand(x: torch.Tensor, residual: torch.Tensor, post: torch.Tensor, comb: torch.Tensor) -> torch.Tensor:
    """Expand the block output ``x`` [..., H] into the 4-branch state:
    out[..., b, :] = BF16(post[..., b] * x + sum_s comb[..., s, b] * residual[..., s, :])
    (FMA chain over s, then the rounded product added;
    native_execution/native_indexer_plan.metal:2362-2389)."""
    dev = N.require_cuda(x, residual, post, comb)
    x = _bf16_rows(x, "hc_expand input")
    residual = _bf16_rows(residual, "hc_expand residual")
    H = x.shape[-1]
    n = HC_BRANCHES
    lead = x.shape[:-1]
    if tuple(residual.shape) != (*lead, n, H):
        raise ValueError(f"residual shape {tuple(residual.shape)} != {(*lead, n, H)}")
    if post.dtype != torch.float32 or tuple(post.shape) != (*lead, n):
        raise ValueError(f"post must be float32 {(*lead, n)}")
    if comb.dtype != torch.float32 or tuple(comb.shape) != (*lead, n, n):
        raise ValueError(f"comb must be float32 {(*lead, n, n)}")
    post = post.contiguous()
    comb = comb.contiguous()
    out = torch.empty_like(residual)
    T = x.numel() // H if H else 0
    N.check(N.lib().glm53_hc_expand(x.data_ptr(), residual.data_ptr(), post.data_ptr(), comb.data_ptr(), T, H, n,
                                    out.data_ptr(), N.stream(dev)), "glm53_hc_expand")
    return out


class FFNBoundary(nn.Module):
    """The FFN half of a layer with the B200 MoE in the middle:
    ``state -> ffn_hc -> post_attention_layernorm -> mlp -> hc_expand``.
    ``mlp`` is any callable on BF16 [..., H] rows (``PackedFP8MoE``,
    ``SortedGroupedFP8MoE``)."""

    def __init__(self, ffn_hc: HyperConnection, post_attention_layernorm: RMSNorm, mlp):
        super().__init__()
        self.ffn_hc = ffn_hc
        self.post_attention_layernorm = post_attention_layernorm
        self.mlp = mlp

    def forward(self, state: torch.Tensor) -> torch.Tensor:
        _, normalized, post, comb = self.ffn_hc.collapse_norm(state, self.post_attention_layernorm)
        fused = getattr(self.mlp, "forward_expand", None)
        if fused is not None:  # a packed MoE: one decode token expands inside its final reduce
            return fused(normalized, state, post, comb)
        return hc_expand(self.mlp(normalized), state, post, comb)
