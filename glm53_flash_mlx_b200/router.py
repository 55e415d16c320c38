"""FP32 MoE router on B200.

Counterpart of ``Float32Gate`` (glm53_flash_mlx/patch.py:131-142), which
computes FP32 logits and calls mlx-vlm's ``group_expert_select`` (mlx-vlm
0.6.17 @ e82d557, a third-party function the reference does not vendor).
The selection is restated in ``csrc/router.cu``; its slot order is descending
biased score with ties to the lower expert id (the reference's argpartition
leaves slot order unspecified).
"""

from __future__ import annotations

import torch
from torch import nn

from . import _native as N


def router_topk(
    x: torch.Tensor,
    weight: torch.Tensor,
    e_score_correction_bias: torch.Tensor,
    *,
    top_k: int,
    n_group: int = 1,
    topk_group: int = 1,
    routed_scaling_factor: float = 1.0,
    norm_topk_prob: bool = True,
    workspace: N.Workspace | None = None,
    return_logits: bool = False,
):
    """Return (indices int32 [..., top_k], scores float32 [..., top_k])
    (and FP32 logits [..., E] when ``return_logits``)."""
    N.require_cuda(x, weight, e_score_correction_bias)
    if x.dtype != torch.bfloat16:
        raise ValueError(f"router input must be BF16, got {x.dtype}")
    if weight.dtype != torch.float32 or weight.dim() != 2:
        raise ValueError("router weight must be a 2-D float32 [experts, hidden] tensor")
    E, H = weight.shape
    if x.shape[-1] != H:
        raise ValueError(f"input width {x.shape[-1]} != router width {H}")
    if e_score_correction_bias.shape != (E,) or e_score_correction_bias.dtype != torch.float32:
        raise ValueError("e_score_correction_bias must be float32 [experts]")
    flat = x.reshape(-1, H).contiguous()
    T = flat.shape[0]
    dev = x.device
    idx = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    sc = torch.empty((T, top_k), dtype=torch.float32, device=dev)
    logits = torch.empty((T, E), dtype=torch.float32, device=dev) if return_logits else None
    ws_bytes = N.lib().glm53_router_workspace_bytes(T, E)
    ws = (workspace or N.Workspace()).get(dev, "router", ws_bytes)
    if T:
        N.check(
            N.lib().glm53_router_topk(
                flat.data_ptr(), T, H, weight.contiguous().data_ptr(), E,
                e_score_correction_bias.contiguous().data_ptr(), int(top_k), int(n_group), int(topk_group),
                int(bool(norm_topk_prob)), float(routed_scaling_factor), idx.data_ptr(), sc.data_ptr(),
                N.ptr(logits), ws.data_ptr(), ws.numel(), N.stream(dev),
            ),
            "glm53_router_topk",
        )
    shape = x.shape[:-1]
    out = (idx.reshape(*shape, top_k), sc.reshape(*shape, top_k))
    if return_logits:
        return (*out, logits.reshape(*shape, E))
    return out


class Float32Gate(nn.Module):
    """MoE gate with FP32 logits: sigmoid, correction bias, (group) top-k,
    normalisation and routed scaling (glm53_flash_mlx/patch.py:131-142)."""

    def __init__(self, config, device=None):
        super().__init__()
        E = config.n_routed_experts
        H = config.hidden_size
        self.top_k = int(config.num_experts_per_tok)
        self.n_group = int(getattr(config, "n_group", 1) or 1)
        self.topk_group = int(getattr(config, "topk_group", 1) or 1)
        self.routed_scaling_factor = float(getattr(config, "routed_scaling_factor", 1.0))
        self.norm_topk_prob = bool(getattr(config, "norm_topk_prob", True))
        self.register_buffer("weight", torch.zeros((E, H), dtype=torch.float32, device=device))
        self.register_buffer("e_score_correction_bias", torch.zeros((E,), dtype=torch.float32, device=device))
        self._workspace = N.Workspace()

    def forward(self, x):
        return router_topk(
            x, self.weight, self.e_score_correction_bias, top_k=self.top_k, n_group=self.n_group,
            topk_group=self.topk_group, routed_scaling_factor=self.routed_scaling_factor,
            norm_topk_prob=self.norm_topk_prob, workspace=self._workspace,
        )
