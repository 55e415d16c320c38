"""Sparse-attention output projection with the post-attention hc expand, on B200.

Counterpart of ``NativePrefillDSAOutputPlan``
(native_execution/native_prefill_dsa_output_plan.h:16-73): the head-major
attention result ``[heads, rows, dim]`` is laid out row-major
(``glm53_head_major_to_rows``), multiplied by the block-128 E4M3 ``o_proj``
(``block_fp8_linear``: the tcgen05 GEMM above 16 rows) and, in
``execute_hc``, expanded into the 4-branch residual state (``hc_expand``).
The reference fixes the geometry at 64 heads x 256 rows x 256 values and
o_proj [4096, 16384]; here it follows the inputs.
"""

from __future__ import annotations

import torch

from . import _native as N
from .fp8 import block_fp8_linear
from .hyper_connection import hc_expand


def head_major_to_rows(head_major: torch.Tensor) -> torch.Tensor:
    """BF16 [heads, rows, dim] -> BF16 [rows, heads * dim] (a copy)."""
    dev = N.require_cuda(head_major)
    if head_major.dtype != torch.bfloat16 or head_major.dim() != 3:
        raise ValueError(f"head_major must be BF16 [heads, rows, dim], got {tuple(head_major.shape)} "
                         f"{head_major.dtype}")
    heads, rows, dim = head_major.shape
    src = head_major.contiguous()
    out = torch.empty((rows, heads * dim), dtype=torch.bfloat16, device=dev)
    N.check(N.lib().glm53_head_major_to_rows(src.data_ptr(), heads, rows, dim, out.data_ptr(), N.stream(dev)),
            "glm53_head_major_to_rows")
    return out


class DSAOutputProjection:
    """``execute(head_major, weight, scale_inv)`` -> BF16 [rows, hidden];
    ``execute_hc(head_major, weight, scale_inv, residual, post, comb)`` ->
    BF16 [rows, 4, hidden] (native_prefill_dsa_output_plan.h:22-30)."""

    def __init__(self) -> None:
        self.execution_count = 0

    def execute(self, head_major: torch.Tensor, weight: torch.Tensor, scale_inv: torch.Tensor) -> torch.Tensor:
        heads, rows, dim = head_major.shape if head_major.dim() == 3 else (None, None, None)
        if heads is None:
            raise ValueError(f"head_major must be [heads, rows, dim], got {tuple(head_major.shape)}")
        if weight.dim() != 2 or weight.shape[1] != heads * dim:
            raise ValueError(f"o_proj weight {tuple(weight.shape)} does not take {heads} x {dim} inputs")
        out = block_fp8_linear(head_major_to_rows(head_major), weight, scale_inv)
        self.execution_count += 1
        return out

    def execute_hc(self, head_major: torch.Tensor, weight: torch.Tensor, scale_inv: torch.Tensor,
                   residual: torch.Tensor, post: torch.Tensor, comb: torch.Tensor) -> torch.Tensor:
        return hc_expand(self.execute(head_major, weight, scale_inv), residual, post, comb)
