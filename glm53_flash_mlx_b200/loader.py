"""Layer-by-layer installers of the packed MoE backends.

Counterpart of glm53_flash_mlx/loader.py:167-254 (``install_packed_moe``,
``install_packed_grouped_moe``, ``install_packed_decode_moe``): every
``DirectFP8MoE`` layer is packed into a ``PackedFP8ExpertBank`` one layer at a
time, the layer's module is swapped, the old per-expert modules are released,
and a per-layer memory report is returned.  Installing twice converts nothing.
Reading a block-FP8 safetensors checkpoint straight into packed banks (no
DirectFP8MoE stage) is ``checkpoint.py``.
"""

from __future__ import annotations

import gc
import logging

import torch

from .fp8 import DirectFP8MoE
from .grouped_fp8 import SortedGroupedFP8MoE
from .packed import PackedFP8ExpertBank, PackedFP8MoE


def _memory() -> int:
    return torch.cuda.memory_allocated() if torch.cuda.is_available() else 0


def _peak() -> int:
    return torch.cuda.max_memory_allocated() if torch.cuda.is_available() else 0


def install_packed_moe(model, *, grouped: bool) -> dict:
    """Pack routed experts layerwise and select the requested execution policy."""
    logger = logging.getLogger(__name__)
    module_type = SortedGroupedFP8MoE if grouped else PackedFP8MoE
    backend = "packed-grouped" if grouped else "packed-decode"
    converted = []
    layers = model.language_model.model.layers
    for layer_id, layer in enumerate(layers):
        direct = layer.mlp
        if isinstance(direct, module_type) and (grouped or not isinstance(direct, SortedGroupedFP8MoE)):
            continue
        if isinstance(direct, PackedFP8MoE):
            raise ValueError(f"cannot convert existing {type(direct).__name__} to {backend} in place")
        if not isinstance(direct, DirectFP8MoE):
            continue
        active_before = _memory()
        bank = PackedFP8ExpertBank.pack(direct.experts)
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        active_materialized = _memory()
        layer.mlp = module_type(bank, direct.config, direct.gate, direct.shared_experts)
        layer.compile_ffn = False
        old_expert_count = len(direct.experts)
        del direct
        gc.collect()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
            torch.cuda.synchronize()
        active_after_clear = _memory()
        converted.append(
            {
                "layer": layer_id,
                "old_expert_count": old_expert_count,
                "bank_bytes": bank.nbytes,
                "active_before_bytes": active_before,
                "active_materialized_bytes": active_materialized,
                "active_after_clear_bytes": active_after_clear,
                "peak_bytes": _peak(),
                "old_expert_modules_detached": not hasattr(layer.mlp, "experts"),
            }
        )
        logger.info("%s MoE layer=%d active=%.3f GB peak=%.3f GB", backend, layer_id,
                    active_after_clear / 1e9, _peak() / 1e9)
    remaining_direct = [
        layer_id
        for layer_id, layer in enumerate(layers)
        if isinstance(layer.mlp, DirectFP8MoE) and not isinstance(layer.mlp, PackedFP8MoE)
    ]
    report = {
        "converted_layers": [row["layer"] for row in converted],
        "converted_count": len(converted),
        "remaining_direct_layers": remaining_direct,
        "all_old_expert_modules_detached": all(row["old_expert_modules_detached"] for row in converted),
        "layers": converted,
    }
    report["backend"] = backend
    report["grouped_enabled"] = grouped
    model._glm53_moe_backend = backend
    setattr(model, f"_glm53_{backend.replace('-', '_')}_report", report)
    return report


def install_packed_grouped_moe(model) -> dict:
    """Install the grouped-prefill policy."""
    return install_packed_moe(model, grouped=True)


def install_packed_decode_moe(model) -> dict:
    """Install packed selected decode while retaining Direct prefill semantics."""
    return install_packed_moe(model, grouped=False)
