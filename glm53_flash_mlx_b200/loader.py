"""Installers that move a model's Direct FP8 MoE layers onto packed banks.

The drop-in contract is that of glm53_flash_mlx/loader.py:167-254
(``install_packed_moe``, ``install_packed_grouped_moe``,
``install_packed_decode_moe``): each ``DirectFP8MoE`` layer is replaced by a
packed module over a ``PackedFP8ExpertBank``, one layer at a time so that at
most one layer's experts exist twice; the replaced per-expert modules are
released; a second install converts nothing; the report carries the keys the
reference's callers read (``converted_layers``, ``converted_count``,
``remaining_direct_layers``, ``all_old_expert_modules_detached``, ``layers``,
``backend``, ``grouped_enabled``) and is attached to the model.

Here the conversion is a policy (which packed module, which report name)
applied to every MoE layer by one routine, and each layer's outcome is a
typed record with its own device-memory readings.  Loading a block-FP8
safetensors checkpoint directly into packed banks, without a Direct stage, is
``checkpoint.py``.
"""

from __future__ import annotations

import gc
import logging
from dataclasses import dataclass

import torch

from .fp8 import DirectFP8MoE
from .grouped_fp8 import SortedGroupedFP8MoE
from .packed import PackedFP8ExpertBank, PackedFP8MoE

_log = logging.getLogger(__name__)


@dataclass(frozen=True)
class InstallPolicy:
    """What a layer becomes: the packed module type and the report's name."""

    backend: str
    module_type: type
    grouped: bool

    def installed(self, mlp) -> bool:
        """True when `mlp` already is this policy's module (nothing to do)."""
        if self.grouped:
            return isinstance(mlp, SortedGroupedFP8MoE)
        return isinstance(mlp, PackedFP8MoE) and not isinstance(mlp, SortedGroupedFP8MoE)


PACKED_DECODE = InstallPolicy("packed-decode", PackedFP8MoE, grouped=False)
PACKED_GROUPED = InstallPolicy("packed-grouped", SortedGroupedFP8MoE, grouped=True)


class _DeviceMemory:
    """Allocated-bytes readings of the current CUDA device (zeros without one)."""

    def __init__(self) -> None:
        self.cuda = torch.cuda.is_available()

    def active(self) -> int:
        return torch.cuda.memory_allocated() if self.cuda else 0

    def peak(self) -> int:
        return torch.cuda.max_memory_allocated() if self.cuda else 0

    def drain(self) -> None:
        """Finish queued work so the next reading sees it."""
        if self.cuda:
            torch.cuda.synchronize()

    def release(self) -> None:
        """Return freed blocks to the device, then finish queued work."""
        gc.collect()
        if self.cuda:
            torch.cuda.empty_cache()
            torch.cuda.synchronize()


@dataclass
class LayerConversion:
    """One converted layer and the device memory around its conversion."""

    layer: int
    old_expert_count: int
    bank_bytes: int
    before: int
    materialized: int
    after_release: int
    peak: int
    detached: bool

    def row(self) -> dict:
        return {
            "layer": self.layer,
            "old_expert_count": self.old_expert_count,
            "bank_bytes": self.bank_bytes,
            "active_before_bytes": self.before,
            "active_materialized_bytes": self.materialized,
            "active_after_clear_bytes": self.after_release,
            "peak_bytes": self.peak,
            "old_expert_modules_detached": self.detached,
        }


def _decoder_layers(model):
    return model.language_model.model.layers


def _is_direct_only(mlp) -> bool:
    return isinstance(mlp, DirectFP8MoE) and not isinstance(mlp, PackedFP8MoE)


def _convert_layer(index: int, layer, policy: InstallPolicy, memory: _DeviceMemory) -> LayerConversion | None:
    mlp = layer.mlp
    if policy.installed(mlp):
        return None
    if isinstance(mlp, PackedFP8MoE):
        raise ValueError(f"cannot convert existing {type(mlp).__name__} to {policy.backend} in place")
    if not isinstance(mlp, DirectFP8MoE):
        return None
    before = memory.active()
    bank = PackedFP8ExpertBank.pack(mlp.experts)
    memory.drain()
    materialized = memory.active()
    replaced_experts = len(mlp.experts)
    layer.mlp = policy.module_type(bank, mlp.config, mlp.gate, mlp.shared_experts)
    layer.compile_ffn = False
    del mlp  # the last reference to the per-expert modules
    memory.release()
    record = LayerConversion(layer=index, old_expert_count=replaced_experts, bank_bytes=bank.nbytes, before=before,
                             materialized=materialized, after_release=memory.active(), peak=memory.peak(),
                             detached=not hasattr(layer.mlp, "experts"))
    _log.info("layer %d -> %s: bank %.3f GB, device %.3f GB (peak %.3f GB)", index, policy.backend,
              record.bank_bytes / 1e9, record.after_release / 1e9, record.peak / 1e9)
    return record


def _install(model, policy: InstallPolicy) -> dict:
    memory = _DeviceMemory()
    layers = _decoder_layers(model)
    records = [r for r in (_convert_layer(i, layer, policy, memory) for i, layer in enumerate(layers)) if r]
    report = {
        "converted_layers": [r.layer for r in records],
        "converted_count": len(records),
        "remaining_direct_layers": [i for i, layer in enumerate(layers) if _is_direct_only(layer.mlp)],
        "all_old_expert_modules_detached": all(r.detached for r in records),
        "layers": [r.row() for r in records],
        "backend": policy.backend,
        "grouped_enabled": policy.grouped,
    }
    model._glm53_moe_backend = policy.backend
    setattr(model, "_glm53_" + policy.backend.replace("-", "_") + "_report", report)
    return report


def install_packed_moe(model, *, grouped: bool) -> dict:
    """Pack every Direct MoE layer's experts (layer by layer) and install the
    grouped-prefill module (``grouped=True``) or the packed decode module."""
    return _install(model, PACKED_GROUPED if grouped else PACKED_DECODE)


def install_packed_grouped_moe(model) -> dict:
    """``install_packed_moe(model, grouped=True)``."""
    return _install(model, PACKED_GROUPED)


def install_packed_decode_moe(model) -> dict:
    """``install_packed_moe(model, grouped=False)``: packed one-token decode,
    Direct semantics for more rows."""
    return _install(model, PACKED_DECODE)
