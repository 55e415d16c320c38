"""Block-FP8 checkpoint (HF safetensors) straight into the packed expert bank.

Counterpart of the checkpoint side of ``glm53_flash_mlx/loader.py``: shard
discovery through ``model.safetensors.index.json`` or ``*.safetensors``
(``loader.py:40-50``) and the layer-by-layer packing of routed experts into a
``PackedFP8ExpertBank`` (``loader.py:167-244``, ``packed.py:782-850``),
restricted to the MoE hot path.  For one decoder layer:

* the routed experts' E4M3 codes (``F8_E4M3`` tensors, kept as bytes) and FP32
  ``weight_scale_inv`` block tables are copied expert by expert into the four
  contiguous bank tensors on the target device -- no BF16 or FP32 copy of any
  weight is made, and only one expert's tensors are in flight at a time;
* the router (``mlp.gate.weight``, ``mlp.gate.e_score_correction_bias``)
  becomes a :class:`Float32Gate` with FP32 parameters (``patch.py:131-142,
  296-318``);
* the shared expert becomes a :class:`DirectFP8Expert` over three
  :class:`BlockFP8Linear` projections.

Key layout (GLM-5 / DeepSeek-V3 HF naming, any prefix before ``.layers.``)::

    {prefix}.layers.{L}.mlp.experts.{e}.{gate,up,down}_proj.weight[_scale_inv]
    {prefix}.layers.{L}.mlp.shared_experts.{gate,up,down}_proj.weight[_scale_inv]
    {prefix}.layers.{L}.mlp.gate.weight
    {prefix}.layers.{L}.mlp.gate.e_score_correction_bias

Every check fails closed with ``ValueError`` (dtype, shape, missing or
non-contiguous experts), as the reference's bank packing does
(``packed.py:793-805``).
"""

from __future__ import annotations

import json
import math
import re
from pathlib import Path

import torch

from .fp8 import BLOCK_SIZE, DirectFP8Expert
from .ownership import TensorLayout, owned_tensor
from .packed import PackedFP8ExpertBank, PackedFP8MoE
from .router import Float32Gate

_EXPERT_KEY = re.compile(r"^(?P<prefix>.*)\.layers\.(?P<layer>\d+)\.mlp\.experts\.(?P<e>\d+)\.gate_proj\.weight$")
_CODE_DTYPES = (torch.uint8, getattr(torch, "float8_e4m3fn", torch.uint8))


class CheckpointIndex:
    """Tensor name -> shard file of a safetensors checkpoint directory (or of
    one ``.safetensors`` file), with lazily opened shard handles."""

    def __init__(self, path) -> None:
        from safetensors import safe_open  # imported here: only checkpoint loading needs it

        self._safe_open = safe_open
        path = Path(path)
        self.root = path if path.is_dir() else path.parent
        if path.is_file():
            files = [path]
        elif (path / "model.safetensors.index.json").exists():
            weight_map = json.loads((path / "model.safetensors.index.json").read_text())["weight_map"]
            files = [path / name for name in sorted(set(weight_map.values()))]
        else:
            files = sorted(path.glob("*.safetensors"))
        if not files:
            raise ValueError(f"no safetensors shards under {path}")
        self.file_of: dict[str, Path] = {}
        for f in files:
            with safe_open(str(f), framework="pt", device="cpu") as h:
                for key in h.keys():
                    self.file_of[key] = f
        self._handles: dict[tuple[Path, str], object] = {}

    def keys(self):
        return self.file_of.keys()

    def __contains__(self, key: str) -> bool:
        return key in self.file_of

    def get(self, key: str, device) -> torch.Tensor:
        if key not in self.file_of:
            raise ValueError(f"checkpoint tensor {key!r} is missing")
        f = self.file_of[key]
        dev = str(torch.device(device))
        h = self._handles.get((f, dev))
        if h is None:
            h = self._safe_open(str(f), framework="pt", device=dev)
            self._handles[(f, dev)] = h
        return h.get_tensor(key)

    def prefix(self) -> str:
        """The name prefix in front of ``.layers.`` (e.g. ``model.language_model``)."""
        for key in self.file_of:
            m = _EXPERT_KEY.match(key)
            if m:
                return m.group("prefix")
        raise ValueError("checkpoint holds no routed expert tensors (*.mlp.experts.*.gate_proj.weight)")

    def moe_layers(self, prefix: str | None = None) -> list[int]:
        prefix = self.prefix() if prefix is None else prefix
        layers = set()
        for key in self.file_of:
            m = _EXPERT_KEY.match(key)
            if m and m.group("prefix") == prefix:
                layers.add(int(m.group("layer")))
        return sorted(layers)

    def expert_count(self, layer: int, prefix: str) -> int:
        ids = set()
        for key in self.file_of:
            m = _EXPERT_KEY.match(key)
            if m and m.group("prefix") == prefix and int(m.group("layer")) == layer:
                ids.add(int(m.group("e")))
        if not ids:
            raise ValueError(f"layer {layer} has no routed experts")
        if ids != set(range(len(ids))):
            raise ValueError(f"layer {layer}: expert ids are not 0..{len(ids) - 1}")
        return len(ids)


def _index(source) -> CheckpointIndex:
    return source if isinstance(source, CheckpointIndex) else CheckpointIndex(source)


def _codes(t: torch.Tensor, key: str, shape: tuple[int, int]) -> torch.Tensor:
    if t.dtype not in _CODE_DTYPES:
        raise ValueError(f"{key}: expected E4M3 codes (F8_E4M3 or U8), got {t.dtype}")
    if tuple(t.shape) != shape:
        raise ValueError(f"{key}: shape {tuple(t.shape)} != {shape}")
    return t.view(torch.uint8)


def _scales(t: torch.Tensor, key: str, rows: int, cols: int) -> torch.Tensor:
    want = (math.ceil(rows / BLOCK_SIZE), math.ceil(cols / BLOCK_SIZE))
    if t.dtype != torch.float32:
        raise ValueError(f"{key}: expected float32 block scales, got {t.dtype}")
    if tuple(t.shape) != want:
        raise ValueError(f"{key}: scale shape {tuple(t.shape)} != block128 shape {want}")
    return t


def load_packed_bank(source, layer: int, *, device, prefix: str | None = None) -> PackedFP8ExpertBank:
    """The routed experts of one layer as a ``PackedFP8ExpertBank`` on ``device``
    (gate rows [0, I), up rows [I, 2I), reference layout ``packed.py:782-850``)."""
    idx = _index(source)
    prefix = idx.prefix() if prefix is None else prefix
    E = idx.expert_count(layer, prefix)
    base = f"{prefix}.layers.{layer}.mlp.experts"
    g0 = idx.get(f"{base}.0.gate_proj.weight", "cpu")
    if g0.dim() != 2:
        raise ValueError(f"{base}.0.gate_proj.weight must be 2-D, got {tuple(g0.shape)}")
    I, H = g0.shape
    del g0
    hb, ib = math.ceil(H / BLOCK_SIZE), math.ceil(I / BLOCK_SIZE)
    gu_w = torch.empty((E, 2 * I, H), dtype=torch.uint8, device=device)
    gu_s = torch.empty((E, 2 * ib, hb), dtype=torch.float32, device=device)
    d_w = torch.empty((E, H, I), dtype=torch.uint8, device=device)
    d_s = torch.empty((E, hb, ib), dtype=torch.float32, device=device)
    for e in range(E):
        p = f"{base}.{e}"
        for row0, srow0, proj in ((0, 0, "gate_proj"), (I, ib, "up_proj")):
            k = f"{p}.{proj}.weight"
            gu_w[e, row0:row0 + I].copy_(_codes(idx.get(k, device), k, (I, H)))
            k = f"{p}.{proj}.weight_scale_inv"
            gu_s[e, srow0:srow0 + ib].copy_(_scales(idx.get(k, device), k, I, H))
        k = f"{p}.down_proj.weight"
        d_w[e].copy_(_codes(idx.get(k, device), k, (H, I)))
        k = f"{p}.down_proj.weight_scale_inv"
        d_s[e].copy_(_scales(idx.get(k, device), k, H, I))
    layout = TensorLayout.ROW_MAJOR_CONTIGUOUS
    return PackedFP8ExpertBank(owned_tensor(gu_w, layout=layout), owned_tensor(gu_s, layout=layout),
                               owned_tensor(d_w, layout=layout), owned_tensor(d_s, layout=layout),
                               intermediate_size=I)


def load_router(source, layer: int, config, *, device, prefix: str | None = None) -> Float32Gate:
    """``mlp.gate`` of one layer as a :class:`Float32Gate` (FP32 weight and
    correction bias; a BF16 checkpoint weight converts exactly)."""
    idx = _index(source)
    prefix = idx.prefix() if prefix is None else prefix
    base = f"{prefix}.layers.{layer}.mlp.gate"
    gate = Float32Gate(config, device=device)
    w = idx.get(f"{base}.weight", device)
    if tuple(w.shape) != tuple(gate.weight.shape) or not w.is_floating_point():
        raise ValueError(f"{base}.weight: {tuple(w.shape)} {w.dtype} does not match the gate "
                         f"{tuple(gate.weight.shape)}")
    gate.weight.copy_(w.to(torch.float32))
    key = f"{base}.e_score_correction_bias"
    if key in idx:
        b = idx.get(key, device)
        if tuple(b.shape) != tuple(gate.e_score_correction_bias.shape):
            raise ValueError(f"{key}: shape {tuple(b.shape)} != {tuple(gate.e_score_correction_bias.shape)}")
        gate.e_score_correction_bias.copy_(b.to(torch.float32))
    return gate


def load_shared_expert(source, layer: int, *, limit: float, device, prefix: str | None = None):
    """``mlp.shared_experts`` of one layer as a :class:`DirectFP8Expert`, or
    None when the layer has no shared expert."""
    idx = _index(source)
    prefix = idx.prefix() if prefix is None else prefix
    base = f"{prefix}.layers.{layer}.mlp.shared_experts"
    if f"{base}.gate_proj.weight" not in idx:
        return None
    g = idx.get(f"{base}.gate_proj.weight", "cpu")
    Is, H = g.shape
    del g
    expert = DirectFP8Expert(H, Is, limit, device=device)
    for name, (rows, cols) in (("gate_proj", (Is, H)), ("up_proj", (Is, H)), ("down_proj", (H, Is))):
        proj = getattr(expert, name)
        k = f"{base}.{name}.weight"
        proj.weight.copy_(_codes(idx.get(k, device), k, (rows, cols)))
        k = f"{base}.{name}.weight_scale_inv"
        proj.weight_scale_inv.copy_(_scales(idx.get(k, device), k, rows, cols))
    return expert


def load_packed_moe(source, layer: int, config, *, device, prefix: str | None = None) -> PackedFP8MoE:
    """One checkpoint layer as a ready ``PackedFP8MoE`` (bank + FP32 router +
    shared expert) on ``device``."""
    idx = _index(source)
    prefix = idx.prefix() if prefix is None else prefix
    bank = load_packed_bank(idx, layer, device=device, prefix=prefix)
    if bank.expert_count != int(config.n_routed_experts) or bank.hidden_size != int(config.hidden_size) or \
            bank.intermediate_size != int(config.moe_intermediate_size):
        raise ValueError(f"layer {layer}: bank ({bank.expert_count}, {bank.hidden_size}, {bank.intermediate_size}) "
                         "does not match the config")
    gate = load_router(idx, layer, config, device=device, prefix=prefix)
    shared = load_shared_expert(idx, layer, limit=float(config.swiglu_limit), device=device, prefix=prefix)
    return PackedFP8MoE(bank, config, gate, shared)
