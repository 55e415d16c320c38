"""Packed FP8 expert bank and exact packed decode MoE on B200.

Counterpart of glm53_flash_mlx/packed.py: ``PackedFP8ExpertBank``
(packed.py:747-876), the per-expert views used by Direct-semantics prefill
(packed.py:658-744) and ``PackedFP8MoE`` (packed.py:879-923).  The one-token
decode runs the router's top-8 through two CUDA launches (fused gate/up/SwiGLU
over the 8 selected experts plus the shared expert, then down + slot-ordered
FP32 weighted reduce + BF16 shared add) with the reference's rounding points.
"""

from __future__ import annotations

import ctypes
import math
import os

import torch
from torch import nn

from . import _native as N
from .abi import PACKED_EXPERT_BANK_ABI  # noqa: F401
from .fp8 import BLOCK_SIZE, DECODE_TOP_K, DirectFP8MoE, block_fp8_linear, swiglu_pair
from .router import Float32Gate
from .ownership import (
    ResidentTensor,
    TensorLayout,
    TensorLease,
    borrowed_stable_tensor,
    owned_tensor,
    require_resident,
    resident_concatenate,
    storage_descriptor,
)

_SYNC_STATUS = os.environ.get("GLM53_SYNC_STATUS", "0") == "1"


class _PackedLinearView:
    """One projection of one expert, addressed inside the bank (no copy)."""

    def __init__(self, weight, scale_inv, *, expert_id: int, row_offset: int, scale_row_offset: int,
                 out_features: int):
        self._bank_weight = weight
        self._bank_scale_inv = scale_inv
        self.expert_id = int(expert_id)
        self.row_offset = int(row_offset)
        self.scale_row_offset = int(scale_row_offset)
        self.out_features = int(out_features)

    @property
    def weight(self):
        start = self.row_offset
        return self._bank_weight[self.expert_id, start : start + self.out_features]

    @property
    def weight_scale_inv(self):
        rows = math.ceil(self.out_features / BLOCK_SIZE)
        start = self.scale_row_offset
        return self._bank_scale_inv[self.expert_id, start : start + rows]

    def __call__(self, x):
        return block_fp8_linear(x, self.weight, self.weight_scale_inv)


class _PackedExpertView:
    def __init__(self, bank: "PackedFP8ExpertBank", expert_id: int, limit: float):
        inter = bank.intermediate_size
        scale_rows = bank.intermediate_scale_rows
        self.gate_proj = _PackedLinearView(bank.gate_up_weight, bank.gate_up_scale_inv, expert_id=expert_id,
                                           row_offset=0, scale_row_offset=0, out_features=inter)
        self.up_proj = _PackedLinearView(bank.gate_up_weight, bank.gate_up_scale_inv, expert_id=expert_id,
                                         row_offset=inter, scale_row_offset=scale_rows, out_features=inter)
        self.down_proj = _PackedLinearView(bank.down_weight, bank.down_scale_inv, expert_id=expert_id,
                                           row_offset=0, scale_row_offset=0,
                                           out_features=bank.down_weight.shape[1])
        self.limit = float(limit)

    def __call__(self, x):
        return self.down_proj(swiglu_pair(self.gate_proj(x), self.up_proj(x), self.limit))


class PackedFP8ExpertBank(nn.Module):
    """Four contiguous canonical-FP8 buffers for one routed MoE layer:
    gate_up_weight [E,2I,H] (gate rows then up rows), gate_up_scale_inv
    [E,2*ceil(I/128),ceil(H/128)], down_weight [E,H,I], down_scale_inv
    [E,ceil(H/128),ceil(I/128)]."""

    def __init__(self, gate_up_weight: TensorLease | ResidentTensor, gate_up_scale_inv: TensorLease | ResidentTensor,
                 down_weight: TensorLease | ResidentTensor, down_scale_inv: TensorLease | ResidentTensor, *,
                 intermediate_size: int):
        super().__init__()
        resident = {
            "gate_up_weight": require_resident(gate_up_weight),
            "gate_up_scale_inv": require_resident(gate_up_scale_inv),
            "down_weight": require_resident(down_weight),
            "down_scale_inv": require_resident(down_scale_inv),
        }
        for name, value in resident.items():
            self.register_buffer(name, value.value, persistent=False)
        self.storage_contracts = {name: storage_descriptor(value) for name, value in resident.items()}
        self._storage_owners = tuple(value.owner for value in resident.values() if value.owner is not None)
        self.intermediate_size = int(intermediate_size)
        self.intermediate_scale_rows = math.ceil(intermediate_size / BLOCK_SIZE)
        E, two_i, H = self.gate_up_weight.shape
        if self.gate_up_weight.dtype != torch.uint8 or self.down_weight.dtype != torch.uint8:
            raise ValueError("packed expert weights must remain uint8 E4M3")
        if self.gate_up_scale_inv.dtype != torch.float32 or self.down_scale_inv.dtype != torch.float32:
            raise ValueError("packed expert scales must remain float32")
        if two_i != 2 * self.intermediate_size or tuple(self.down_weight.shape) != (E, H, self.intermediate_size):
            raise ValueError("packed expert bank shapes are inconsistent")

    @classmethod
    def pack(cls, experts) -> "PackedFP8ExpertBank":
        experts = list(experts)
        if not experts:
            raise ValueError("cannot pack an empty expert list")
        hidden_size = experts[0].gate_proj.weight.shape[1]
        intermediate_size = experts[0].gate_proj.weight.shape[0]
        expert_count = len(experts)
        scale_rows = math.ceil(intermediate_size / BLOCK_SIZE)
        hidden_scale_rows = math.ceil(hidden_size / BLOCK_SIZE)
        for expert in experts:
            expected = (
                (tuple(expert.gate_proj.weight.shape), (intermediate_size, hidden_size)),
                (tuple(expert.up_proj.weight.shape), (intermediate_size, hidden_size)),
                (tuple(expert.down_proj.weight.shape), (hidden_size, intermediate_size)),
            )
            if any(actual != wanted for actual, wanted in expected):
                raise ValueError("expert projection shapes are not uniform")
            for projection in (expert.gate_proj, expert.up_proj, expert.down_proj):
                if projection.weight.dtype != torch.uint8:
                    raise ValueError("packed expert weights must remain uint8 E4M3")
                if projection.weight_scale_inv.dtype != torch.float32:
                    raise ValueError("packed expert scales must remain float32")

        def stable(projection, name: str):
            return borrowed_stable_tensor(getattr(projection, name), owner=projection,
                                          layout=TensorLayout.ROW_MAJOR_CONTIGUOUS)

        gate_up_weight = resident_concatenate(
            [stable(p, "weight") for e in experts for p in (e.gate_proj, e.up_proj)], axis=0
        ).value.reshape(expert_count, 2 * intermediate_size, hidden_size)
        gate_up_scale_inv = resident_concatenate(
            [stable(p, "weight_scale_inv") for e in experts for p in (e.gate_proj, e.up_proj)], axis=0
        ).value.reshape(expert_count, 2 * scale_rows, hidden_scale_rows)
        down_weight = resident_concatenate([stable(e.down_proj, "weight") for e in experts], axis=0
                                           ).value.reshape(expert_count, hidden_size, intermediate_size)
        down_scale_inv = resident_concatenate([stable(e.down_proj, "weight_scale_inv") for e in experts], axis=0
                                              ).value.reshape(expert_count, hidden_scale_rows, scale_rows)
        layout = TensorLayout.ROW_MAJOR_CONTIGUOUS
        return cls(
            owned_tensor(gate_up_weight, layout=layout),
            owned_tensor(gate_up_scale_inv, layout=layout),
            owned_tensor(down_weight, layout=layout),
            owned_tensor(down_scale_inv, layout=layout),
            intermediate_size=intermediate_size,
        )

    @property
    def expert_count(self) -> int:
        return self.gate_up_weight.shape[0]

    @property
    def hidden_size(self) -> int:
        return self.gate_up_weight.shape[2]

    @property
    def nbytes(self) -> int:
        return sum(
            t.numel() * t.element_size()
            for t in (self.gate_up_weight, self.gate_up_scale_inv, self.down_weight, self.down_scale_inv)
        )

    def expert(self, expert_id: int, *, limit: float) -> _PackedExpertView:
        if not 0 <= expert_id < self.expert_count:
            raise IndexError(expert_id)
        return _PackedExpertView(self, expert_id, limit)


def shared_fp8_tensors(shared) -> tuple | None:
    """(gate_w, gate_s, up_w, up_s, down_w, down_s) of a shared expert made of
    BlockFP8Linear projections, or None when it is some other module."""
    if shared is None:
        return None
    try:
        parts = []
        for name in ("gate_proj", "up_proj", "down_proj"):
            proj = getattr(shared, name)
            if getattr(proj, "bias", None) is not None:
                return None
            if proj.weight.dtype != torch.uint8 or proj.weight_scale_inv.dtype != torch.float32:
                return None
            parts += [proj.weight.contiguous(), proj.weight_scale_inv.contiguous()]
        return tuple(parts)
    except AttributeError:
        return None


def packed_decode_moe(x: torch.Tensor, expert_ids: torch.Tensor, scores: torch.Tensor, bank: PackedFP8ExpertBank,
                      shared: tuple | None, *, limit: float, workspace: N.Workspace | None = None,
                      status: torch.Tensor | None = None, split: str | None = None,
                      after_router: bool = False, hc: tuple | None = None) -> torch.Tensor | None:
    """One-token routed MoE (+ shared expert) over the packed bank.

    x: BF16 [H]; expert_ids: int32/uint32 [top_k]; scores: float32 [top_k].
    Returns BF16 [H].  ``split="shared"`` computes only the shared expert into
    ``workspace`` (ids and scores unread, returns None); a later
    ``split="routed"`` call on the same workspace, ordered after it, finishes
    the layer (GLM53_FLAG_SHARED_ONLY / GLM53_FLAG_SKIP_SHARED).
    ``after_router=True`` states that the last kernel on the current stream
    is the router that produced ``expert_ids``/``scores`` from ``x``: when no
    argument needs a copy here, the shared expert then streams while that
    router still runs (GLM53_FLAG_AFTER_ROUTER; same result bits).
    ``hc=(residual [4, H] BF16, post [4] FP32, comb [4, 4] FP32)`` fuses the
    layer's mHC post-expand into the final reduce and returns the next state
    BF16 [4, H] (``glm53_packed_decode_moe_hc``; the bits of the decode
    followed by ``hc_expand``)."""
    dev = N.require_cuda(x, expert_ids, scores, bank.gate_up_weight)
    H = bank.hidden_size
    I = bank.intermediate_size
    top_k = expert_ids.numel()
    if x.numel() != H:
        raise ValueError(f"decode input width {x.numel()} != bank hidden {H}")
    # no kernel may run between the router and this call's launch for the
    # programmatic overlap: every argument must be usable as it is
    overlap = (after_router and split is None and x.is_contiguous() and expert_ids.is_contiguous() and
               scores.is_contiguous() and expert_ids.dtype == torch.int32 and
               scores.dtype == torch.float32 and (hc is None or all(t.is_contiguous() for t in hc)))
    x = x.reshape(H).contiguous()
    ids = expert_ids.reshape(-1).to(torch.int32).contiguous()
    sc = scores.reshape(-1).to(torch.float32).contiguous()
    if shared is not None:
        sg_w, sg_s, su_w, su_s, sd_w, sd_s = shared
        Is = sg_w.shape[0]
    else:
        sg_w = sg_s = su_w = su_s = sd_w = sd_s = None
        Is = 0
    weights = (bank.gate_up_weight, bank.down_weight, *(() if shared is None else (sg_w, su_w, sd_w)))
    overlap = overlap and N.e4m3_scanned(*weights)
    flags = N.decode_flags(*weights)
    if split is not None:
        if shared is None or split not in ("shared", "routed"):
            raise ValueError("split decode needs a shared expert and split='shared' or 'routed'")
        flags |= N.FLAG_SHARED_ONLY if split == "shared" else N.FLAG_SKIP_SHARED
    ws_bytes = N.lib().glm53_packed_decode_workspace_bytes(top_k, H, I, Is)
    wsp = workspace or N.Workspace()
    overlap = overlap and wsp.has(dev, "decode", ws_bytes) and (status is not None or wsp.has(dev, "status", 4))
    ws = wsp.get(dev, "decode", ws_bytes)
    if status is None:
        status = wsp.get(dev, "status", 4)
    if overlap:  # nothing was launched since the router: no copy, scan or zero-fill above
        flags |= N.FLAG_AFTER_ROUTER
    if hc is not None:
        residual, post, comb = hc
        if split is not None:
            raise ValueError("the fused hc expand takes the whole decode (no split)")
        if (residual.dtype != torch.bfloat16 or residual.numel() != 4 * H or post.dtype != torch.float32 or
                post.numel() != 4 or comb.dtype != torch.float32 or comb.numel() != 16):
            raise ValueError("hc needs residual BF16 [4, H], post FP32 [4] and comb FP32 [4, 4]")
        residual, post, comb = residual.contiguous(), post.contiguous(), comb.contiguous()
        state = torch.empty((4, H), dtype=torch.bfloat16, device=dev)
        N.check(
            N.lib().glm53_packed_decode_moe_hc(
                x.data_ptr(), H, ids.data_ptr(), sc.data_ptr(), top_k,
                bank.gate_up_weight.data_ptr(), bank.gate_up_scale_inv.data_ptr(),
                bank.down_weight.data_ptr(), bank.down_scale_inv.data_ptr(), bank.expert_count, I,
                N.ptr(sg_w), N.ptr(sg_s), N.ptr(su_w), N.ptr(su_s), N.ptr(sd_w), N.ptr(sd_s), Is,
                float(limit), residual.data_ptr(), post.data_ptr(), comb.data_ptr(), state.data_ptr(),
                ws.data_ptr(), ws.numel(), status.data_ptr(), flags, N.stream(dev),
            ),
            "glm53_packed_decode_moe_hc",
        )
        if _SYNC_STATUS:
            check_status(status)
        return state
    out = torch.empty(H, dtype=torch.bfloat16, device=dev)
    N.check(
        N.lib().glm53_packed_decode_moe(
            x.data_ptr(), H, ids.data_ptr(), sc.data_ptr(), top_k,
            bank.gate_up_weight.data_ptr(), bank.gate_up_scale_inv.data_ptr(),
            bank.down_weight.data_ptr(), bank.down_scale_inv.data_ptr(), bank.expert_count, I,
            N.ptr(sg_w), N.ptr(sg_s), N.ptr(su_w), N.ptr(su_s), N.ptr(sd_w), N.ptr(sd_s), Is,
            float(limit), out.data_ptr(), ws.data_ptr(), ws.numel(), status.data_ptr(), flags, N.stream(dev),
        ),
        "glm53_packed_decode_moe",
    )
    if _SYNC_STATUS:
        check_status(status)
    return None if split == "shared" else out


# Routes the coalesced batched decode takes in one call (kBdMaxRoutes in
# csrc/batched_decode.cu), counting each token's shared-expert route: with
# top-8 routing, batches of 2..455 rows run on the device with the Direct
# module's multi-row semantics (below the grouped path's 256-route threshold
# that is every batch of up to 31 rows, as grouped_fp8.py:323-326 routes them).
BATCHED_DECODE_MAX_ROUTES = 4096
BATCHED_DECODE_MAX_ROWS = BATCHED_DECODE_MAX_ROUTES // (DECODE_TOP_K + 1)


def batched_decode_moe(x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor, bank: PackedFP8ExpertBank,
                       shared_experts, *, limit: float, workspace: N.Workspace | None = None,
                       status: torch.Tensor | None = None) -> torch.Tensor:
    """A few decode rows through the packed bank with the Direct module's
    semantics (glm53_flash_mlx/fp8.py:384-399): each touched expert streams its
    weights once for all its routes, the weighted rows are added in BF16 in
    ascending expert id (``glm53_batched_decode_moe``), plus the shared expert
    module's output.  A block-FP8 shared expert of the routed experts' width
    rides in the same kernels as one more route per token of weight 1.0
    (``glm53_batched_decode_moe_shared``).  x: BF16 [T, H]; indices / scores:
    [T, top_k]."""
    dev = N.require_cuda(x, indices, scores, bank.gate_up_weight)
    T, H = x.shape
    if H != bank.hidden_size:
        raise ValueError(f"decode input width {H} != bank hidden {bank.hidden_size}")
    top_k = indices.shape[-1]
    E, I = bank.expert_count, bank.intermediate_size
    x = x.contiguous()
    ids = indices.reshape(-1).to(torch.int32).contiguous()
    sc = scores.reshape(-1).to(torch.float32).contiguous()
    wsp = workspace or N.Workspace()
    if status is None:
        status = wsp.get(dev, "status", 4)
    out = torch.empty_like(x)
    sw = shared_fp8_tensors(shared_experts)
    flags = N.decode_flags(bank.gate_up_weight, bank.down_weight, *(() if sw is None else sw[0::2]))
    if sw is not None and sw[0].shape == (I, H) and sw[4].shape == (H, I) and top_k < 32:
        # the shared expert rides in the coalesced kernels as one more route per token
        ws = wsp.get(dev, "batched_shared", N.lib().glm53_batched_decode_shared_workspace_bytes(T, top_k, E, H, I))
        N.check(
            N.lib().glm53_batched_decode_moe_shared(
                x.data_ptr(), T, H, ids.data_ptr(), sc.data_ptr(), top_k, bank.gate_up_weight.data_ptr(),
                bank.gate_up_scale_inv.data_ptr(), bank.down_weight.data_ptr(), bank.down_scale_inv.data_ptr(), E, I,
                *(t.data_ptr() for t in sw), float(limit), out.data_ptr(), ws.data_ptr(), ws.numel(),
                status.data_ptr(), flags, N.stream(dev),
            ),
            "glm53_batched_decode_moe_shared",
        )
        if _SYNC_STATUS:
            check_status(status)
        return out
    ws = wsp.get(dev, "batched", N.lib().glm53_batched_decode_workspace_bytes(T, top_k, E, H, I))
    shared = shared_experts(x).contiguous() if shared_experts is not None else None
    N.check(
        N.lib().glm53_batched_decode_moe(
            x.data_ptr(), T, H, ids.data_ptr(), sc.data_ptr(), top_k, bank.gate_up_weight.data_ptr(),
            bank.gate_up_scale_inv.data_ptr(), bank.down_weight.data_ptr(), bank.down_scale_inv.data_ptr(), E, I,
            float(limit), N.ptr(shared), out.data_ptr(), ws.data_ptr(), ws.numel(), status.data_ptr(),
            N.decode_flags(bank.gate_up_weight, bank.down_weight), N.stream(dev),
        ),
        "glm53_batched_decode_moe",
    )
    if _SYNC_STATUS:
        check_status(status)
    return out


def _raise_status(word: int) -> None:
    if word & N.STATUS_BAD_EXPERT:
        raise IndexError("expert id out of range in routed MoE")
    if word & N.STATUS_WAIT_TIMEOUT:
        raise RuntimeError("a bounded device wait gave up")
    if word:
        raise RuntimeError(f"device status 0x{word:x}")


def check_status(status: torch.Tensor, *, clear: bool = True) -> None:
    """Raise for device-side fail-closed signals (one device->host read);
    the word is cleared first so the next call starts clean."""
    word = int(status.view(torch.int32)[0].item()) & 0xFFFFFFFF
    if clear and word:
        status.view(torch.int32)[:1].zero_()
    _raise_status(word)


class StatusWord:
    """A layer's device status word and its pinned host mirror.

    The kernels OR fail-closed bits into ``word`` (an out-of-range expert id,
    a bounded wait that gave up) instead of trapping, as the reference's
    device-side invalid-route counter does (native_indexer_plan.metal:1880-1900).
    ``publish()`` enqueues a one-thread kernel that copies the word into the
    pinned host mirror; ``raise_pending()`` reads the mirror with a plain host
    read -- no device synchronisation on the success path -- and raises the
    reference's exception (``IndexError`` for a bad expert id, packed.py:868-876;
    ``RuntimeError`` otherwise).  A module publishes after its kernels and checks
    at the start of its next call, so an error surfaces one call late at the
    latest; ``check()`` synchronises and raises at once."""

    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        # one int32 word (in a 256-byte allocation of its own)
        self.word = torch.zeros(64, dtype=torch.int32, device=self.device)[:1]
        self.host = torch.zeros(4, dtype=torch.int32).pin_memory()
        # a plain host read of the mirror (indexing the tensor costs ~3 us a call)
        self._host_word = ctypes.c_int32.from_address(self.host.data_ptr())

    def publish(self) -> None:
        N.check(N.lib().glm53_status_mirror(self.word.data_ptr(), self.host.data_ptr(), N.stream(self.device)),
                "glm53_status_mirror")

    def _fail(self, word: int) -> None:
        # let every enqueued mirror copy land before clearing, so no stale
        # copy re-raises at the next call
        torch.cuda.synchronize(self.device)
        word |= int(self.word[0].item()) | int(self.host[0])
        self.word.zero_()
        torch.cuda.synchronize(self.device)
        self.host.zero_()
        _raise_status(word & 0xFFFFFFFF)

    def raise_pending(self) -> None:
        word = self._host_word.value
        if word:
            self._fail(word)

    def check(self) -> None:
        """Synchronise the device and raise for any bit set so far."""
        torch.cuda.synchronize(self.device)
        word = int(self.word[0].item()) | int(self.host[0])
        if word:
            self._fail(word)


class CapturedDecode:
    """One decode token through a MoE module (its gate, the decode kernels and
    the shared expert) captured into a CUDA graph with static buffers.

    ``step(x, out=None)`` copies ``x`` (host or device, ``hidden`` values) into
    the static input, replays the graph on the current stream and returns the
    static output (or copies it into ``out``, e.g. pinned host memory); the
    static output is overwritten by the next call.  Every operation stays
    stream-ordered, so host buffers may be pinned and the copies asynchronous.
    With a host input (and a host ``out`` or none) the copy in, the replay and
    the copy out are one library call (``glm53_graph_step``).
    """

    def __init__(self, module: nn.Module, hidden: int, device):
        device = torch.device(device)
        # the module's status word (its captured calls publish into the
        # mirror): raise at the next step, as the module call itself would
        words = getattr(module, "status_word", None)
        self._status = words(device) if callable(words) else None
        self.x = torch.zeros((1, 1, hidden), dtype=torch.bfloat16, device=device)
        side = torch.cuda.Stream(device=device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):  # buffers, scans and kernel attributes outside the capture
            for _ in range(2):
                module(self.x)
        torch.cuda.current_stream(device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=side):
            self.out = module(self.x)
        if self.out.dtype != self.x.dtype or self.out.numel() != self.x.numel():
            raise ValueError("CapturedDecode needs a module whose output has its input's shape and dtype")
        self._exec = self.graph.raw_cuda_graph_exec()  # instantiated at the end of the capture
        if not self._exec:
            raise RuntimeError("CapturedDecode: the captured graph has no executable instance")

    def check(self) -> None:
        """Synchronise and raise for any fail-closed bit the captured kernels set."""
        if self._status is not None:
            self._status.check()

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if self._status is not None:
            self._status.raise_pending()
        nbytes = self.x.numel() * self.x.element_size()
        host_in = x.device.type == "cpu" and x.dtype == self.x.dtype and x.is_contiguous() and x.numel() == self.x.numel()
        host_out = out is not None and out.device.type == "cpu" and out.dtype == self.out.dtype and \
            out.is_contiguous() and out.numel() == self.out.numel()
        if host_in and (out is None or host_out):
            # host buffers: H2D copy, graph launch and D2H copy in one library call
            N.check(N.lib().glm53_graph_step(self._exec, x.data_ptr(), self.x.data_ptr(), nbytes, self.out.data_ptr(),
                                             out.data_ptr() if host_out else None, nbytes, N.stream(self.x.device)),
                    "glm53_graph_step")
            return self.out if out is None else out
        self.x.copy_(x.reshape(self.x.shape), non_blocking=True)
        self.graph.replay()
        if out is None:
            return self.out
        out.copy_(self.out.reshape(out.shape), non_blocking=True)
        return out


class PackedDecodeStep:
    """One decode token through a PackedFP8MoE layer (its Float32Gate router
    and the packed decode) as one library call per step, on static device
    buffers (``glm53_decode_step_host``).

    ``step(x, out=None)`` takes the ``hidden``-wide BF16 row on the host (a
    pinned row is read by a kernel through its device mapping) or on the
    device; the result goes into ``out`` (host or device; into a pinned host
    ``out`` straight from the decode kernel) or, with ``out=None``, into the
    static output that is returned and overwritten by the next call.  Every
    operation is ordered on the current stream.  Same bits as the module call.
    """

    def __init__(self, module: PackedFP8MoE):
        bank, gate = module.bank, module.gate
        dev = bank.gate_up_weight.device
        H, I, E = bank.hidden_size, bank.intermediate_size, bank.expert_count
        shared = shared_fp8_tensors(module.shared_experts)
        Is = shared[0].shape[0] if shared is not None else 0
        lib = N.lib()
        self.x = torch.zeros((1, 1, H), dtype=torch.bfloat16, device=dev)
        self.out = torch.zeros((1, 1, H), dtype=torch.bfloat16, device=dev)
        self._ids = torch.zeros(DECODE_TOP_K, dtype=torch.int32, device=dev)
        self._scores = torch.zeros(DECODE_TOP_K, dtype=torch.float32, device=dev)
        ws = module._workspace
        rws = ws.get(dev, "step_router", lib.glm53_router_workspace_bytes(1, E))
        dws = ws.get(dev, "step_decode", lib.glm53_packed_decode_workspace_bytes(DECODE_TOP_K, H, I, Is))
        self._status = module.status_word(dev)
        status = self._status.word
        weights = (bank.gate_up_weight, bank.down_weight, *(() if shared is None else shared[0::2]))
        router_w = gate.weight.contiguous()
        router_b = gate.e_score_correction_bias.contiguous()
        sh = shared if shared is not None else (None,) * 6
        # the step binds raw device addresses: hold every bound tensor and
        # remember its identity, so a replaced or rewritten weight is refused
        # (the reference plan's check, native_packed_moe_plan.cpp:270-272)
        self._bound = self._bound_tensors(module)
        self._identity = self._identities(self._bound)
        self._slots = self._binding_slots(module)
        self._keep = (router_w, router_b, rws, dws, status, sh)
        self._desc = N.DecodeStepDesc(
            H=H, E=E, I=I, I_shared=Is, top_k=DECODE_TOP_K, n_group=gate.n_group, topk_group=gate.topk_group,
            norm_topk_prob=int(gate.norm_topk_prob), routed_scaling_factor=gate.routed_scaling_factor,
            limit=float(module.config.swiglu_limit), flags=N.decode_flags(*weights),
            router_w=router_w.data_ptr(), router_bias=router_b.data_ptr(),
            gate_up_w=bank.gate_up_weight.data_ptr(), gate_up_s=bank.gate_up_scale_inv.data_ptr(),
            down_w=bank.down_weight.data_ptr(), down_s=bank.down_scale_inv.data_ptr(),
            shared_gate_w=N.ptr(sh[0]), shared_gate_s=N.ptr(sh[1]), shared_up_w=N.ptr(sh[2]),
            shared_up_s=N.ptr(sh[3]), shared_down_w=N.ptr(sh[4]), shared_down_s=N.ptr(sh[5]),
            x=self.x.data_ptr(), expert_ids=self._ids.data_ptr(), scores=self._scores.data_ptr(),
            out=self.out.data_ptr(), router_workspace=rws.data_ptr(), router_workspace_bytes=rws.numel(),
            decode_workspace=dws.data_ptr(), decode_workspace_bytes=dws.numel(), status=status.data_ptr(),
            status_host=self._status.host.data_ptr())
        self._pdesc = ctypes.pointer(self._desc)
        self._lib = lib
        self._device = self.x.device
        # a second descriptor whose input and output point at the caller's
        # device rows (run_device): no copy into or out of the static buffers
        self._ddesc = N.DecodeStepDesc.from_buffer_copy(self._desc)
        self._pddesc = ctypes.pointer(self._ddesc)

    @staticmethod
    def _bound_tensors(module) -> tuple:
        bank, gate = module.bank, module.gate
        shared = shared_fp8_tensors(module.shared_experts)
        return (bank.gate_up_weight, bank.gate_up_scale_inv, bank.down_weight, bank.down_scale_inv,
                gate.weight, gate.e_score_correction_bias, *(() if shared is None else shared))

    @staticmethod
    def _identities(tensors) -> tuple:
        return tuple((t.data_ptr(), t._version) for t in tensors)

    @staticmethod
    def _binding_slots(module) -> tuple:
        """(dict, name, object) for every attribute the step read its tensors
        through: the layer's bank / gate / shared expert, the bank's four
        buffers, the gate's weight and bias, the shared projections' tensors."""
        def slot(owner, name):
            for d in (owner._parameters, owner._buffers, owner._modules, owner.__dict__):
                if name in d:
                    return (d, name, d[name])
            raise AttributeError(name)

        slots = [slot(module, "bank"), slot(module, "gate"), slot(module, "shared_experts")]
        slots += [slot(module.bank, n) for n in ("gate_up_weight", "gate_up_scale_inv", "down_weight",
                                                 "down_scale_inv")]
        slots += [slot(module.gate, "weight"), slot(module.gate, "e_score_correction_bias")]
        if shared_fp8_tensors(module.shared_experts) is not None:
            for proj in ("gate_proj", "up_proj", "down_proj"):
                p = getattr(module.shared_experts, proj)
                slots += [slot(module.shared_experts, proj), slot(p, "weight"), slot(p, "weight_scale_inv")]
        return tuple(slots)

    def bound_ok(self) -> bool:
        """True while every tensor the step bound is still the layer's, unchanged."""
        for (d, name, obj) in self._slots:
            if d.get(name) is not obj:
                return False
        return tuple([(t.data_ptr(), t._version) for t in self._bound]) == self._identity

    def _check_bound(self) -> None:
        if not self.bound_ok():
            raise RuntimeError("packed MoE decode step: a bound weight's identity changed (replaced, reallocated or "
                               "written in place); capture a new step with capture_decode()")

    def check(self) -> None:
        """Synchronise and raise for any fail-closed bit the step's kernels set
        (the per-call check sees the bits of earlier calls only)."""
        self._status.check()

    def run_device(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """One token from the device row `x` into the device row `out` (both
        BF16, contiguous, ``hidden`` values, 16-byte aligned): the router reads
        `x` and the decode writes `out` directly, one library call."""
        self._check_bound()
        self._status.raise_pending()
        d = self._ddesc
        d.x = x.data_ptr()
        d.out = out.data_ptr()
        N.check(self._lib.glm53_decode_step_host(self._pddesc, None, None, N.stream(self._device)),
                "glm53_decode_step_host")
        if _SYNC_STATUS:
            self._status.check()
        return out

    @staticmethod
    def device_row_ok(t: torch.Tensor, H: int) -> bool:
        return (t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous() and t.numel() == H and
                t.data_ptr() % 16 == 0)

    @staticmethod
    def supported(module) -> bool:
        from .router import Float32Gate

        bank = module.bank
        shared = shared_fp8_tensors(module.shared_experts)
        limit = module.config.swiglu_limit
        return (isinstance(module.gate, Float32Gate) and module.gate.top_k == DECODE_TOP_K and
                float(limit) == int(limit) and bank.hidden_size % BLOCK_SIZE == 0 and
                bank.intermediate_size % BLOCK_SIZE == 0 and
                (module.shared_experts is None or (shared is not None and shared[0].shape[0] % BLOCK_SIZE == 0)))

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        H = self._desc.H
        if x.numel() != H:
            raise ValueError(f"decode step input has {x.numel()} values, layer width {H}")
        self._check_bound()
        # bits of earlier steps, mirrored into pinned host memory by this
        # step's predecessors on the stream: a host read, no synchronisation
        self._status.raise_pending()
        if not x.is_cuda:
            if x.dtype != torch.bfloat16 or not x.is_contiguous():
                x = x.to(torch.bfloat16).contiguous()
            x_host = x.data_ptr()
        else:
            self.x.copy_(x.reshape(self.x.shape))
            x_host = None
        out_host = None
        if out is not None:
            if out.numel() != H or out.dtype != torch.bfloat16 or not out.is_contiguous():
                raise ValueError("decode step output must be a contiguous BF16 row of the layer width")
            if not out.is_cuda:
                out_host = out.data_ptr()
        N.check(self._lib.glm53_decode_step_host(self._pdesc, x_host, out_host, N.stream(self._device)),
                "glm53_decode_step_host")
        if _SYNC_STATUS:
            self._status.check()
        if out is None:
            return self.out
        if out_host is None:
            out.copy_(self.out.reshape(out.shape))
        return out


class PackedFP8MoE(DirectFP8MoE):
    """Exact fused batch-1 decode and Direct semantics over a packed bank."""

    def __init__(self, bank, config, gate, shared_experts):
        nn.Module.__init__(self)
        self.bank = bank
        self.config = config
        self.gate = gate
        self.shared_experts = shared_experts
        self._expert_views = tuple(
            bank.expert(expert_id, limit=config.swiglu_limit) for expert_id in range(bank.expert_count)
        )
        self._workspace = N.Workspace()
        self._status_words: dict = {}

    def _expert(self, expert_id: int):
        return self._expert_views[expert_id]

    def status_word(self, device=None) -> StatusWord:
        """This layer's StatusWord on `device` (default: the bank's device)."""
        dev = torch.device(device) if device is not None else self.bank.gate_up_weight.device
        sw = self._status_words.get(dev)
        if sw is None:
            sw = self._status_words[dev] = StatusWord(dev)
        return sw

    @property
    def status(self) -> torch.Tensor:
        """The device status word the layer's kernels write (int32, word 0)."""
        return self.status_word().word

    def check_status(self) -> None:
        """Synchronise and raise for any fail-closed bit the layer's kernels set."""
        for sw in self._status_words.values():
            sw.check()

    def capture_decode(self) -> PackedDecodeStep | CapturedDecode:
        """This layer's one-token decode on static buffers, called once per
        token: one library call (router + packed decode, host or device row)
        when the layer has the Float32Gate router and the tensor-core shapes,
        else a replayable CUDA graph of the module call."""
        if PackedDecodeStep.supported(self):
            return PackedDecodeStep(self)
        return CapturedDecode(self, self.bank.hidden_size, self.bank.gate_up_weight.device)

    def forward_expand(self, x, residual, post, comb):
        """The layer followed by the mHC post-expand: ``hc_expand(self(x),
        residual, post, comb)``.  One token with the Float32Gate router and the
        tensor-core shapes runs the expand inside the decode's final reduce
        (``glm53_packed_decode_moe_hc``, same bits); anything else calls the
        two steps.  x [..., H]; residual [..., 4, H]; returns [..., 4, H]."""
        from .hyper_connection import hc_expand

        flat_x = x.reshape(-1, x.shape[-1])
        shared = shared_fp8_tensors(self.shared_experts)
        limit = self.config.swiglu_limit
        H, I = self.bank.hidden_size, self.bank.intermediate_size
        fused = (flat_x.shape[0] == 1 and flat_x.is_cuda and isinstance(self.gate, Float32Gate) and
                 self.gate.top_k == DECODE_TOP_K and float(limit) == int(limit) and H % BLOCK_SIZE == 0 and
                 I % BLOCK_SIZE == 0 and (self.shared_experts is None or
                                          (shared is not None and shared[0].shape[0] == I)))
        if not fused:
            return hc_expand(self(x), residual, post, comb)
        sw = self.status_word(flat_x.device)
        sw.raise_pending()
        indices, scores = self.gate(x)
        state = packed_decode_moe(flat_x[0], indices.reshape(-1), scores.reshape(-1), self.bank, shared, limit=limit,
                                  workspace=self._workspace, status=sw.word, after_router=True,
                                  hc=(residual, post, comb))
        sw.publish()
        return state.reshape(residual.shape)

    def forward(self, x):
        flat_x = x.reshape(-1, x.shape[-1])
        if flat_x.shape[0] != 1:
            if not 2 <= flat_x.shape[0] <= BATCHED_DECODE_MAX_ROWS or not flat_x.is_cuda:
                return super().forward(x)
            sw = self.status_word(flat_x.device)
            sw.raise_pending()
            indices, scores = self.gate(x)
            limit = self.config.swiglu_limit
            if (indices.shape[-1] != DECODE_TOP_K or float(limit) != int(limit) or
                    self.bank.hidden_size % BLOCK_SIZE or self.bank.intermediate_size % BLOCK_SIZE):
                return self._forward_routes(x, indices, scores)
            out = batched_decode_moe(flat_x, indices.reshape(flat_x.shape[0], -1),
                                     scores.reshape(flat_x.shape[0], -1), self.bank, self.shared_experts,
                                     limit=limit, workspace=self._workspace, status=sw.word).reshape(x.shape)
            sw.publish()
            return out
        if flat_x.is_cuda:
            self.status_word(flat_x.device).raise_pending()
            step = self.__dict__.get("_device_step")
            if step is not None and not step.bound_ok():  # the layer's weights were replaced: rebind
                step = self.__dict__["_device_step"] = None
            if step is None and PackedDecodeStep.device_row_ok(flat_x, self.bank.hidden_size) and \
                    PackedDecodeStep.supported(self):
                step = self.__dict__["_device_step"] = PackedDecodeStep(self)
            if step is not None and PackedDecodeStep.device_row_ok(flat_x, self.bank.hidden_size):
                # one token, FP32 router, tensor-core shapes: router + decode in one library call
                out = torch.empty_like(flat_x)
                return step.run_device(flat_x, out).reshape(x.shape)
        indices, scores = self.gate(x)
        if indices.shape[-1] != DECODE_TOP_K:
            return super().forward(x)
        limit = self.config.swiglu_limit
        if float(limit) != int(limit):
            raise ValueError("exact fused packed decode requires an integral clamp limit")
        shared = shared_fp8_tensors(self.shared_experts)
        sw = self.status_word(flat_x.device)
        result = packed_decode_moe(flat_x[0], indices.reshape(-1), scores.reshape(-1), self.bank, shared,
                                   limit=limit, workspace=self._workspace, status=sw.word,
                                   after_router=isinstance(self.gate, Float32Gate)).reshape(x.shape)
        if shared is None and self.shared_experts is not None:
            result = result + self.shared_experts(x)
        sw.publish()
        return result
