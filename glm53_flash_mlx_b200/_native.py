"""ctypes binding of the sm_100a C-ABI library (``include/glm53_b200.h``).

The library is built in-tree by ``glm53_flash_mlx_b200.build`` into
``_lib/libglm53_b200.so``.  There is no fallback: every operator raises
``RuntimeError`` when the library is missing or no CUDA device is present,
mirroring the reference's fail-closed ``RuntimeError`` when Metal is absent
(glm53_flash_mlx/fp8.py:256-257).
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libglm53_b200.so"

GLM53_OK = 0
GLM53_ERR_INVALID = 1
GLM53_ERR_CUDA = 2
GLM53_ERR_INDEX = 3

FLAG_E4M3_FINITE = 1
FLAG_SHARED_ONLY = 2
FLAG_SKIP_SHARED = 4
FLAG_AFTER_ROUTER = 8
FLAG_F8_MMA = 16

STATUS_BAD_EXPERT = 1
STATUS_WAIT_TIMEOUT = 2
STATUS_BAD_GEOMETRY = 4

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t
_u32 = ctypes.c_uint32

# name -> (restype, argtypes); mirrors include/glm53_b200.h
SIGNATURES: dict[str, tuple] = {
    "glm53_kernel_abi": (ctypes.c_char_p, []),
    "glm53_last_error": (ctypes.c_char_p, []),
    "glm53_fp8_linear": (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _vp, _u32, _vp]),
    "glm53_e4m3_scan": (_int, [_vp, _i64, _vp, _vp]),
    "glm53_graph_step": (_int, [_vp, _vp, _vp, _sz, _vp, _vp, _sz, _vp]),
    "glm53_router_workspace_bytes": (_sz, [_i64, _i64]),
    "glm53_router_topk": (
        _int,
        [_vp, _i64, _i64, _vp, _i64, _vp, _int, _int, _int, _int, _f, _vp, _vp, _vp, _vp, _sz, _vp],
    ),
    "glm53_fp8_linear_workspace_bytes": (_sz, [_i64, _i64]),
    "glm53_fp8_linear_splitk_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "glm53_fp8_linear_ws": (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _sz, _vp, _u32, _vp]),
    "glm53_packed_decode_workspace_bytes": (_sz, [_int, _i64, _i64, _i64]),
    "glm53_packed_decode_moe": (
        _int,
        [_vp, _i64, _vp, _vp, _int, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _f,
         _vp, _vp, _sz, _vp, _u32, _vp],
    ),
    "glm53_packed_decode_moe_static_scratch": (
        _int,
        [_vp, _i64, _vp, _vp, _int, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _f,
         _vp, _vp, _u32, _vp],
    ),
    "glm53_packed_decode_moe_hc": (
        _int,
        [_vp, _i64, _vp, _vp, _int, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _f,
         _vp, _vp, _vp, _vp, _vp, _sz, _vp, _u32, _vp],
    ),
    "glm53_selected_decode_moe": (
        _int,
        [_vp, _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _f,
         _vp, _vp, _sz, _vp, _u32, _vp],
    ),
    "glm53_direct_combine": (_int, [_vp, _vp, _vp, _i64, _int, _i64, _vp, _vp, _vp]),
    "glm53_batched_decode_workspace_bytes": (_sz, [_i64, _int, _i64, _i64, _i64]),
    "glm53_batched_decode_shared_workspace_bytes": (_sz, [_i64, _int, _i64, _i64, _i64]),
    "glm53_batched_decode_moe_shared": (
        _int,
        [_vp, _i64, _i64, _vp, _vp, _int, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _f, _vp, _vp,
         _sz, _vp, _u32, _vp],
    ),
    "glm53_batched_decode_moe": (
        _int,
        [_vp, _i64, _i64, _vp, _vp, _int, _vp, _vp, _vp, _vp, _i64, _i64, _f, _vp, _vp, _vp, _sz, _vp, _u32, _vp],
    ),
    "glm53_routes_decode_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "glm53_routes_decode_coalesced_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "glm53_routes_decode_coalesced": (
        _int,
        [_vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f, _vp, _vp, _sz, _vp, _u32, _vp],
    ),
    "glm53_routes_decode": (
        _int,
        [_vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f, _vp, _vp, _sz, _vp, _u32, _vp],
    ),
    "glm53_ep_dispatch_pack": (
        _int,
        [_vp, _i64, _i64, _vp, _vp, _int, _i64, _int, _i64, _vp, _vp, _vp, _vp, _vp, _vp],
    ),
    "glm53_ep_combine": (_int, [_vp, _vp, _vp, _i64, _int, _i64, _vp, _vp, _vp]),
    "glm53_ep_shared_bytes": (_sz, [_int, _i64, _i64]),
    "glm53_ep_buffer_alloc": (_int, [_sz, _vp, _vp]),
    "glm53_ep_buffer_free": (_int, [_vp]),
    "glm53_ep_ipc_open": (_int, [_vp, _vp]),
    "glm53_ep_ipc_close": (_int, [_vp]),
    "glm53_ep_dispatch_p2p": (
        _int,
        [_vp, _i64, _i64, _vp, _vp, _int, _i64, _int, _int, _i64, _vp, _vp, _vp, _vp, _vp, _vp],
    ),
    "glm53_ep_owner_decode_p2p": (
        _int,
        [_vp, _i64, _int, _i64, _int, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp,
         _i64, _vp, _f, _vp, _vp, _sz, _vp, _u32, _vp],
    ),
    "glm53_ep_combine_p2p": (_int, [_vp, _vp, _vp, _i64, _int, _i64, _int, _i64, _vp, _vp, _vp, _vp]),
    "glm53_packed_decode_gate_up": (
        _int,
        [_vp, _i64, _vp, _int, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _f, _vp, _sz, _vp, _u32, _vp],
    ),
    "glm53_route_plan": (
        _int,
        [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    ),
    "glm53_gather_rows": (_int, [_vp, _i64, _vp, _i64, _int, _vp, _vp]),
    "glm53_grouped_fp8_linear": (
        _int,
        [_vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _vp, _vp, _u32, _vp],
    ),
    "glm53_grouped_fp8_linear_workspace_bytes": (_sz, [_i64, _i64]),
    "glm53_grouped_fp8_linear_ws": (
        _int,
        [_vp, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _sz, _vp, _u32, _vp],
    ),
    "glm53_activate_gate_up": (_int, [_vp, _i64, _i64, _f, _vp, _vp]),
    "glm53_restore_and_reduce": (_int, [_vp, _vp, _vp, _i64, _int, _i64, _vp, _vp, _vp]),
    "glm53_grouped_moe_workspace_bytes": (_sz, [_i64, _int, _i64, _i64, _i64, _i64]),
    "glm53_grouped_moe": (
        _int,
        [_vp, _i64, _i64, _vp, _vp, _int, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp,
         _i64, _f, _vp, _vp, _sz, _vp, _u32, _vp],
    ),
    "glm53_sigmoid_bf16": (_int, [_vp, _i64, _vp, _vp]),
    "glm53_decode_step_host": (_int, [_vp, _vp, _vp, _vp]),
    "glm53_status_mirror": (_int, [_vp, _vp, _vp]),
    "glm53_packed_decode_workspace_layout": (_int, [_int, _i64, _i64, _i64, _vp]),
    "glm53_grouped_moe_workspace_layout": (_int, [_i64, _int, _i64, _i64, _i64, _i64, _vp]),
    "glm53_grouped_moe_term_layout": (_int, [_i64, _int, _i64, _i64, _i64, _i64, _vp]),
    "glm53_e4m3_split_rows": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "glm53_set_wait_limit_ns": (_int, [ctypes.c_ulonglong]),
    "glm53_hc_collapse_workspace_bytes": (_sz, [_i64, _i64]),
    "glm53_hc_collapse_norm": (
        _int,
        [_vp, _i64, _i64, _int, _vp, _vp, _vp, _int, _f, _f, _vp, _f, _vp, _vp, _vp, _vp, _vp, _sz, _vp],
    ),
    "glm53_rms_norm": (_int, [_vp, _i64, _i64, _vp, _f, _vp, _vp]),
    "glm53_hc_expand": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _int, _vp, _vp]),
    "glm53_head_major_to_rows": (_int, [_vp, _i64, _i64, _i64, _vp, _vp]),
}


class DecodeStepDesc(ctypes.Structure):
    """glm53_decode_step_desc (include/glm53_b200.h), field for field."""

    _fields_ = [
        ("H", _i64), ("E", _i64), ("I", _i64), ("I_shared", _i64),
        ("top_k", _int), ("n_group", _int), ("topk_group", _int), ("norm_topk_prob", _int),
        ("routed_scaling_factor", _f), ("limit", _f), ("flags", _u32),
        ("router_w", _vp), ("router_bias", _vp),
        ("gate_up_w", _vp), ("gate_up_s", _vp), ("down_w", _vp), ("down_s", _vp),
        ("shared_gate_w", _vp), ("shared_gate_s", _vp), ("shared_up_w", _vp), ("shared_up_s", _vp),
        ("shared_down_w", _vp), ("shared_down_s", _vp),
        ("x", _vp), ("expert_ids", _vp), ("scores", _vp), ("out", _vp),
        ("router_workspace", _vp), ("router_workspace_bytes", _sz),
        ("decode_workspace", _vp), ("decode_workspace_bytes", _sz),
        ("status", _vp), ("status_host", _vp),
    ]

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load_library(path: Path | None = None) -> ctypes.CDLL:
    """Load the C-ABI library (no CUDA device needed to load it)."""
    global _lib
    with _lock:
        if _lib is None or path is not None:
            p = Path(path) if path is not None else LIB_PATH
            if not p.exists():
                raise RuntimeError(
                    f"GLM-5.3 B200 CUDA extension not built ({p} missing); run "
                    "`python -m glm53_flash_mlx_b200.build`"
                )
            lib = ctypes.CDLL(str(p))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if path is not None:
                return lib
            _lib = lib
    return _lib


def lib() -> ctypes.CDLL:
    """The library, for a CUDA device: raises RuntimeError otherwise."""
    if not torch.cuda.is_available():
        raise RuntimeError("direct GLM-5.3 FP8 execution requires the CUDA (sm_100a) backend")
    return load_library()


def kernel_abi() -> str:
    return load_library().glm53_kernel_abi().decode()


def check(rc: int, what: str) -> None:
    if rc == GLM53_OK:
        return
    msg = (load_library().glm53_last_error() or b"").decode() or what
    if rc == GLM53_ERR_INVALID:
        raise ValueError(msg)
    if rc == GLM53_ERR_INDEX:
        raise IndexError(msg)
    raise RuntimeError(msg)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream(device: torch.device | None = None) -> int:
    """The current CUDA stream of `device` as a raw handle."""
    if _raw_stream is not None and isinstance(device, torch.device) and device.index is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    lib()
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("direct GLM-5.3 FP8 execution requires CUDA tensors")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


_finite_cache: dict[tuple, bool] = {}


def e4m3_finite(*weights: torch.Tensor) -> bool:
    """True when none of the E4M3 weight tensors holds code 0x7F or 0xFF:
    GLM53_FLAG_E4M3_FINITE may be used.  One device pass per tensor at first
    use; the answer is cached per (storage, shape, version), so an in-place
    write to a weight triggers a new scan."""
    dev = require_cuda(*weights)
    ok = True
    for w in weights:
        key = (w.data_ptr(), tuple(w.shape), w._version, w.device.index)
        hit = _finite_cache.get(key)
        if hit is None:
            wc = w.contiguous()
            count = torch.zeros(1, dtype=torch.int32, device=dev)
            check(lib().glm53_e4m3_scan(wc.data_ptr(), wc.numel(), count.data_ptr(), stream(dev)),
                  "glm53_e4m3_scan")
            hit = int(count.item()) == 0
            if len(_finite_cache) > 4096:
                _finite_cache.clear()
            _finite_cache[key] = hit
        ok = ok and hit
    return ok


def decode_flags(*weights: torch.Tensor) -> int:
    return FLAG_E4M3_FINITE if e4m3_finite(*weights) else 0


def e4m3_scanned(*weights: torch.Tensor) -> bool:
    """True when e4m3_finite(*weights) answers from its cache (no device pass)."""
    return all((w.data_ptr(), tuple(w.shape), w._version, w.device.index) in _finite_cache for w in weights)


class Workspace:
    """Per-device, grow-only, zero-initialised scratch buffers owned by a plan.

    Addresses are stable until a larger size is requested (the reference's
    plan-owned scratch rule, glm53_flash_mlx/native_execution.py:141-165)."""

    def __init__(self) -> None:
        self._buffers: dict[tuple, torch.Tensor] = {}

    def has(self, device: torch.device, key: str, nbytes: int) -> bool:
        """True when get() would return an existing buffer (no allocation)."""
        buf = self._buffers.get((device, key))
        return buf is not None and buf.numel() >= nbytes

    def get(self, device: torch.device, key: str, nbytes: int) -> torch.Tensor:
        k = (device, key)
        buf = self._buffers.get(k)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)
            self._buffers[k] = buf
        return buf
