"""Fail-closed behaviour of the decode paths: device status bits reach the
caller as the reference's exceptions (IndexError for an out-of-range expert,
glm53_flash_mlx/packed.py:868-876; RuntimeError for a wait that gave up),
a decode step refuses to run on weights whose identity changed
(native_execution/native_packed_moe_plan.cpp:270-272), and a bounded peer wait
that nothing satisfies runs out, reports GLM53_STATUS_WAIT_TIMEOUT and returns.
"""

import ctypes
import time

import numpy as np
import pytest
import torch


class _FixedGate(torch.nn.Module):
    """A gate returning fixed routes (optionally with an out-of-range id)."""

    def __init__(self, ids, scores):
        super().__init__()
        self.ids, self.scores = ids, scores

    def forward(self, x):
        T = x.reshape(-1, x.shape[-1]).shape[0]
        return self.ids[:T].reshape(*x.shape[:-1], -1), self.scores[:T].reshape(*x.shape[:-1], -1)


def _step_without_device(module):
    """A PackedDecodeStep's binding records, built without a device: the
    identity check is host logic."""
    from glm53_flash_mlx_b200.packed import PackedDecodeStep

    step = PackedDecodeStep.__new__(PackedDecodeStep)
    step._bound = PackedDecodeStep._bound_tensors(module)
    step._identity = PackedDecodeStep._identities(step._bound)
    step._slots = PackedDecodeStep._binding_slots(module)
    return step


def _cpu_layer():
    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.packed import PackedFP8MoE
    from glm53_flash_mlx_b200.router import Float32Gate

    H, I, E = 256, 128, 8
    bank = S.make_bank(E, H, I, seed=1, device="cpu")
    cfg = S.moe_config(H, I, E, 8, 10.0)
    return PackedFP8MoE(bank, cfg, Float32Gate(cfg, device="cpu"), S.make_shared(H, I, seed=2, device="cpu"))


def test_decode_step_refuses_a_swapped_bank():
    from glm53_flash_mlx_b200 import synthetic as S

    module = _cpu_layer()
    step = _step_without_device(module)
    step._check_bound()  # unchanged: accepted
    module.bank = S.make_bank(8, 256, 128, seed=9, device="cpu")
    with pytest.raises(RuntimeError, match="identity changed"):
        step._check_bound()


@pytest.mark.parametrize("change", ["inplace", "buffer", "data", "router", "shared"])
def test_decode_step_refuses_changed_weights(change):
    module = _cpu_layer()
    step = _step_without_device(module)
    if change == "inplace":
        module.bank.down_weight[0, 0, 0] ^= 1
    elif change == "buffer":
        module.bank.gate_up_scale_inv = module.bank.gate_up_scale_inv.clone()
    elif change == "data":
        w = module.bank.gate_up_weight
        w.data = w.data.clone()
    elif change == "router":
        module.gate.e_score_correction_bias.add_(1.0)
    else:
        module.shared_experts.down_proj.weight = module.shared_experts.down_proj.weight.clone()
    with pytest.raises(RuntimeError, match="identity changed"):
        step._check_bound()


def test_wait_limit_range_is_checked():
    from glm53_flash_mlx_b200 import _native as N

    lib = N.load_library()
    assert lib.glm53_set_wait_limit_ns(10) == N.GLM53_ERR_INVALID
    assert lib.glm53_set_wait_limit_ns(61 * 10**9) == N.GLM53_ERR_INVALID
    assert lib.glm53_set_wait_limit_ns(50 * 10**6) == N.GLM53_OK
    assert lib.glm53_set_wait_limit_ns(0) == N.GLM53_OK  # default again


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [1, 3, 40])
def test_bad_expert_id_raises_at_the_next_call(rows):
    """An out-of-range expert id sets a status bit on the device (no trap).
    Without any synchronisation in the call, the next call of the layer raises
    IndexError; the word is then clear and the layer computes again."""
    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.grouped_fp8 import SortedGroupedFP8MoE

    dev = torch.device("cuda", 0)
    E, H, I = 16, 512, 256
    bank = S.make_bank(E, H, I, seed=3, device=dev)
    cfg = S.moe_config(H, I, E, 8, 10.0)
    good = torch.stack([torch.randperm(E)[:8] for _ in range(rows)]).to(torch.int32).to(dev)
    bad = good.clone()
    bad[rows // 2, 3] = E + 7
    sc = torch.full((rows, 8), 0.125, device=dev)
    shared = S.make_shared(H, I, seed=4, device=dev)
    x = S.random_bf16((rows, H), seed=5, device=dev)
    layer = SortedGroupedFP8MoE(bank, cfg, _FixedGate(bad, sc), shared, min_routes=256)
    layer(x)  # returns; the bit is set on the device
    torch.cuda.synchronize()
    with pytest.raises(IndexError):
        layer(x)
    layer.gate = _FixedGate(good, sc)
    y = layer(x)
    layer.check_status()  # clean
    assert torch.isfinite(y.float()).all()


@pytest.mark.gpu
def test_decode_step_raises_for_bad_routes_and_changed_weights():
    """PackedDecodeStep: the status bits of a step are mirrored into pinned host
    memory by the next step's first kernel and raised there; replacing a bound
    weight makes the next step refuse to run."""
    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.packed import PackedFP8MoE
    from glm53_flash_mlx_b200.router import Float32Gate

    dev = torch.device("cuda", 0)
    E, H, I = 16, 512, 256
    cfg = S.moe_config(H, I, E, 8, 10.0)
    gate = Float32Gate(cfg, device=dev)
    w, b = S.make_router(E, H, seed=6, device=dev)
    gate.weight.copy_(w)
    gate.e_score_correction_bias.copy_(b)
    layer = PackedFP8MoE(S.make_bank(E, H, I, seed=7, device=dev), cfg, gate, S.make_shared(H, I, seed=8, device=dev))
    step = layer.capture_decode()
    x = S.random_bf16((1, 1, H), seed=9, device=dev).cpu().pin_memory()
    out = torch.empty((1, 1, H), dtype=torch.bfloat16).pin_memory()
    step(x, out=out)
    step.check()
    # a fail-closed bit as a kernel would set it: raised at the following step
    layer.status.view(torch.int32)[0] = 1
    step(x, out=out)  # its first kernel mirrors the bit
    torch.cuda.synchronize()
    with pytest.raises(IndexError):
        step(x, out=out)
    step(x, out=out)
    step.check()
    layer.bank.gate_up_weight[0, 0, 0] ^= 1  # an in-place write to a bound weight
    with pytest.raises(RuntimeError, match="identity changed"):
        step(x, out=out)


@pytest.mark.gpu
def test_peer_waits_run_out_when_a_rank_never_dispatches():
    """Two virtual ranks on one GPU with peer-memory buffers; rank 1 never
    dispatches.  Rank 0's owner decode waits for rank 1's slots and its combine
    for rank 1's rows: with a 20 ms bound both waits run out, set
    GLM53_STATUS_WAIT_TIMEOUT and return (every access stays inside the two
    zero-filled buffers), and the device stays usable."""
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.packed import StatusWord

    dev = torch.device("cuda", 0)
    lib = N.lib()
    world, E, H, I, T, top_k = 2, 16, 256, 128, 1, 8
    cap = T * top_k
    bank = S.make_bank(E // world, H, I, seed=10, device=dev)  # rank 0's experts 0..7
    nbytes = lib.glm53_ep_shared_bytes(world, cap, H)
    bufs = []
    for _ in range(world):
        p = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        N.check(lib.glm53_ep_buffer_alloc(nbytes, ctypes.byref(p), handle), "alloc")
        bufs.append(p.value)
    try:
        peer_base = torch.tensor(np.array(bufs, dtype=np.uint64).view(np.int64), device=dev)
        x = S.random_bf16((T, H), seed=11, device=dev)
        ids = torch.tensor([[0, 9, 2, 11, 4, 13, 6, 15]], dtype=torch.int32, device=dev)  # both owners
        sc = torch.full((T, top_k), 0.125, device=dev)
        slot_route = torch.zeros(world * cap, dtype=torch.int32, device=dev)
        slot_scores = torch.zeros(world * cap, dtype=torch.float32, device=dev)
        route_pos = torch.zeros(T * top_k, dtype=torch.int32, device=dev)
        ws = torch.zeros(lib.glm53_routes_decode_workspace_bytes(world * cap, H, I), dtype=torch.uint8, device=dev)
        shared_rows = torch.zeros((T, H), dtype=torch.bfloat16, device=dev)
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        sw = StatusWord(dev)
        flags = N.decode_flags(bank.gate_up_weight, bank.down_weight)
        st = N.stream(dev)
        N.check(lib.glm53_set_wait_limit_ns(20 * 10**6), "wait limit")
        torch.cuda.synchronize()
        t0 = time.monotonic()
        N.check(lib.glm53_ep_dispatch_p2p(x.data_ptr(), T, H, ids.data_ptr(), sc.data_ptr(), top_k, E, world, 0, cap,
                                          peer_base.data_ptr(), slot_route.data_ptr(), slot_scores.data_ptr(),
                                          route_pos.data_ptr(), sw.word.data_ptr(), st), "dispatch")
        N.check(lib.glm53_ep_owner_decode_p2p(bufs[0], H, world, cap, 0, bank.gate_up_weight.data_ptr(),
                                              bank.gate_up_scale_inv.data_ptr(), bank.down_weight.data_ptr(),
                                              bank.down_scale_inv.data_ptr(), bank.expert_count, I, x.data_ptr(), 0,
                                              None, None, None, None, None, None, 0, shared_rows.data_ptr(), 10.0,
                                              peer_base.data_ptr(), ws.data_ptr(), ws.numel(), sw.word.data_ptr(),
                                              flags, st), "owner decode")
        N.check(lib.glm53_ep_combine_p2p(bufs[0], route_pos.data_ptr(), slot_scores.data_ptr(), T, top_k, H, world,
                                         cap, None, out.data_ptr(), sw.word.data_ptr(), st), "combine")
        sw.publish()
        torch.cuda.synchronize()
        elapsed = time.monotonic() - t0
        assert int(sw.host[0]) & N.STATUS_WAIT_TIMEOUT
        assert elapsed < 1.5, f"the 20 ms bound did not apply ({elapsed:.3f} s)"
        with pytest.raises(RuntimeError, match="bounded device wait"):
            sw.raise_pending()
        assert int(sw.word[0].item()) == 0 and int(sw.host[0]) == 0
    finally:
        lib.glm53_set_wait_limit_ns(0)
        torch.cuda.synchronize()
        for p in bufs:
            lib.glm53_ep_buffer_free(p)
    # the context is still usable: a decode on the same device is exact
    from glm53_flash_mlx_b200.packed import packed_decode_moe

    xs = S.random_bf16((H,), seed=12, device=dev)
    good = torch.arange(8, dtype=torch.int32, device=dev)
    y1 = packed_decode_moe(xs, good, torch.full((8,), 0.125, device=dev), bank, None, limit=10.0)
    y2 = packed_decode_moe(xs, good, torch.full((8,), 0.125, device=dev), bank, None, limit=10.0)
    assert torch.equal(y1, y2) and torch.isfinite(y1.float()).all()
