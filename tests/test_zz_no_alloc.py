"""glm53_packed_decode_moe_static_scratch: the packed decode entry point that
allocates nothing, checked through the C-ABI against glm53_packed_decode_moe
(caller-provided workspace) on consecutive calls.  The file name makes pytest
collect it last, so it also runs after every other GPU test in one process."""

import ctypes

import pytest
import torch

from gpu_util import assert_layer_close, bits


def _shared_ptrs(N, shared):
    if shared is None:
        return [None] * 6, 0
    return [N.ptr(t) for t in shared], shared[0].shape[0]


def _call_static(N, bank, shared, x, ids, sc, limit, out, status, flags):
    sp, Is = _shared_ptrs(N, shared)
    return N.lib().glm53_packed_decode_moe_static_scratch(
        x.data_ptr(), x.numel(), ids.data_ptr(), sc.data_ptr(), ids.numel(),
        bank.gate_up_weight.data_ptr(), bank.gate_up_scale_inv.data_ptr(),
        bank.down_weight.data_ptr(), bank.down_scale_inv.data_ptr(), bank.expert_count, bank.intermediate_size,
        *sp, Is, float(limit), out.data_ptr(), status.data_ptr(), flags, N.stream(x.device),
    )


def _call_workspace(N, bank, shared, x, ids, sc, limit, out, status, flags):
    sp, Is = _shared_ptrs(N, shared)
    nbytes = N.lib().glm53_packed_decode_workspace_bytes(ids.numel(), x.numel(), bank.intermediate_size, Is)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=x.device)
    rc = N.lib().glm53_packed_decode_moe(
        x.data_ptr(), x.numel(), ids.data_ptr(), sc.data_ptr(), ids.numel(),
        bank.gate_up_weight.data_ptr(), bank.gate_up_scale_inv.data_ptr(),
        bank.down_weight.data_ptr(), bank.down_scale_inv.data_ptr(), bank.expert_count, bank.intermediate_size,
        *sp, Is, float(limit), out.data_ptr(), ws.data_ptr(), nbytes, status.data_ptr(), flags, N.stream(x.device),
    )
    return rc, ws


@pytest.mark.gpu
@pytest.mark.parametrize("E,H,I,limit,with_shared", [(16, 4096, 1536, 10.0, True), (8, 257, 129, 3.0, False)])
def test_static_scratch_decode_matches_workspace_decode(E, H, I, limit, with_shared):
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    dev = torch.device("cuda", 0)
    bank = S.make_bank(E, H, I, seed=E + H, device=dev)
    shared = shared_fp8_tensors(S.make_shared(H, I, seed=5, limit=limit, device=dev)) if with_shared else None
    weights = [bank.gate_up_weight, bank.down_weight] + ([shared[0], shared[2], shared[4]] if shared else [])
    flags = N.decode_flags(*weights)
    gen = torch.Generator().manual_seed(H)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for call in range(2):
        ids = torch.randperm(E, generator=gen)[:8].to(torch.int32).to(dev)
        sc = (torch.rand(8, generator=gen) * 0.25 + 0.05).to(dev)
        x = S.random_bf16((H,), seed=call, device=dev, std=2.0)
        out_s = torch.empty(H, dtype=torch.bfloat16, device=dev)
        out_w = torch.empty(H, dtype=torch.bfloat16, device=dev)
        assert _call_static(N, bank, shared, x, ids, sc, limit, out_s, status, flags) == 0, N.lib().glm53_last_error()
        rc, _ = _call_workspace(N, bank, shared, x, ids, sc, limit, out_w, status, flags)
        assert rc == 0, N.lib().glm53_last_error()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert_layer_close(bits(out_s), bits(out_w))
        # the same kernels run on the same values: the results are bit-identical
        assert torch.equal(out_s, out_w), f"call {call}"


@pytest.mark.gpu
def test_static_scratch_recovers_after_a_rejected_expert():
    """A call that flags an out-of-range expert id (status bit, no trap) is
    followed by a correct call: the scratch counters are cleared per call."""
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200 import synthetic as S

    dev = torch.device("cuda", 0)
    E, H, I = 8, 256, 128
    bank = S.make_bank(E, H, I, seed=3, device=dev)
    flags = N.decode_flags(bank.gate_up_weight, bank.down_weight)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    x = S.random_bf16((H,), seed=9, device=dev)
    sc = torch.full((8,), 0.125, device=dev)
    bad = torch.tensor([0, 1, 2, 3, 4, 5, 6, 99], dtype=torch.int32, device=dev)
    out = torch.empty(H, dtype=torch.bfloat16, device=dev)
    assert _call_static(N, bank, None, x, bad, sc, 3.0, out, status, flags) == 0
    torch.cuda.synchronize()
    assert int(status.item()) & N.STATUS_BAD_EXPERT
    status.zero_()
    good = torch.arange(8, dtype=torch.int32, device=dev)
    out_w = torch.empty(H, dtype=torch.bfloat16, device=dev)
    assert _call_static(N, bank, None, x, good, sc, 3.0, out, status, flags) == 0
    assert _call_workspace(N, bank, None, x, good, sc, 3.0, out_w, status, flags)[0] == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(out, out_w)


def test_static_scratch_rejects_sizes_beyond_the_fixed_maximum():
    """Host-side check, made before any CUDA call (runs without a GPU)."""
    from glm53_flash_mlx_b200 import _native as N

    lib = N.load_library()
    H, I, top_k = 65536, 1536, 8
    need = lib.glm53_packed_decode_workspace_bytes(top_k, H, I, I)
    assert need > (1 << 20)
    fake = ctypes.c_void_p(256)  # never dereferenced: the call is rejected first
    rc = lib.glm53_packed_decode_moe_static_scratch(
        fake, H, fake, fake, top_k, fake, fake, fake, fake, 16, I, fake, fake, fake, fake, fake, fake, I, 10.0,
        fake, fake, 0, None)
    assert rc == N.GLM53_ERR_INVALID
    msg = lib.glm53_last_error().decode()
    assert "fixed maximum" in msg and str(need) in msg


def test_static_scratch_rejects_the_after_router_flag():
    """The scratch counters are cleared by a stream operation before the decode,
    so the decode cannot be launched as the router's programmatic dependent:
    GLM53_FLAG_AFTER_ROUTER is refused (before any CUDA call) instead of being
    dropped silently."""
    from glm53_flash_mlx_b200 import _native as N

    lib = N.load_library()
    H, I, top_k = 4096, 1536, 8
    fake = ctypes.c_void_p(256)  # never dereferenced: the call is rejected first
    rc = lib.glm53_packed_decode_moe_static_scratch(
        fake, H, fake, fake, top_k, fake, fake, fake, fake, 16, I, fake, fake, fake, fake, fake, fake, I, 10.0,
        fake, fake, N.FLAG_AFTER_ROUTER | N.FLAG_E4M3_FINITE, None)
    assert rc == N.GLM53_ERR_INVALID
    assert "GLM53_FLAG_AFTER_ROUTER" in lib.glm53_last_error().decode()
