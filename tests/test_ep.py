"""Expert-parallel decode: the dispatch layout, the protocol over a process
group, and the CUDA path through the C-ABI.

CPU tests run the protocol as gloo ranks with the oracle computing each
owner's per-route rows; the result must be bit-identical to the one-device
packed decode.  GPU tests compare the dispatch kernel with the host layout and
run the whole expert-parallel decode (as virtual ranks on one GPU, and over
NCCL when two GPUs are present) against glm53_packed_decode_moe bit for bit.
"""

import os
import socket

import numpy as np
import pytest
import torch

from glm53_flash_mlx_b200 import ep


def test_expert_partition_and_layout():
    assert ep.expert_range(0, 8, 288) == (0, 36)
    assert ep.expert_range(7, 8, 288) == (252, 288)
    assert [ep.owner_of(e, 4, 288) for e in (0, 71, 72, 287)] == [0, 0, 1, 3]
    with pytest.raises(ValueError):
        ep.expert_range(0, 5, 288)
    ids = np.array([[5, 0, 7, 2], [1, 6, 3, 4]], dtype=np.uint32)  # E=8, world=2: experts 0-3 | 4-7
    send, pos = ep.plan_slots(ids, 8, 2, capacity=8)
    # destination 0 gets routes 1, 3, 4, 6 (experts 0, 2, 1, 3) in route order
    assert send[:4].tolist() == [0, 2, 1, 3] and (send[4:8] == ep.EMPTY_SLOT).all()
    # destination 1 gets routes 0, 2, 5, 7 (experts 5, 7, 6, 4 -> local 1, 3, 2, 0)
    assert send[8:12].tolist() == [1, 3, 2, 0]
    assert pos.tolist() == [8, 0, 9, 1, 2, 10, 3, 11]
    # a full destination drops routes in route order
    send, pos = ep.plan_slots(np.array([4, 5, 6, 7], dtype=np.uint32), 8, 2, capacity=2)
    assert pos.tolist() == [2, 3, ep.EMPTY_SLOT, ep.EMPTY_SLOT]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, case, result_dir):
    """One rank of the expert-parallel protocol on CPU: the oracle plays the
    kernels, gloo carries the two all-to-alls."""
    import torch.distributed as dist

    import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x_all, ids_all, sc_all, bank, shared, limit = case
        E = bank[0].shape[0]
        H = x_all.shape[1]
        T = x_all.shape[0] // world  # tokens per home rank
        x, ids, sc = x_all[rank * T:(rank + 1) * T], ids_all[rank * T:(rank + 1) * T], sc_all[rank * T:(rank + 1) * T]
        top_k = ids.shape[1]
        cap = T * top_k
        send_e, pos = ep.plan_slots(ids, E, world, cap)
        send_x = np.zeros((world * cap, H), dtype=np.uint16)
        for r, p in enumerate(pos.tolist()):
            if p != ep.EMPTY_SLOT:
                send_x[p] = x[r // top_k]
        # gloo carries 32-bit words: two BF16 values per word
        recv_x = torch.empty((world * cap, H // 2), dtype=torch.int32)
        recv_e = torch.empty(world * cap, dtype=torch.int64)
        dist.all_to_all_single(recv_x, torch.from_numpy(send_x.view(np.int32)))
        dist.all_to_all_single(recv_e, torch.from_numpy(send_e.astype(np.int64)))
        lo, hi = ep.expert_range(rank, world, E)
        local = tuple(t[lo:hi] for t in bank)
        rows = np.zeros((world * cap, H), dtype=np.uint16)
        for s, e in enumerate(recv_e.numpy().tolist()):
            if e != ep.EMPTY_SLOT:  # one route: BF16(1.0 * bf16(down)) = its BF16 down row
                rows[s] = O.packed_decode_moe(recv_x[s].numpy().view(np.uint16), np.array([e], np.uint32),
                                              np.array([1.0], np.float32), local, None, limit)
        back = torch.empty((world * cap, H // 2), dtype=torch.int32)
        dist.all_to_all_single(back, torch.from_numpy(rows.view(np.int32)))
        back = back.numpy().view(np.uint16)
        out = np.zeros((T, H), dtype=np.uint16)
        for t in range(T):
            sh = O.packed_decode_moe(x[t], np.zeros(0, np.uint32), np.zeros(0, np.float32), bank, shared, limit) \
                if shared is not None else None
            total = np.zeros(H, dtype=np.float32)
            for j in range(top_k):
                p = pos[t * top_k + j]
                row = O.f32_from_bf16(back[p])
                total = (total + row * np.float32(sc[t, j])).astype(np.float32)
            res = O.f32_from_bf16(O.bf16_from_f32(total))
            if sh is not None:
                res = (res + O.f32_from_bf16(sh)).astype(np.float32)
            out[t] = O.bf16_from_f32(res)
        np.save(os.path.join(result_dir, f"out{rank}.npy"), out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_protocol_is_bit_identical_on_gloo(oracle, tmp_path, world):
    """gloo ranks on CPU (the oracle playing the kernels) carry the dispatch
    and combine all-to-alls; every rank's tokens equal the one-device MoE."""
    import torch.multiprocessing as mp

    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    E, H, I, T = 8, 256, 128, 3
    bank_t = S.make_bank(E, H, I, seed=31)
    bank = tuple(t.numpy() for t in (bank_t.gate_up_weight, bank_t.gate_up_scale_inv, bank_t.down_weight,
                                      bank_t.down_scale_inv))
    shared = tuple(t.numpy() for t in shared_fp8_tensors(S.make_shared(H, I, seed=32, limit=3.0)))
    gen = np.random.default_rng(33)
    x = (S.random_bf16((world * T, H), seed=34, std=2.0).view(torch.int16).numpy().view(np.uint16))
    ids = np.stack([gen.permutation(E)[:8] for _ in range(world * T)]).astype(np.uint32)
    sc = gen.uniform(0.05, 0.3, (world * T, 8)).astype(np.float32)
    case = (x, ids, sc, bank, shared, 3.0)
    mp.start_processes(_gloo_rank, args=(world, _free_port(), case, str(tmp_path)), nprocs=world, start_method="spawn")
    got = np.concatenate([np.load(tmp_path / f"out{r}.npy") for r in range(world)])
    want = np.stack([oracle.packed_decode_moe(x[t], ids[t], sc[t], bank, shared, 3.0) for t in range(world * T)])
    assert np.array_equal(got, want)


# ---------------------------------------------------------------------------
# CUDA path
# ---------------------------------------------------------------------------


@pytest.mark.gpu
def test_dispatch_pack_matches_host_layout():
    from glm53_flash_mlx_b200 import _native as N

    dev = torch.device("cuda", 0)
    world, E, H, T, k = 4, 288, 256, 5, 8
    gen = np.random.default_rng(5)
    ids = np.stack([gen.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    ids[2, :] = np.arange(8)  # a token whose routes all go to rank 0
    sc = gen.uniform(0.0, 1.0, (T, k)).astype(np.float32)
    x = torch.randn((T, H), device=dev).to(torch.bfloat16)
    cap = T * k
    send_x = torch.zeros((world * cap, H), dtype=torch.bfloat16, device=dev)
    send_e = torch.zeros(world * cap, dtype=torch.int32, device=dev)
    slot_sc = torch.zeros(world * cap, dtype=torch.float32, device=dev)
    pos = torch.zeros(T * k, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    it = torch.from_numpy(ids.astype(np.int32)).to(dev)
    st = torch.from_numpy(sc).to(dev)
    N.check(N.lib().glm53_ep_dispatch_pack(x.data_ptr(), T, H, it.data_ptr(), st.data_ptr(), k, E, world, cap,
                                           send_x.data_ptr(), send_e.data_ptr(), slot_sc.data_ptr(), pos.data_ptr(),
                                           status.data_ptr(), N.stream(dev)), "pack")
    torch.cuda.synchronize()
    want_e, want_pos = ep.plan_slots(ids, E, world, cap)
    assert np.array_equal(send_e.cpu().numpy().view(np.uint32), want_e)
    assert np.array_equal(pos.cpu().numpy().view(np.uint32), want_pos)
    assert int(status.item()) == 0
    for r, p in enumerate(want_pos.tolist()):
        assert torch.equal(send_x[p], x[r // k])
        assert slot_sc[p].item() == sc.reshape(-1)[r]


def _single_device(bank, shared, x, ids, sc, limit):
    from glm53_flash_mlx_b200.packed import packed_decode_moe

    return torch.stack([packed_decode_moe(x[t], ids[t], sc[t], bank, shared, limit=limit) for t in range(x.shape[0])])


@pytest.mark.gpu
@pytest.mark.parametrize("world,E,H,I", [(4, 16, 4096, 1536), (2, 8, 256, 128)])
def test_expert_parallel_decode_virtual_ranks_bitwise(world, E, H, I):
    """All ranks in one process on one GPU; the all-to-alls are slicing."""
    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    dev = torch.device("cuda", 0)
    bank = S.make_bank(E, H, I, seed=41, device=dev)
    shared = shared_fp8_tensors(S.make_shared(H, I, seed=42, device=dev))
    T = 2  # tokens per rank
    gen = torch.Generator().manual_seed(43)
    x = S.random_bf16((world * T, H), seed=44, device=dev, std=2.0)
    ids = torch.stack([torch.randperm(E, generator=gen)[:8] for _ in range(world * T)]).to(torch.int32).to(dev)
    sc = (torch.rand((world * T, 8), generator=gen) * 0.25 + 0.05).to(dev)
    plans = [ep.ExpertParallelDecode(ep.local_bank(bank, r, world), experts=E, rank=r, world=world, shared=shared,
                                     limit=10.0, max_tokens=T, transport="nccl") for r in range(world)]
    outs = []
    # step by step across virtual ranks (each all-to-all = chunk transpose)
    from glm53_flash_mlx_b200 import _native as N

    lib = N.lib()
    st = N.stream(dev)
    cap = plans[0].capacity
    for r, p in enumerate(plans):
        xs, ii, ss = x[r * T:(r + 1) * T], ids[r * T:(r + 1) * T], sc[r * T:(r + 1) * T]
        N.check(lib.glm53_ep_dispatch_pack(xs.data_ptr(), T, H, ii.contiguous().data_ptr(), ss.contiguous().data_ptr(),
                                           8, E, world, cap, p.send_x.data_ptr(), p.send_e.data_ptr(),
                                           p.slot_scores.data_ptr(), p.route_pos.data_ptr(), p.status.data_ptr(), st),
                "pack")
    for d, p in enumerate(plans):  # rank d receives chunk d of every rank's send buffer
        p.recv_x.copy_(torch.cat([q.send_x[d * cap:(d + 1) * cap] for q in plans]))
        p.recv_e.copy_(torch.cat([q.send_e[d * cap:(d + 1) * cap] for q in plans]))
        ep.routes_decode(p.recv_x, p.recv_e, p.bank, limit=10.0, out=p.rows, workspace=p.workspace,
                         status=p.status)
    for r, p in enumerate(plans):
        p.back.copy_(torch.cat([q.rows[r * cap:(r + 1) * cap] for q in plans]))
        xs = x[r * T:(r + 1) * T]
        shared_rows = ep.routes_decode(xs, p.zero_ids[:T], p.shared_bank, limit=10.0)
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        N.check(lib.glm53_ep_combine(p.back.data_ptr(), p.route_pos.data_ptr(), p.slot_scores.data_ptr(), T, 8, H,
                                     shared_rows.data_ptr(), out.data_ptr(), st), "combine")
        outs.append(out)
    torch.cuda.synchronize()
    for p in plans:
        assert int(p.status.item()) == 0
    assert torch.equal(torch.cat(outs), _single_device(bank, shared, x, ids, sc, 10.0))


@pytest.mark.gpu
def test_expert_parallel_decode_world1_module_bitwise():
    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    dev = torch.device("cuda", 0)
    E, H, I = 16, 4096, 1536
    bank = S.make_bank(E, H, I, seed=51, device=dev)
    shared = shared_fp8_tensors(S.make_shared(H, I, seed=52, device=dev))
    plan = ep.ExpertParallelDecode(bank, experts=E, rank=0, world=1, shared=shared, limit=10.0, max_tokens=64)
    gen = torch.Generator().manual_seed(53)
    for T in (1, 4, 16, 64):  # 16 and 64: config 4's batches, the owner decode coalesced by expert
        x = S.random_bf16((T, H), seed=54 + T, device=dev)
        ids = torch.stack([torch.randperm(E, generator=gen)[:8] for _ in range(T)]).to(torch.int32).to(dev)
        sc = (torch.rand((T, 8), generator=gen) * 0.25 + 0.05).to(dev)
        out = plan(x, ids, sc)
        torch.cuda.synchronize()
        assert torch.equal(out, _single_device(bank, shared, x, ids, sc, 10.0))


@pytest.mark.gpu
def test_coalesced_routes_decode_equals_per_route_bitwise():
    """glm53_routes_decode_coalesced (slots sorted by expert, each expert's
    weights streamed once per four slots) gives every slot the bits of
    glm53_routes_decode; empty slots (id 0xFFFFFFFF) keep their rows."""
    from glm53_flash_mlx_b200 import synthetic as S

    dev = torch.device("cuda", 0)
    E, H, I, R = 24, 4096, 1536, 300
    bank = S.make_bank(E, H, I, seed=71, device=dev)
    tensors = (bank.gate_up_weight, bank.gate_up_scale_inv, bank.down_weight, bank.down_scale_inv)
    gen = torch.Generator().manual_seed(72)
    ids = torch.randint(0, E, (R,), generator=gen, dtype=torch.int32)
    ids[torch.randperm(R, generator=gen)[:60]] = -1  # 0xFFFFFFFF: empty slots
    ids = ids.to(dev)
    x = S.random_bf16((R, H), seed=73, device=dev, std=1.5)
    live = ids >= 0
    want = ep.routes_decode(x[live], ids[live].contiguous(), tensors, limit=10.0)
    sentinel = torch.full((R, H), 7.0, dtype=torch.bfloat16, device=dev)
    got = ep.routes_decode_coalesced(x, ids, tensors, limit=10.0, out=sentinel.clone())
    torch.cuda.synchronize()
    assert torch.equal(got[live], want)
    assert torch.equal(got[~live], sentinel[~live])


def _nccl_rank(rank, world, port, result_dir, transport):
    import torch.distributed as dist

    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.packed import packed_decode_moe, shared_fp8_tensors

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        E, H, I, T = 16, 4096, 1536, 2
        bank = S.make_bank(E, H, I, seed=61, device=dev)  # same seeds on every rank: identical full banks
        shared = shared_fp8_tensors(S.make_shared(H, I, seed=62, device=dev))
        gen = torch.Generator().manual_seed(63)
        x = S.random_bf16((world * T, H), seed=64, device=dev)
        ids = torch.stack([torch.randperm(E, generator=gen)[:8] for _ in range(world * T)]).to(torch.int32).to(dev)
        sc = (torch.rand((world * T, 8), generator=gen) * 0.25 + 0.05).to(dev)
        plan = ep.ExpertParallelDecode(ep.local_bank(bank, rank, world), experts=E, rank=rank, world=world,
                                       shared=shared, limit=10.0, max_tokens=T, transport=transport)
        ok = True
        for step in range(3):  # consecutive steps reuse the buffers and counters
            sl = slice(rank * T, (rank + 1) * T)
            xs = (x[sl] * (step + 1)).to(torch.bfloat16)
            out = plan(xs, ids[sl], sc[sl])
            want = torch.stack([packed_decode_moe(xs[t], ids[sl][t], sc[sl][t], bank, shared, limit=10.0)
                                for t in range(T)])
            torch.cuda.synchronize()
            ok = ok and bool(torch.equal(out, want))
        ok = ok and int(plan.status.item()) == 0
        plan.close()
        with open(os.path.join(result_dir, f"ok{rank}"), "w") as f:
            f.write("1" if ok else "0")
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("transport", ["nccl", "p2p"])
def test_expert_parallel_decode_gpus(tmp_path, transport, world):
    """One process per GPU: every rank's tokens through expert-parallel decode
    (3 consecutive steps) equal the one-GPU packed decode bit for bit."""
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_nccl_rank, args=(world, _free_port(), str(tmp_path), transport), nprocs=world,
                       start_method="spawn")
    assert [(tmp_path / f"ok{r}").read_text() for r in range(world)] == ["1"] * world
