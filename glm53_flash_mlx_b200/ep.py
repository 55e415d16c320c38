"""Expert-parallel decode MoE across the GPUs of one node.

One process per GPU.  Rank ``r`` of ``world`` holds the contiguous expert range
``expert_range(r, world, E)`` of every layer's bank (E / world experts), and a
full copy of the router and the shared expert; tokens stay on their home rank.
Per layer and decode step:

1. the home rank routes its tokens (``glm53_router_topk``);
2. ``glm53_ep_dispatch_pack`` places every route into ``capacity`` slots per
   destination rank (slots in route order) and an all-to-all of equal chunks
   delivers token rows and local expert ids to the owners;
3. each owner runs ``glm53_routes_decode`` on the slots it received (gate/up,
   SwiGLU, down: one BF16 row per route, the K7 + K6 arithmetic of the packed
   decode);
4. a second all-to-all returns the rows to their home slots;
5. ``glm53_ep_combine`` reduces them in slot order and adds the shared expert
   (computed at home with the same kernels).

Because every route's row is computed by the same kernels as the one-GPU
packed decode and reduced in the same order, the result is bit-identical for
every world size.  The reference runs this layer on one device only
(glm53_flash_mlx/packed.py:879-923); the partition, the fixed capacity and the
slot order are this package's design.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _native as N

EMPTY_SLOT = 0xFFFFFFFF


def expert_range(rank: int, world: int, experts: int) -> tuple[int, int]:
    """Experts [start, stop) owned by ``rank``: E / world contiguous ids."""
    if world < 1 or experts % world:
        raise ValueError(f"{experts} experts do not split evenly over {world} ranks")
    per = experts // world
    return rank * per, (rank + 1) * per


def owner_of(expert: int, world: int, experts: int) -> int:
    return int(expert) // (experts // world)


def plan_slots(indices: np.ndarray, experts: int, world: int, capacity: int):
    """Host statement of the dispatch layout that ``glm53_ep_dispatch_pack``
    builds on the device: returns ``(send_expert [world*capacity] uint32,
    route_pos [T*top_k] uint32)``.  Route r = t*top_k + j goes to the next free
    slot of its owner, in route order; a full destination drops the route
    (position ``EMPTY_SLOT``)."""
    ids = np.asarray(indices, dtype=np.uint32).reshape(-1)
    per = experts // world
    send = np.full(world * capacity, EMPTY_SLOT, dtype=np.uint32)
    pos = np.full(ids.size, EMPTY_SLOT, dtype=np.uint32)
    fill = [0] * world
    for r, e in enumerate(ids.tolist()):
        if e >= experts:
            continue
        d = e // per
        if fill[d] < capacity:
            p = d * capacity + fill[d]
            send[p] = e - d * per
            pos[r] = p
            fill[d] += 1
    return send, pos


def local_bank(bank, rank: int, world: int):
    """This rank's experts of a full bank, as a bank of borrowed-stable views
    (the full bank stays their owner)."""
    from .ownership import TensorLayout, borrowed_stable_tensor
    from .packed import PackedFP8ExpertBank

    lo, hi = expert_range(rank, world, bank.expert_count)
    lay = TensorLayout.ROW_MAJOR_CONTIGUOUS

    def view(t):
        return borrowed_stable_tensor(t[lo:hi], owner=bank, layout=lay)

    return PackedFP8ExpertBank(view(bank.gate_up_weight), view(bank.gate_up_scale_inv), view(bank.down_weight),
                               view(bank.down_scale_inv), intermediate_size=bank.intermediate_size)


def pack_shared_bank(shared) -> tuple[torch.Tensor, ...] | None:
    """The shared expert's six tensors as a one-expert bank (gate rows then up
    rows), so the per-route kernels run it like any routed expert."""
    if shared is None:
        return None
    sg_w, sg_s, su_w, su_s, sd_w, sd_s = shared
    gu_w = torch.cat([sg_w, su_w], dim=0).unsqueeze(0).contiguous()
    gu_s = torch.cat([sg_s, su_s], dim=0).unsqueeze(0).contiguous()
    return gu_w, gu_s, sd_w.unsqueeze(0).contiguous(), sd_s.unsqueeze(0).contiguous()


def routes_decode(x_rows: torch.Tensor, expert_ids: torch.Tensor, bank: tuple, *, limit: float,
                  out: torch.Tensor | None = None, workspace: N.Workspace | None = None,
                  status: torch.Tensor | None = None, flags: int | None = None) -> torch.Tensor:
    """One BF16 down row per route slot (``glm53_routes_decode``).  ``bank`` is
    ``(gate_up_w [E,2I,H], gate_up_s, down_w [E,H,I], down_s)``."""
    gu_w, gu_s, d_w, d_s = bank
    dev = N.require_cuda(x_rows, expert_ids, gu_w)
    R, H = x_rows.shape
    E, I2, _ = gu_w.shape
    I = I2 // 2
    if out is None:
        out = torch.empty((R, H), dtype=torch.bfloat16, device=dev)
    wsp = workspace or N.Workspace()
    ws = wsp.get(dev, "routes", N.lib().glm53_routes_decode_workspace_bytes(R, H, I))
    if status is None:
        status = wsp.get(dev, "status", 4)
    if flags is None:
        flags = N.decode_flags(gu_w, d_w)
    N.check(
        N.lib().glm53_routes_decode(
            x_rows.data_ptr(), R, H, expert_ids.data_ptr(), gu_w.data_ptr(), gu_s.data_ptr(), d_w.data_ptr(),
            d_s.data_ptr(), E, I, float(limit), out.data_ptr(), ws.data_ptr(), ws.numel(), status.data_ptr(), flags,
            N.stream(dev),
        ),
        "glm53_routes_decode",
    )
    return out


def routes_decode_coalesced(x_rows: torch.Tensor, expert_ids: torch.Tensor, bank: tuple, *, limit: float,
                            out: torch.Tensor | None = None, workspace: N.Workspace | None = None,
                            status: torch.Tensor | None = None, flags: int | None = None) -> torch.Tensor:
    """``routes_decode`` with expert coalescing (``glm53_routes_decode_coalesced``):
    each touched expert's weights stream once per four of its slots; same bits
    per slot.  Slots with an id >= E (e.g. ``EMPTY_SLOT``) are left untouched."""
    gu_w, gu_s, d_w, d_s = bank
    dev = N.require_cuda(x_rows, expert_ids, gu_w)
    R, H = x_rows.shape
    E, I2, _ = gu_w.shape
    I = I2 // 2
    if out is None:
        out = torch.empty((R, H), dtype=torch.bfloat16, device=dev)
    wsp = workspace or N.Workspace()
    ws = wsp.get(dev, "routes_coalesced", N.lib().glm53_routes_decode_coalesced_workspace_bytes(R, E, H, I))
    if status is None:
        status = wsp.get(dev, "status", 4)
    if flags is None:
        flags = N.decode_flags(gu_w, d_w)
    N.check(
        N.lib().glm53_routes_decode_coalesced(
            x_rows.data_ptr(), R, H, expert_ids.data_ptr(), gu_w.data_ptr(), gu_s.data_ptr(), d_w.data_ptr(),
            d_s.data_ptr(), E, I, float(limit), out.data_ptr(), ws.data_ptr(), ws.numel(), status.data_ptr(), flags,
            N.stream(dev),
        ),
        "glm53_routes_decode_coalesced",
    )
    return out


# Slots per step above which the owners decode with expert coalescing (a
# batch of tokens per rank touches experts more than once per step).
COALESCE_MIN_SLOTS = 16


class ExpertParallelDecode:
    """Plan-owned buffers and the five steps above for one layer.

    ``bank`` holds this rank's experts ``expert_range(rank, world, experts)``;
    ``shared`` the shared expert's six tensors (or None).  ``max_tokens`` sizes
    the fixed capacity (``max_tokens * top_k`` slots per destination, which
    never drops a route).  ``group`` is the ``torch.distributed`` process group
    (NCCL for CUDA tensors); ``world == 1`` needs none."""

    def __init__(self, bank, *, experts: int, rank: int, world: int, shared, limit: float,
                 group=None, max_tokens: int = 1, top_k: int = 8, transport: str = "p2p"):
        self.bank = (bank.gate_up_weight, bank.gate_up_scale_inv, bank.down_weight, bank.down_scale_inv)
        self.experts, self.rank, self.world, self.group = int(experts), int(rank), int(world), group
        lo, hi = expert_range(rank, world, experts)
        if bank.expert_count != hi - lo:
            raise ValueError(f"rank {rank} bank holds {bank.expert_count} experts, expected {hi - lo}")
        self.limit = float(limit)
        self.top_k = int(top_k)
        self.max_tokens = int(max_tokens)
        self.capacity = self.max_tokens * self.top_k
        self.H = bank.hidden_size
        self.shared = None if shared is None else tuple(t.contiguous() for t in shared)
        self.shared_bank = pack_shared_bank(shared)
        dev = bank.gate_up_weight.device
        self.device = dev
        slots = world * self.capacity
        self.send_x = torch.zeros((slots, self.H), dtype=torch.bfloat16, device=dev)
        self.recv_x = torch.zeros_like(self.send_x)
        self.send_e = torch.full((slots,), -1, dtype=torch.int32, device=dev)
        self.recv_e = torch.full_like(self.send_e, -1)
        self.rows = torch.zeros_like(self.send_x)
        self.back = torch.zeros_like(self.send_x)
        self.slot_scores = torch.zeros(slots, dtype=torch.float32, device=dev)
        self.route_pos = torch.zeros(self.max_tokens * self.top_k, dtype=torch.int32, device=dev)
        self.zero_ids = torch.zeros(self.max_tokens, dtype=torch.int32, device=dev)
        self.shared_rows = torch.zeros((self.max_tokens, self.H), dtype=torch.bfloat16, device=dev)
        self.workspace = N.Workspace()
        from .packed import StatusWord

        # fail-closed bits (bad expert id, a peer wait that gave up): published
        # into a pinned host word after every call, raised at the next one
        self.status_word = StatusWord(dev)
        self.status = self.status_word.word
        self.flags = N.decode_flags(self.bank[0], self.bank[2])
        self.shared_flags = N.decode_flags(self.shared_bank[0], self.shared_bank[2]) if self.shared_bank else 0
        if transport not in ("p2p", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport if world > 1 else "nccl"
        self._buffer = None
        self._opened: list[int] = []
        if self.transport == "p2p":
            self._setup_p2p()

    def _setup_p2p(self) -> None:
        """One buffer per rank, every peer's mapped through CUDA IPC."""
        import ctypes

        import torch.distributed as dist

        lib = N.lib()
        nbytes = lib.glm53_ep_shared_bytes(self.world, self.capacity, self.H)
        if nbytes == 0:
            raise ValueError("geometry unsupported by the peer-memory transport")
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        with torch.cuda.device(self.device):
            N.check(lib.glm53_ep_buffer_alloc(nbytes, ctypes.byref(ptr), handle), "glm53_ep_buffer_alloc")
            self._buffer = ptr.value
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=self.group)
            bases = []
            for d in range(self.world):
                if d == self.rank:
                    bases.append(self._buffer)
                    continue
                peer = ctypes.c_void_p()
                N.check(lib.glm53_ep_ipc_open(ctypes.create_string_buffer(handles[d], 64), ctypes.byref(peer)),
                        "glm53_ep_ipc_open")
                self._opened.append(peer.value)
                bases.append(peer.value)
        self.peer_base = torch.tensor(np.array(bases, dtype=np.uint64).view(np.int64), device=self.device)
        self.slot_route = torch.zeros(self.world * self.capacity, dtype=torch.int32, device=self.device)
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: every
        rank calls it once, after its last step)."""
        if self._buffer is None:
            return
        import torch.distributed as dist

        lib = N.lib()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            lib.glm53_ep_ipc_close(p)
        self._opened = []
        dist.barrier(group=self.group)
        lib.glm53_ep_buffer_free(self._buffer)
        self._buffer = None

    def _exchange(self, recv: torch.Tensor, send: torch.Tensor) -> None:
        if self.world == 1:
            recv.copy_(send)
            return
        import torch.distributed as dist

        dist.all_to_all_single(recv, send, group=self.group)

    def __call__(self, x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        flat = x.reshape(-1, self.H)
        T = flat.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the plan's max_tokens={self.max_tokens}")
        if indices.shape[-1] != self.top_k:
            raise ValueError(f"expected top-{self.top_k} routes, got {indices.shape[-1]}")
        lib = N.lib()
        self.status_word.raise_pending()
        st = N.stream(self.device)
        ids = indices.reshape(-1).to(torch.int32).contiguous()
        sc = scores.reshape(-1).to(torch.float32).contiguous()
        flat = flat.contiguous()
        if out is None:
            out = torch.empty((T, self.H), dtype=torch.bfloat16, device=self.device)
        if self.transport == "p2p":
            self._call_p2p(lib, st, flat, T, ids, sc, out)
            self.status_word.publish()
            return out.reshape(x.shape)
        N.check(lib.glm53_ep_dispatch_pack(flat.data_ptr(), T, self.H, ids.data_ptr(), sc.data_ptr(), self.top_k,
                                           self.experts, self.world, self.capacity, self.send_x.data_ptr(),
                                           self.send_e.data_ptr(), self.slot_scores.data_ptr(),
                                           self.route_pos.data_ptr(), self.status.data_ptr(), st),
                "glm53_ep_dispatch_pack")
        self._exchange(self.recv_x, self.send_x)
        self._exchange(self.recv_e, self.send_e)
        decode = routes_decode_coalesced if self.recv_e.numel() >= COALESCE_MIN_SLOTS else routes_decode
        decode(self.recv_x, self.recv_e, self.bank, limit=self.limit, out=self.rows, workspace=self.workspace,
               status=self.status, flags=self.flags)
        shared_ptr = None
        if self.shared_bank is not None:
            decode_s = routes_decode_coalesced if T > 1 else routes_decode
            decode_s(flat, self.zero_ids[:T], self.shared_bank, limit=self.limit, out=self.shared_rows[:T],
                     workspace=self.workspace, status=self.status, flags=self.shared_flags)
            shared_ptr = self.shared_rows.data_ptr()
        self._exchange(self.back, self.rows)
        N.check(lib.glm53_ep_combine(self.back.data_ptr(), self.route_pos.data_ptr(), self.slot_scores.data_ptr(), T,
                                     self.top_k, self.H, shared_ptr, out.data_ptr(), st),
                "glm53_ep_combine")
        self.status_word.publish()
        return out.reshape(x.shape)


    def _shared_rows(self, flat, T):
        if self.shared_bank is None:
            return None
        routes_decode(flat, self.zero_ids[:T], self.shared_bank, limit=self.limit, out=self.shared_rows[:T],
                      workspace=self.workspace, status=self.status, flags=self.shared_flags)
        return self.shared_rows.data_ptr()

    def _call_p2p(self, lib, st, flat, T, ids, sc, out):
        gu_w, gu_s, d_w, d_s = self.bank
        R = self.world * self.capacity
        sh = self.shared
        Ts = T if sh is not None else 0
        ws = self.workspace.get(self.device, "routes",
                                lib.glm53_routes_decode_workspace_bytes(R + Ts, self.H, gu_w.shape[1] // 2))
        N.check(lib.glm53_ep_dispatch_p2p(flat.data_ptr(), T, self.H, ids.data_ptr(), sc.data_ptr(), self.top_k,
                                          self.experts, self.world, self.rank, self.capacity,
                                          self.peer_base.data_ptr(), self.slot_route.data_ptr(),
                                          self.slot_scores.data_ptr(), self.route_pos.data_ptr(),
                                          self.status.data_ptr(), st), "glm53_ep_dispatch_p2p")
        sp = [N.ptr(t) for t in sh] if sh is not None else [None] * 6
        Is = sh[0].shape[0] if sh is not None else 0
        N.check(lib.glm53_ep_owner_decode_p2p(self._buffer, self.H, self.world, self.capacity, self.rank,
                                              gu_w.data_ptr(), gu_s.data_ptr(), d_w.data_ptr(), d_s.data_ptr(),
                                              gu_w.shape[0], gu_w.shape[1] // 2, flat.data_ptr(), Ts, *sp, Is,
                                              self.shared_rows.data_ptr(), self.limit, self.peer_base.data_ptr(),
                                              ws.data_ptr(), ws.numel(), self.status.data_ptr(),
                                              self.flags & self.shared_flags if sh is not None else self.flags, st),
                "glm53_ep_owner_decode_p2p")
        shared_ptr = self.shared_rows.data_ptr() if sh is not None else None
        N.check(lib.glm53_ep_combine_p2p(self._buffer, self.route_pos.data_ptr(), self.slot_scores.data_ptr(), T,
                                         self.top_k, self.H, self.world, self.capacity, shared_ptr, out.data_ptr(),
                                         self.status.data_ptr(), st), "glm53_ep_combine_p2p")
        return out


class ExpertParallelMoE(torch.nn.Module):
    """Decode MoE layer run expert-parallel: this rank's ``gate`` (the full
    router, replicated), its expert slice and the replicated shared expert.
    ``forward(x)`` takes this rank's tokens ``[..., H]`` (at most
    ``max_tokens``) and returns their layer outputs; every rank of the group
    must call it the same number of times (the all-to-alls are collective)."""

    def __init__(self, bank, config, gate, shared, *, rank: int, world: int, group=None, max_tokens: int = 1,
                 transport: str = "p2p"):
        super().__init__()
        from .packed import shared_fp8_tensors

        self.gate = gate
        self.config = config
        self.plan = ExpertParallelDecode(bank, experts=config.n_routed_experts, rank=rank, world=world,
                                         shared=shared_fp8_tensors(shared), limit=config.swiglu_limit, group=group,
                                         max_tokens=max_tokens, top_k=config.num_experts_per_tok,
                                         transport=transport)

    def forward(self, x):
        indices, scores = self.gate(x)
        return self.plan(x, indices, scores)

    def status_word(self, device=None):
        """The plan's StatusWord (fail-closed bits of its kernels)."""
        return self.plan.status_word

    def capture_decode(self):
        """One-token expert-parallel decode as a replayable CUDA graph (every
        rank captures and replays in the same order)."""
        from .packed import CapturedDecode

        return CapturedDecode(self, self.plan.H, self.plan.device)
