#!/usr/bin/env python
"""Benchmark of the B200 FP8 MoE hot path (one JSON line on rank 0).

Headline workload: one packed-decode MoE layer at L=1,
batch 1 -- FP32 router (288 experts, top-8) + fused gate/up/SwiGLU over the 8
selected experts and the shared expert + down / weighted reduce / shared add,
H=4096, I=1536, E4M3 weights with 128x128 FP32 scales, swiglu_limit 10.
A step is one token through one layer.  Steps rotate over --layers distinct
seeded layers (8 x 5.44 GB of experts, far above the 126 MB L2) and a pool of
64 activation vectors, so every step streams its weights from HBM; no L2 flush
is needed.  Steps are CUDA-graph captured; `value` = steps / device time.

`e2e` runs the same steps through `PackedFP8MoE.capture_decode()`: one
`PackedDecodeStep` call per token (one library call: a kernel reads the pinned
host input row, the Float32Gate router, the packed decode writing the pinned
host output row), with both host copies inside the timed region.
`e2e_module` times the plain module call the reference's decode makes
(`layer.mlp(x)` -> `PackedFP8MoE.__call__`, glm53_flash_mlx/packed.py:896),
with the input copied from pinned host memory and the result copied back.

Before the warm-up every captured graph is replayed once, and the same step
graph is replayed for about half a second so that the clock sampler sees the
GPU under this load; `clocks` covers that settle phase, the warm-up and the
timed region (`timed_samples` counts the samples inside the timed region).

`--impl reference` times the CPU restatement of the reference kernels (the
reference's MLX/Metal path cannot run off Apple hardware) on all host cores.

Multi-GPU (torchrun, N>1): expert-parallel decode -- rank r holds experts
[r*288/N, (r+1)*288/N) of every layer, each step routes `--ep-batch` tokens
per rank, dispatches them to the experts' owners over NVLink peer memory (or
NCCL all-to-all with --ep-transport nccl), decodes and combines at home;
value = total tokens / max-over-ranks device time.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, I, E, TOP_K, LIMIT = 4096, 1536, 288, 8, 10.0
POOL = 64
GRAPH_STEPS = 64  # decode steps chained in one CUDA graph


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20000)
    p.add_argument("--warmup", type=int, default=2000)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--layers", type=int, default=8, help="distinct layers rotated through (L2 defeat)")
    p.add_argument("--no-prefill", action="store_true", help="skip the secondary T=2048 grouped measurement")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="bounded CPU-baseline sample")
    p.add_argument("--experts", type=int, default=E, help="routed experts per layer (profiling uses fewer)")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    p.add_argument("--no-e2e", action="store_true", help="skip the module-API end-to-end pass")
    p.add_argument("--quick-linear", action="store_true", help="config-5 sweep at M in {1, 64, 512} only")
    p.add_argument("--linear-only", action="store_true", help="run only the config-1/5 block-linear sweep")
    p.add_argument("--batched-only", action="store_true", help="run only the batched decode measurements (B = 16, 24, 64; config 4 at N = 1)")
    p.add_argument("--batched-tokens", default="16,24,64", help="batch sizes of the batched decode measurement")
    p.add_argument("--prefill-only", action="store_true",
                   help="profiling aid: only the T=2048 grouped prefill measurement (prints its JSON and exits)")
    p.add_argument("--prefill-reps", type=int, default=8, help="timed grouped prefill layers")
    p.add_argument("--prefill-tokens", default="256,2048,8192", help="--prefill-only: token counts")
    p.add_argument("--prefill-mma", choices=["f16", "f8", "both"], default="both",
                   help="--prefill-only: grouped GEMM kernel(s) to time")
    p.add_argument("--hc-only", action="store_true",
                   help="run only the FFN-boundary (mHC collapse + RMSNorm, hc expand) measurement")
    p.add_argument("--hc-tokens", default="1,256,2048", help="token counts of the FFN-boundary measurement")
    p.add_argument("--ep-transport", choices=["p2p", "nccl"], default="p2p",
                   help="N > 1: expert-parallel dispatch/combine through peer memory or NCCL all-to-alls")
    return p.parse_args()


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------


def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([time.monotonic()] + [c.strip() for c in line.split(",")])

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread is not None:
                self.thread.join(timeout=2)

    def summary(self, t0: float | None = None, t1: float | None = None) -> dict:
        """Clocks sampled between host times t0 and t1 (the timed region)."""
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if (t0 is not None and r[0] < t0) or (t1 is not None and r[0] > t1):
                continue
            r = r[1:]
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}

    def window(self, t_settle: float, t0: float, t1: float) -> dict:
        """Clocks over the settle phase, the warm-up and the timed region
        (t_settle..t1), with the count of samples inside the timed region."""
        d = self.summary(t_settle, t1)
        d["timed_samples"] = self.summary(t0, t1)["samples"]
        d["window"] = "settle (~0.5 s of the timed step graph) + warm-up + timed region"
        return d


def settle_clocks(graph, world: int, seconds: float = 0.5) -> float:
    """Replay `graph` (the timed step graph) for about `seconds` before the
    warm-up so that the 200 ms clock sampler sees the GPU under this load
    even when the timed region is a millisecond; returns the host time the
    settle phase started."""
    import math

    import torch

    barrier(world)
    t0 = time.monotonic()
    graph.replay()
    torch.cuda.synchronize()
    one = max(time.monotonic() - t0, 1e-5)
    # every rank replays the same number of times (the graphs may hold
    # collectives or peer handshakes)
    n = int(max_over_ranks(float(math.ceil(seconds / one)), world))
    for _ in range(min(n, 100000)):
        graph.replay()
    torch.cuda.synchronize()
    return t0


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d.get("bf16_tflops", 1590.0)),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------

# algorithmic bytes of one decode step (config 2, I = 1536)
ROUTER_BYTES = E * H * 4 + E * 4 + H * 2
GATE_UP_BYTES = (TOP_K + 1) * 2 * I * H + TOP_K * 2 * (I // 128) * (H // 128) * 4 + 2 * (I // 128) * (H // 128) * 4 \
    + H * 2 + (TOP_K * I + I) * 2 + TOP_K * 4
DOWN_BYTES = (TOP_K + 1) * H * I + (TOP_K + 1) * (H // 128) * (I // 128) * 4 + (TOP_K * I + I) * 2 + H * 2 + TOP_K * 8
STEP_BYTES = ROUTER_BYTES + GATE_UP_BYTES + DOWN_BYTES
# DRAM bytes (read + write) of one gate/up launch in one ncu capture of the
# decode (dram__bytes_read.sum 113,314,304 + dram__bytes_write.sum 3,461,888;
# 64-expert bank of these shapes, 1.2 GB > L2, so every weight byte came from
# DRAM): the same nine experts' bytes as any config-2 step.
GATE_UP_TRAFFIC = 113_314_304 + 3_461_888


def build_layers(n_layers: int, seed0: int, device, experts: int = E):
    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    layers = []
    for l in range(n_layers):
        seed = seed0 + 17 * l
        bank = S.make_bank(experts, H, I, seed=seed, device=device)
        shared_mod = S.make_shared(H, I, seed=seed + 1, limit=LIMIT, device=device)
        w, b = S.make_router(experts, H, seed=seed + 2, device=device)
        layers.append({"bank": bank, "shared_mod": shared_mod, "shared": shared_fp8_tensors(shared_mod),
                       "router_w": w, "router_b": b})
    return layers


def time_stage_graph(fn, n, reps, stream, dev):
    """Average device time (ms) of one fn(i, stream) call: n calls are
    captured into one CUDA graph (after an eager pass that sets kernel
    attributes), replayed `reps` times between CUDA events."""
    import torch

    with torch.cuda.stream(stream):
        for i in range(n):
            fn(i, stream.cuda_stream)
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(n):
            fn(i, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        g.replay()
    stop.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / (reps * n)
    del g
    return ms


def bench_b200(args, world, rank, local):
    import torch

    import glm53_flash_mlx_b200 as G
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.router import Float32Gate

    dev = torch.device("cuda", local)
    lib = N.lib()
    n_exp = args.experts
    layers = build_layers(args.layers, 1000 + 101 * rank, dev, n_exp)
    xs = S.random_bf16((POOL, H), seed=77 + rank, device=dev)

    # ---- one step = router + packed decode, captured per (layer, x) -------
    ws = N.Workspace()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    n_graphs = POOL
    outs = [torch.empty(H, dtype=torch.bfloat16, device=dev) for _ in range(n_graphs)]
    idxs = [torch.empty((1, TOP_K), dtype=torch.int32, device=dev) for _ in range(n_graphs)]
    scs = [torch.empty((1, TOP_K), dtype=torch.float32, device=dev) for _ in range(n_graphs)]
    rws = ws.get(dev, "router", lib.glm53_router_workspace_bytes(1, n_exp))
    flags = [N.decode_flags(L["bank"].gate_up_weight, L["bank"].down_weight, L["shared"][0], L["shared"][2],
                            L["shared"][4]) for L in layers]
    dws = ws.get(dev, "decode", lib.glm53_packed_decode_workspace_bytes(TOP_K, H, I, I))

    def step(i, stream):
        L = layers[i % args.layers]
        x = xs[i % POOL]
        N.check(lib.glm53_router_topk(x.data_ptr(), 1, H, L["router_w"].data_ptr(), n_exp, L["router_b"].data_ptr(),
                                      TOP_K, 1, 1, 1, 1.0, idxs[i].data_ptr(), scs[i].data_ptr(), None,
                                      rws.data_ptr(), rws.numel(), stream), "router")
        sh = L["shared"]
        bank = L["bank"]
        N.check(lib.glm53_packed_decode_moe(
            x.data_ptr(), H, idxs[i].data_ptr(), scs[i].data_ptr(), TOP_K, bank.gate_up_weight.data_ptr(),
            bank.gate_up_scale_inv.data_ptr(), bank.down_weight.data_ptr(), bank.down_scale_inv.data_ptr(), n_exp,
            I, sh[0].data_ptr(), sh[1].data_ptr(), sh[2].data_ptr(), sh[3].data_ptr(), sh[4].data_ptr(),
            sh[5].data_ptr(), I, LIMIT, outs[i].data_ptr(), dws.data_ptr(), dws.numel(), status.data_ptr(),
            flags[i % args.layers] | N.FLAG_AFTER_ROUTER, stream), "decode")

    # A model's decode graph chains its layers back to back; here one CUDA
    # graph chains GRAPH_STEPS steps (rotating layers and inputs), and a
    # second graph holds the remainder so that exactly K steps are timed.
    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        for i in range(n_graphs):  # eager warm-up (sets kernel attributes)
            step(i, s.cuda_stream)
    s.synchronize()

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(n):
                step(i, torch.cuda.current_stream().cuda_stream)
        return g

    full = capture(GRAPH_STEPS)
    rem_w, rem_t = args.warmup % GRAPH_STEPS, args.steps % GRAPH_STEPS
    rem = {n: capture(n) for n in {rem_w, rem_t} if n}
    torch.cuda.synchronize()
    # every graph's first launch (its upload) happens here, outside the timing
    for g in (full, *rem.values()):
        g.replay()
    torch.cuda.synchronize()

    def run(k):
        for _ in range(k // GRAPH_STEPS):
            full.replay()
        if k % GRAPH_STEPS:
            rem[k % GRAPH_STEPS].replay()

    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        hs = settle_clocks(full, world)
        run(args.warmup)
        torch.cuda.synchronize()
        barrier(world)
        h0 = time.monotonic()
        start.record()
        run(args.steps)
        stop.record()
        torch.cuda.synchronize()
        h1 = time.monotonic()
        barrier(world)
    t_ms = max_over_ranks(start.elapsed_time(stop), world)
    if int(status.item()) != 0:
        raise RuntimeError(f"device status 0x{int(status.item()):x} during the timed region")
    clk = clocks.window(hs, h0, h1)
    tokens = args.steps * world
    value = tokens / (t_ms / 1e3)

    # ---- single stages, each captured 64 times into one graph -------------
    def router_only(i, stream):
        L = layers[i % args.layers]
        N.check(lib.glm53_router_topk(xs[i % POOL].data_ptr(), 1, H, L["router_w"].data_ptr(), n_exp,
                                      L["router_b"].data_ptr(), TOP_K, 1, 1, 1, 1.0, idxs[i % n_graphs].data_ptr(),
                                      scs[i % n_graphs].data_ptr(), None, rws.data_ptr(), rws.numel(), stream),
                "router")

    def gate_up_only(i, stream):
        L = layers[i % args.layers]
        sh = L["shared"]
        bank = L["bank"]
        N.check(lib.glm53_packed_decode_gate_up(
            xs[i % POOL].data_ptr(), H, idxs[i % n_graphs].data_ptr(), TOP_K, bank.gate_up_weight.data_ptr(),
            bank.gate_up_scale_inv.data_ptr(), n_exp, I, sh[0].data_ptr(), sh[1].data_ptr(), sh[2].data_ptr(),
            sh[3].data_ptr(), I, LIMIT, dws.data_ptr(), dws.numel(), status.data_ptr(), flags[i % args.layers],
            stream), "gate_up")

    reps = max(4, min(args.steps // 64, 64))
    router_ms = time_stage_graph(router_only, 64, reps, s, dev)
    k_ms = time_stage_graph(gate_up_only, 64, reps, s, dev)
    peaks = measured_peaks()
    achieved = GATE_UP_BYTES / (k_ms / 1e3) / 1e9
    roofline = {"kernel": "decode_gate_up_v4", "bound": "hbm", "achieved": round(achieved, 1),
                "peak": peaks["hbm_gbs"], "peak_source": peaks["source"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": GATE_UP_TRAFFIC,
                "traffic_source": "ncu capture (dram__bytes_read.sum + dram__bytes_write.sum), 64-expert case",
                "algorithmic_bytes_per_launch": GATE_UP_BYTES, "avg_launch_us": round(k_ms * 1e3, 2),
                "launches_timed": reps * 64, "step_bytes": STEP_BYTES,
                "step_frac": round(STEP_BYTES / (t_ms / args.steps / 1e3) / 1e9 / peaks["hbm_gbs"], 4)}

    # ---- e2e through the public module API -------------------------------
    e2e = e2e_module = None
    if not args.no_e2e:
        mods = []
        for L in layers:
            cfg = S.moe_config(H, I, n_exp, TOP_K, LIMIT)
            gate = Float32Gate(cfg, device=dev)
            gate.weight.copy_(L["router_w"])
            gate.e_score_correction_bias.copy_(L["router_b"])
            mods.append(G.PackedFP8MoE(L["bank"], cfg, gate, L["shared_mod"]))
        caps = [m.capture_decode() for m in mods]
        x_host = xs.cpu().reshape(POOL, 1, 1, H).pin_memory()
        y_host = torch.empty((POOL, 1, 1, H), dtype=torch.bfloat16).pin_memory()
        for i in range(min(args.warmup, 500)):
            caps[i % args.layers](x_host[i % POOL], out=y_host[i % POOL])
        torch.cuda.synchronize()
        barrier(world)
        e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record()
        for i in range(args.steps):
            caps[i % args.layers](x_host[i % POOL], out=y_host[i % POOL])
        e_stop.record()
        torch.cuda.synchronize()
        barrier(world)
        e_ms = max_over_ranks(e_start.elapsed_time(e_stop), world)
        e2e = {"value": round(tokens / (e_ms / 1e3), 2), "unit": "tokens/s", "h2d_bytes_per_step": H * 2,
               "d2h_bytes_per_step": H * 2,
               "api": "PackedFP8MoE.capture_decode() step per token: one glm53_decode_step_host call (a kernel "
                      "reads the pinned host input row, Float32Gate router, packed decode writing the pinned host "
                      "output row)"}
        for c in caps:
            c.check()
        del caps
        # the plain module call (layer.mlp(x) -> PackedFP8MoE.__call__), with
        # the row copied in from pinned host memory and the result copied back
        n_mod = args.steps
        for i in range(min(args.warmup, 200)):
            y = mods[i % args.layers](x_host[i % POOL].to(dev, non_blocking=True))
            y_host[i % POOL].copy_(y, non_blocking=True)
        torch.cuda.synchronize()
        barrier(world)
        m_start, m_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        m_start.record()
        for i in range(n_mod):
            y = mods[i % args.layers](x_host[i % POOL].to(dev, non_blocking=True))
            y_host[i % POOL].copy_(y, non_blocking=True)
        m_stop.record()
        torch.cuda.synchronize()
        barrier(world)
        for m in mods:
            m.check_status()
        m_ms = max_over_ranks(m_start.elapsed_time(m_stop), world)
        e2e_module = {"value": round(n_mod * world / (m_ms / 1e3), 2), "unit": "tokens/s",
                      "h2d_bytes_per_step": H * 2, "d2h_bytes_per_step": H * 2,
                      "api": "PackedFP8MoE(bank, config, Float32Gate, shared)(x) per token (the reference's "
                             "layer.mlp(x)), x copied from pinned host memory, result copied back"}

    step_us = t_ms / args.steps * 1e3
    extra = {"stages_us": {"router": round(router_ms * 1e3, 2), "gate_up": round(k_ms * 1e3, 2),
                           "down_and_boundaries": round(step_us - (router_ms + k_ms) * 1e3, 2),
                           "note": "router and gate/up each timed alone (64 calls per CUDA graph)"}}
    if e2e_module is not None:
        extra["e2e_module"] = e2e_module
    if not args.no_prefill:
        for T in (256, 2048, 8192):
            extra[f"prefill_{T}"] = bench_prefill(layers, dev, args, T)
            extra[f"prefill_{T}_f8"] = bench_prefill(layers, dev, args, T, "f8")
        extra["linear_config1_5"] = bench_linear(dev, args)
        extra["batched_decode"] = bench_batched(layers, dev, args)
        extra["ep_batched"] = {f"B{B}": bench_ep_batched(layers, dev, args, 1, 0, B) for B in (16, 64)}
        extra["ffn_boundary"] = bench_hc(dev, args)
    return {"value": value, "t_ms": t_ms, "clocks": clk, "roofline": roofline, "e2e": e2e,
            "gpu_launches": args.steps * 3, **extra}, layers, xs


def bench_batched(layers, dev, args):
    """Secondary: batched decode on one GPU -- B = 16, 24 and 64 tokens through
    PackedFP8MoE (router + expert-coalesced batched decode + BF16 combine in
    ascending expert id + shared expert: the Direct module's multi-row
    semantics) versus the Direct module's per-expert loop on the same layer."""
    import torch

    import glm53_flash_mlx_b200 as G
    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.router import Float32Gate

    L = layers[0]
    n_exp = L["bank"].expert_count
    cfg = S.moe_config(H, I, n_exp, TOP_K, LIMIT)
    gate = Float32Gate(cfg, device=dev)
    gate.weight.copy_(L["router_w"])
    gate.e_score_correction_bias.copy_(L["router_b"])
    mod = G.PackedFP8MoE(L["bank"], cfg, gate, L["shared_mod"])
    out = {}
    for B in (int(b) for b in args.batched_tokens.split(",")):
        xs = [S.random_bf16((1, B, H), seed=500 + i, device=dev) for i in range(8)]
        for i in range(3):
            mod(xs[i % 8])
        torch.cuda.synchronize()
        st, sp = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 40
        st.record()
        for i in range(n):
            mod(xs[i % 8])
        sp.record()
        torch.cuda.synchronize()
        us = st.elapsed_time(sp) * 1e3 / n
        idx, sc = mod.gate(xs[0])
        mod._forward_routes(xs[0], idx, sc)
        torch.cuda.synchronize()
        st.record()
        for i in range(3):
            idx, sc = mod.gate(xs[i % 8])
            mod._forward_routes(xs[i % 8], idx, sc)
        sp.record()
        torch.cuda.synchronize()
        loop_us = st.elapsed_time(sp) * 1e3 / 3
        touched = int(torch.unique(idx).numel())
        mean_touched = statistics.mean(int(torch.unique(mod.gate(x)[0]).numel()) for x in xs)
        # bytes one call streams: the touched experts, the shared expert and the router
        call_bytes = (mean_touched + 1) * 3 * H * I + n_exp * H * 4
        out[f"B{B}"] = {"us": round(us, 1), "tokens_per_s": round(B / (us / 1e6), 1), "touched_experts": touched,
                        "mean_touched_experts": round(mean_touched, 1),
                        "hbm_frac": round(call_bytes / (us / 1e6) / 1e9 / measured_peaks()["hbm_gbs"], 4),
                        "direct_loop_us": round(loop_us, 1)}
    return out


def bench_linear(dev, args):
    """Secondary: config 1 (block-FP8 GEMV y = x . W^T, W E4M3 [6144, 4096] +
    128x128 scales, x BF16 [1, 4096]) and the config-5 sweep: W in {[6144, 4096],
    [4096, 4096], [12288, 4096], [4096, 12288], [576, 4096]} at M in {1, 8, 64,
    512, 2048, 8192}.  Weight copies rotate (>= 200 MB per shape, above L2); 64
    calls per CUDA graph, CUDA events.  M <= 16 calls glm53_fp8_linear (GEMV
    tiles), larger M glm53_fp8_linear_ws (tcgen05 GEMM), as block_fp8_linear does."""
    import torch

    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200 import synthetic as S

    lib = N.lib()
    peaks = measured_peaks()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    s = torch.cuda.Stream(device=dev)
    shapes = [(6144, 4096), (4096, 4096), (12288, 4096), (4096, 12288), (576, 4096)]
    ms_list = (1, 8, 64, 512, 2048, 8192) if not args.quick_linear else (1, 64, 512)
    out = {}
    for (Nn, K) in shapes:
        copies = max(2, -(-200_000_000 // (Nn * K)))
        wts = [S.random_block_fp8(Nn, K, seed=c, tensor=0, std=0.02, device=dev) for c in range(copies)]
        fl = N.decode_flags(*[w for w, _ in wts])
        res = {}
        for M in ms_list:
            x = S.random_bf16((M, K), seed=M, device=dev)
            y = torch.empty((M, Nn), dtype=torch.bfloat16, device=dev)
            wsb = lib.glm53_fp8_linear_splitk_workspace_bytes(M, K, Nn)
            wsp = torch.zeros(max(wsb, 256), dtype=torch.uint8, device=dev)

            def call(i, stream):
                w, sc = wts[i % copies]
                if M > 16:
                    N.check(lib.glm53_fp8_linear_ws(x.data_ptr(), M, K, w.data_ptr(), Nn, sc.data_ptr(), y.data_ptr(),
                                                    wsp.data_ptr(), wsp.numel(), status.data_ptr(), fl, stream),
                            "linear_ws")
                else:
                    N.check(lib.glm53_fp8_linear(x.data_ptr(), M, K, w.data_ptr(), Nn, sc.data_ptr(), y.data_ptr(),
                                                 fl, stream), "linear")

            n_calls = 64 if M <= 2048 else 16
            ms = time_stage_graph(call, n_calls, 4, s, dev)
            bytes_ = Nn * K + 4 * (-(-Nn // 128)) * (K // 128) + 2 * M * K + 2 * M * Nn
            flops = 2 * M * Nn * K
            res[f"M{M}"] = {"us": round(ms * 1e3, 2),
                            "hbm_frac": round(bytes_ / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
                            "tflops": round(flops / (ms / 1e3) / 1e12, 1),
                            "tensor_frac": round(flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops"], 4)}
            del x, y, wsp
        out[f"{Nn}x{K}"] = res
        del wts
    if int(status.item()) != 0:
        raise RuntimeError(f"device status 0x{int(status.item()):x} in the linear sweep")
    return {"shapes": "W [N, K] E4M3 + FP32 128x128 scales; x BF16 [M, K]; 6144x4096 at M=1 is config 1",
            "results": out,
            "note": "M <= 16: tensor-core GEMV tiles (HBM-bound); M > 16: tcgen05 GEMM (kind::f16, exact FP16 "
                    "weights, FP32 promotion per 128-K block); tensor_frac against the measured BF16 peak"}


def build_ep_layers(n_layers: int, rank: int, world: int, device, experts: int = E):
    """Per-rank expert slices (E / world experts of each layer) plus the
    replicated router and shared expert (same seeds on every rank)."""
    from glm53_flash_mlx_b200 import synthetic as S
    from glm53_flash_mlx_b200.packed import shared_fp8_tensors

    layers = []
    for l in range(n_layers):
        seed = 1000 + 17 * l
        bank = S.make_bank(experts // world, H, I, seed=seed + 7919 * (rank + 1), device=device)
        shared_mod = S.make_shared(H, I, seed=seed + 1, limit=LIMIT, device=device)
        w, b = S.make_router(experts, H, seed=seed + 2, device=device)
        layers.append({"bank": bank, "shared_mod": shared_mod, "shared": shared_fp8_tensors(shared_mod),
                       "router_w": w, "router_b": b})
    return layers


def bench_ep(args, world, rank, local):
    """N > 1: expert-parallel decode (config 4 at batch 1 per rank): each rank
    routes its own token, the routes travel to their experts' ranks and back
    through peer memory (``--ep-transport nccl``: NCCL all-to-alls), 64 steps
    per CUDA graph."""
    import torch

    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200 import ep
    from glm53_flash_mlx_b200 import synthetic as S

    dev = torch.device("cuda", local)
    lib = N.lib()
    n_exp = args.experts
    layers = build_ep_layers(args.layers, rank, world, dev, n_exp)
    xs = S.random_bf16((POOL, H), seed=77 + rank, device=dev)
    plans = [ep.ExpertParallelDecode(L["bank"], experts=n_exp, rank=rank, world=world, shared=L["shared"],
                                     limit=LIMIT, max_tokens=1, transport=args.ep_transport) for L in layers]
    ws = N.Workspace()
    rws = ws.get(dev, "router", lib.glm53_router_workspace_bytes(1, n_exp))
    idxs = [torch.empty((1, TOP_K), dtype=torch.int32, device=dev) for _ in range(GRAPH_STEPS)]
    scs = [torch.empty((1, TOP_K), dtype=torch.float32, device=dev) for _ in range(GRAPH_STEPS)]
    outs = [torch.empty((1, H), dtype=torch.bfloat16, device=dev) for _ in range(GRAPH_STEPS)]

    def step(i, stream):
        L = layers[i % args.layers]
        x = xs[i % POOL].reshape(1, H)
        N.check(lib.glm53_router_topk(x.data_ptr(), 1, H, L["router_w"].data_ptr(), n_exp, L["router_b"].data_ptr(),
                                      TOP_K, 1, 1, 1, 1.0, idxs[i].data_ptr(), scs[i].data_ptr(), None,
                                      rws.data_ptr(), rws.numel(), stream), "router")
        plans[i % args.layers](x, idxs[i], scs[i], out=outs[i])

    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        for i in range(GRAPH_STEPS):
            step(i, s.cuda_stream)
    s.synchronize()
    barrier(world)
    graph_mode = "64 EP decode steps per CUDA graph (NCCL all-to-alls captured)"
    try:
        full = torch.cuda.CUDAGraph()
        with torch.cuda.graph(full, stream=s):
            for i in range(GRAPH_STEPS):
                step(i, torch.cuda.current_stream().cuda_stream)
        rem_w, rem_t = args.warmup % GRAPH_STEPS, args.steps % GRAPH_STEPS
        rem = {}
        for n in sorted({rem_w, rem_t} - {0}):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for i in range(n):
                    step(i, torch.cuda.current_stream().cuda_stream)
            rem[n] = g

        def run(k):
            for _ in range(k // GRAPH_STEPS):
                full.replay()
            if k % GRAPH_STEPS:
                rem[k % GRAPH_STEPS].replay()
    except Exception:  # capture unsupported: eager steps on the side stream
        full, rem = None, {}
        graph_mode = "eager EP decode steps (graph capture unavailable)"

        def run(k):
            with torch.cuda.stream(s):
                for i in range(k):
                    step(i % GRAPH_STEPS, s.cuda_stream)

    torch.cuda.synchronize()
    barrier(world)
    if full is not None:  # every graph's first launch happens here, outside the timing
        for g in (full, *rem.values()):
            g.replay()
    torch.cuda.synchronize()
    barrier(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        hs = settle_clocks(full, world) if full is not None else time.monotonic()
        run(args.warmup)
        torch.cuda.synchronize()
        barrier(world)
        h0 = time.monotonic()
        start.record()
        run(args.steps)
        stop.record()
        torch.cuda.synchronize()
        h1 = time.monotonic()
        barrier(world)
    t_ms = max_over_ranks(start.elapsed_time(stop), world)
    bad = max_over_ranks(float(max(int(p.status.item()) for p in plans)), world)
    if bad:
        raise RuntimeError(f"device status 0x{int(bad):x} during the timed region")
    clk = clocks.window(hs, h0, h1)
    tokens = args.steps * world
    value = tokens / (t_ms / 1e3)
    peaks = measured_peaks()
    step_s = t_ms / args.steps / 1e3
    roofline = {"kernel": "EP decode step (per rank: ~8 received routes + shared + router)", "bound": "hbm",
                "achieved": round(STEP_BYTES / step_s / 1e9, 1), "peak": peaks["hbm_gbs"],
                "peak_source": peaks["source"], "unit": "GB/s",
                "frac": round(STEP_BYTES / step_s / 1e9 / peaks["hbm_gbs"], 4), "traffic": None,
                "algorithmic_bytes_per_launch": STEP_BYTES,
                "note": "per-rank bytes of an average step: world tokens x 8 routes spread over world ranks"}
    # release the graphs (they hold NCCL work) before any later teardown
    rem.clear()
    del full, run
    torch.cuda.synchronize()
    # e2e: the module API with host copies, every rank one token per step
    e2e = None
    if not args.no_e2e:
        from types import SimpleNamespace

        from glm53_flash_mlx_b200.router import Float32Gate

        cfg = SimpleNamespace(hidden_size=H, moe_intermediate_size=I, swiglu_limit=LIMIT, n_routed_experts=n_exp,
                              num_experts_per_tok=TOP_K)
        mods = []
        for L in layers:
            gate = Float32Gate(cfg, device=dev)
            gate.weight.copy_(L["router_w"])
            gate.e_score_correction_bias.copy_(L["router_b"])
            mods.append(ep.ExpertParallelMoE(L["bank"], cfg, gate, L["shared_mod"], rank=rank, world=world,
                                             transport=args.ep_transport))
        caps = [m.capture_decode() for m in mods]
        hx = xs.cpu().reshape(POOL, 1, 1, H).pin_memory()
        hout = torch.empty((POOL, 1, 1, H), dtype=torch.bfloat16).pin_memory()
        n_e2e = min(args.steps, 4096)
        for i in range(min(args.warmup, 64)):
            caps[i % len(caps)](hx[i % POOL], out=hout[i % POOL])
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(n_e2e):
            caps[i % len(caps)](hx[i % POOL], out=hout[i % POOL])
        e1.record()
        torch.cuda.synchronize()
        e_ms = max_over_ranks(e0.elapsed_time(e1), world)
        e2e = {"value": round(n_e2e * world / (e_ms / 1e3), 2), "unit": "tokens/s", "h2d_bytes_per_step": H * 2,
               "d2h_bytes_per_step": H * 2,
               "api": "ExpertParallelMoE.capture_decode() replays (Float32Gate router + expert-parallel decode), "
                      "pinned host input copied in and output copied out every step", "steps": n_e2e}
        del caps
        torch.cuda.synchronize()
    for p in plans + ([m.plan for m in mods] if not args.no_e2e else []):
        p.close()
    launches = 5 if args.ep_transport == "p2p" else 8
    res = {"value": value, "t_ms": t_ms, "clocks": clk, "roofline": roofline, "e2e": e2e,
           "gpu_launches": args.steps * launches, "graph": graph_mode + f"; transport {args.ep_transport}"}
    if not args.no_prefill:
        res["ep_batched"] = {f"B{B}": bench_ep_batched(layers, dev, args, world, rank, B) for B in (16, 64)}
    return res


def bench_ep_batched(layers, dev, args, world: int, rank: int, B: int) -> dict:
    """Config 4 at B tokens per rank: each step routes B tokens through one
    layer (the FP32 router, then ExpertParallelDecode with max_tokens = B:
    dispatch to the experts' ranks over NCCL all-to-all -- a local copy at
    N = 1 -- the owners' expert-coalesced decode, the return all-to-all and the
    slot-ordered combine with the shared expert).  Layers rotate (8 distinct
    seeded layers: the 42-layer stack does not fit one GPU's HBM, 228 GB of
    experts), so the figure is per layer; `tokens_per_s_42_layers` divides it
    by 42.  Steps are CUDA-graph captured, device-timed, max over ranks."""
    import torch

    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200 import ep
    from glm53_flash_mlx_b200 import synthetic as S

    lib = N.lib()
    n_exp = args.experts
    plans = [ep.ExpertParallelDecode(L["bank"], experts=n_exp, rank=rank, world=world, shared=L["shared"],
                                     limit=LIMIT, max_tokens=B, transport="nccl") for L in layers]
    xs = S.random_bf16((4, B, H), seed=91 + rank, device=dev)
    ws = N.Workspace()
    rws = ws.get(dev, "router", lib.glm53_router_workspace_bytes(B, n_exp))
    n_graph = 2 * len(layers)
    idxs = [torch.empty((B, TOP_K), dtype=torch.int32, device=dev) for _ in range(n_graph)]
    scs = [torch.empty((B, TOP_K), dtype=torch.float32, device=dev) for _ in range(n_graph)]
    outs = [torch.empty((B, H), dtype=torch.bfloat16, device=dev) for _ in range(n_graph)]
    touched = []

    def step(i, stream):
        L = layers[i % len(layers)]
        x = xs[i % 4]
        N.check(lib.glm53_router_topk(x.data_ptr(), B, H, L["router_w"].data_ptr(), n_exp, L["router_b"].data_ptr(),
                                      TOP_K, 1, 1, 1, 1.0, idxs[i].data_ptr(), scs[i].data_ptr(), None,
                                      rws.data_ptr(), rws.numel(), stream), "router")
        plans[i % len(layers)](x, idxs[i], scs[i], out=outs[i])

    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        for i in range(n_graph):
            step(i, s.cuda_stream)
    s.synchronize()
    touched = [int(torch.unique(idxs[i]).numel()) for i in range(n_graph)]
    barrier(world)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(n_graph):
            step(i, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    barrier(world)
    reps = max(3, min(50, 2000 // n_graph // max(1, B // 8)))
    st, sp = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(reps):
        g.replay()
    sp.record()
    torch.cuda.synchronize()
    t_ms = max_over_ranks(st.elapsed_time(sp), world) / (reps * n_graph)
    bad = max_over_ranks(float(max(int(p.status.item()) for p in plans)), world)
    del g
    torch.cuda.synchronize()
    for p in plans:
        p.close()
    if bad:
        raise RuntimeError(f"device status 0x{int(bad):x} in the batched expert-parallel decode")
    peaks = measured_peaks()
    mean_touched = statistics.mean(touched)
    # bytes one rank streams per step: its share of the touched experts, the
    # shared expert and the router
    step_bytes = (mean_touched / world) * 3 * H * I + 3 * H * I + n_exp * H * 4
    return {"batch_per_rank": B, "tokens_per_step": B * world, "ms_per_layer_step": round(t_ms, 4),
            "tokens_per_s_per_layer": round(B * world / (t_ms / 1e3), 1),
            "tokens_per_s_42_layers": round(B * world / (42 * t_ms / 1e3), 1),
            "touched_experts_per_step": round(mean_touched, 1),
            "hbm_frac_per_rank": round(step_bytes / (t_ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
            "transport": "nccl all-to-all" if world > 1 else "local (one GPU)",
            "owner_decode": "expert-coalesced (glm53_routes_decode_coalesced)",
            "layers_rotated": len(layers), "steps_timed": reps * n_graph}


def bench_prefill(layers, dev, args, T: int = 2048, mma: str = "f16"):
    """Secondary: config 3 grouped prefill at T tokens (256, 2048, 8192),
    Zipf-skewed router bias; layers rotate so weights stream from HBM.
    mma="f8": the grouped GEMMs on the kind::f8f6f4 kernel (GLM53_FLAG_F8_MMA),
    with the output's agreement with the kind::f16 kernel's on the same layer."""
    import torch

    import glm53_flash_mlx_b200 as G
    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200 import synthetic as S

    x = S.random_bf16((T, H), seed=4242, device=dev)
    n_exp = layers[0]["bank"].expert_count
    w, b = S.make_router(n_exp, H, seed=4243, device=dev, zipf_alpha=0.5)
    ws = N.Workspace()
    idx, sc = G.router_topk(x, w, b, top_k=TOP_K, workspace=ws)
    touched = int(torch.unique(idx).numel())
    for i in range(3):
        L = layers[i % len(layers)]
        G.router_topk(x, w, b, top_k=TOP_K, workspace=ws)
        G.grouped_moe(x, idx, sc, L["bank"], L["shared"], limit=LIMIT, workspace=ws, mma=mma)
    torch.cuda.synchronize()
    reps = args.prefill_reps
    st, sp = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for i in range(reps):
        L = layers[i % len(layers)]
        G.router_topk(x, w, b, top_k=TOP_K, workspace=ws)
        G.grouped_moe(x, idx, sc, L["bank"], L["shared"], limit=LIMIT, workspace=ws, mma=mma)
    sp.record()
    torch.cuda.synchronize()
    ms = st.elapsed_time(sp) / reps
    bytes_ = (touched + 1) * 3 * H * I + n_exp * H * 4 + 2 * T * H * 2
    flops = 2 * T * TOP_K * 3 * H * I + 2 * T * 3 * H * I + 2 * T * n_exp * H
    peaks = measured_peaks()
    t_hbm = bytes_ / (peaks["hbm_gbs"] * 1e9)
    t_tc = flops / (peaks["bf16_tflops"] * 1e12)
    loads = torch.bincount(idx.reshape(-1).long(), minlength=n_exp)
    agree = None
    if mma == "f8":
        L = layers[0]
        o8 = G.grouped_moe(x, idx, sc, L["bank"], L["shared"], limit=LIMIT, workspace=ws, mma="f8").float()
        o16 = G.grouped_moe(x, idx, sc, L["bank"], L["shared"], limit=LIMIT, workspace=ws, mma="f16").float()
        d = (o8 - o16).abs()
        agree = {"max_abs": float(d.max()), "cosine": float(torch.nn.functional.cosine_similarity(
                     o8.reshape(1, -1).double(), o16.reshape(1, -1).double()).item()),
                 "bit_identical": float((o8 == o16).float().mean())}
    res = {"tokens": T, "tokens_per_s": round(T / (ms / 1e3), 1), "ms_per_layer": round(ms, 3),
            "touched_experts": touched, "max_routes_per_expert": int(loads.max()),
            "mean_routes_per_touched_expert": round(T * TOP_K / max(touched, 1), 1),
            "algorithmic_bytes": bytes_, "flops": flops,
            "hbm_frac": round(t_hbm / (ms / 1e3), 4),
            "tensor_frac": round(t_tc / (ms / 1e3), 4),
            "roofline_frac": round(max(t_hbm, t_tc) / (ms / 1e3), 4),
            "roofline_bound": "hbm" if t_hbm >= t_tc else "tensor (bf16, measured)",
            "mma": "kind::f8f6f4 (E4M3 weights, hi + lo E4M3 activation terms)" if mma == "f8" else "kind::f16",
            "note": "router + route plan + grouped gate/up (SwiGLU epilogue) + grouped down + shared + combine; "
                    "tensor_frac against the measured dense BF16 peak"}
    if agree is not None:
        res["vs_f16_kernel"] = agree
    return res


def bench_hc(dev, args):
    """Secondary: the FFN boundary around the MoE -- mHC collapse + post-attention
    RMSNorm before the router (2 launches), hc expand after the MoE (1 launch) --
    at T = 1 (decode), 256 (the reference's profiled prefill) and 2048.  Inputs
    rotate through enough sets to exceed L2 (fn sets at T = 1, states above)."""
    import torch

    from glm53_flash_mlx_b200 import _native as N
    from glm53_flash_mlx_b200 import synthetic as S

    lib = N.lib()
    peaks = measured_peaks()
    K = 4 * H
    stream = torch.cuda.Stream(device=dev)
    res = {}
    plan = {1: (192, 20), 256: (16, 20), 2048: (4, 10)}
    for T in (int(v) for v in args.hc_tokens.split(",")):
        sets, reps = plan.get(T, (4, 10))
        n_fn = sets if T == 1 else 1
        fns = [S.random_bf16((24, K), seed=5000 + i, device=dev, std=1.0 / 128) for i in range(n_fn)]
        scale = torch.tensor([1.0, 0.8, 1.5], dtype=torch.float32, device=dev)
        base = torch.randn(24, generator=torch.Generator(device=dev).manual_seed(5), device=dev) * 0.5
        norm_w = S.random_bf16((H,), seed=5999, device=dev, std=0.1) + 1.0
        states = [S.random_bf16((T, 4, H), seed=6000 + i, device=dev) for i in range(sets)]
        moes = [S.random_bf16((T, H), seed=7000 + i, device=dev) for i in range(sets)]
        collapsed = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        normalized = torch.empty_like(collapsed)
        post = torch.empty((sets, T, 4), dtype=torch.float32, device=dev)
        comb = torch.empty((sets, T, 4, 4), dtype=torch.float32, device=dev)
        outs = [torch.empty((T, 4, H), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        ws_bytes = lib.glm53_hc_collapse_workspace_bytes(T, H)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)

        def collapse(i, s):
            N.check(lib.glm53_hc_collapse_norm(
                states[i].data_ptr(), T, H, 4, fns[i % n_fn].data_ptr(), scale.data_ptr(), base.data_ptr(), 20,
                1e-6, 1e-6, norm_w.data_ptr(), 1e-6, collapsed.data_ptr(), normalized.data_ptr(),
                post[i].data_ptr(), comb[i].data_ptr(), ws.data_ptr(), ws_bytes, s), "glm53_hc_collapse_norm")

        def expand(i, s):
            N.check(lib.glm53_hc_expand(moes[i].data_ptr(), states[i].data_ptr(), post[i].data_ptr(),
                                        comb[i].data_ptr(), T, H, 4, outs[i % 2].data_ptr(), s), "glm53_hc_expand")

        c_ms = time_stage_graph(collapse, sets, reps, stream, dev)
        e_ms = time_stage_graph(expand, sets, reps, stream, dev)
        c_bytes = T * 4 * H * 2 + 24 * K * 2 + H * 2 + 2 * T * H * 2 + T * 20 * 4
        e_bytes = T * H * 2 + 2 * T * 4 * H * 2 + T * 20 * 4
        res[f"T{T}"] = {
            "collapse_norm_us": round(c_ms * 1e3, 2), "collapse_norm_bytes": c_bytes,
            "collapse_norm_hbm_frac": round(c_bytes / (c_ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
            "expand_us": round(e_ms * 1e3, 2), "expand_bytes": e_bytes,
            "expand_hbm_frac": round(e_bytes / (e_ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
        }
        del fns, states, moes, outs, ws
    if 256 in (int(v) for v in args.hc_tokens.split(",")):
        res["post_attention_q256"] = bench_dsa_output(dev, stream, peaks)
        res["T256"]["reference_m3ultra_ms"] = {"ffn_hc_collapse": 0.435, "post_attention_norm": 0.2255}
        if not args.no_cpu:
            res["cpu_oracle_T256"] = cpu_hc(256)
    res["note"] = ("glm53_hc_collapse_norm (hc_mix_kernel + hc_finish_kernel) and glm53_hc_expand, each timed "
                   "alone in CUDA graphs of one call per input set; fraction of measured HBM copy bandwidth")
    return res


def cpu_hc(T: int) -> dict:
    """The CPU restatement (oracle port) of the collapse + RMSNorm and of the hc
    expand on seeded inputs of T tokens, all host threads, a few repetitions."""
    import oracle as O

    rng = np.random.default_rng(9)
    K = 4 * H
    state = O.bf16_from_f32(rng.standard_normal((T, 4, H)).astype(np.float32))
    fn = O.bf16_from_f32((rng.standard_normal((24, K)) / np.sqrt(K)).astype(np.float32))
    scale = np.array([1.0, 0.8, 1.5], np.float32)
    base = (rng.standard_normal(24) * 0.5).astype(np.float32)
    norm_w = O.bf16_from_f32((1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    moe = O.bf16_from_f32(rng.standard_normal((T, H)).astype(np.float32))
    threads = O.default_threads()
    O.hc_collapse_norm(state[:1], fn, scale, base, norm_w, threads=threads)  # warm
    reps, t0 = 3, time.perf_counter()
    for _ in range(reps):
        _, _, post, comb, _ = O.hc_collapse_norm(state, fn, scale, base, norm_w, threads=threads)
    c_s = (time.perf_counter() - t0) / reps
    t0 = time.perf_counter()
    for _ in range(reps):
        O.hc_expand(moe, state, post, comb)
    e_s = (time.perf_counter() - t0) / reps
    return {"collapse_norm_us": round(c_s * 1e6, 1), "expand_us": round(e_s * 1e6, 1), "cores": threads,
            "expand_cores": 1, "kind": "port",
            "sample": f"T = {T}: collapse + norm on {threads} host threads (double-precision dot products), "
                      f"expand single-threaded, mean of {reps}"}


def bench_dsa_output(dev, stream, peaks):
    """The reference's post-attention seam at its geometry (Q256: 64 heads x 256
    rows x 256 values, o_proj [4096, 16384], 4 branches): head-major layout,
    block-FP8 o_proj (tcgen05 GEMM) and hc expand, through
    DSAOutputProjection.execute_hc; four weight sets (256 MB) rotate past L2."""
    import torch

    import glm53_flash_mlx_b200 as G
    from glm53_flash_mlx_b200 import synthetic as S

    heads, rows, dim, hidden, sets = 64, 256, 256, 4096, 4
    weights = [S.random_block_fp8(hidden, heads * dim, seed=8000 + i, device=dev) for i in range(sets)]
    hms = [S.random_bf16((heads, rows, dim), seed=8100 + i, device=dev) for i in range(sets)]
    residual = S.random_bf16((rows, 4, hidden), seed=8200, device=dev)
    post = torch.rand((rows, 4), generator=torch.Generator(device=dev).manual_seed(1), device=dev) * 2
    comb = torch.rand((rows, 4, 4), generator=torch.Generator(device=dev).manual_seed(2), device=dev)
    plan = G.DSAOutputProjection()

    def step(i, s):
        w, sc = weights[i % sets]
        plan.execute_hc(hms[i % sets], w, sc, residual, post, comb)

    ms = time_stage_graph(step, sets, 10, stream, dev)
    flops = 2 * rows * hidden * heads * dim
    bytes_ = hidden * heads * dim + rows * heads * dim * 2 * 3 + rows * hidden * 2 * 10
    del weights, hms
    return {"us": round(ms * 1e3, 2), "flops": flops, "tflops": round(flops / (ms / 1e3) / 1e12, 1),
            "bf16_frac": round(flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops"], 4), "algorithmic_bytes": bytes_,
            "reference_m3ultra_ms": 25.45,
            "note": "head-major layout + o_proj + hc expand (DSAOutputProjection.execute_hc), 3 launches + the "
                    "GEMM's activation conversion; reference_m3ultra_ms = the reference's native plan on its "
                    "M3 Ultra (bench-results/m3ultra512-native-prefill-post-attention-hc-20260909.json)"}


# ---------------------------------------------------------------------------
# CPU side (oracle port of the reference kernels)
# ---------------------------------------------------------------------------


def host_layer(layer):
    """Host copies of one layer's weights for the CPU restatement."""
    bank = layer["bank"]
    return {
        "bank": tuple(t.cpu().numpy() for t in (bank.gate_up_weight, bank.gate_up_scale_inv, bank.down_weight,
                                                bank.down_scale_inv)),
        "shared": tuple(t.cpu().numpy() for t in layer["shared"]),
        "router_w": layer["router_w"].cpu().numpy(),
        "router_b": layer["router_b"].cpu().numpy(),
    }


def cpu_token(O, hl, x_bits, threads):
    idx, sc, _, _ = O.router(x_bits[None, :], hl["router_w"], hl["router_b"], top_k=TOP_K, threads=threads)
    return O.packed_decode_moe(x_bits, idx[0], sc[0], hl["bank"], hl["shared"], LIMIT, threads=threads)


def cpu_baseline(hl, xs_bits, seconds: float) -> dict:
    import oracle as O

    threads = O.default_threads()
    cpu_token(O, hl, xs_bits[0], threads)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_token(O, hl, xs_bits[n % len(xs_bits)], threads)
        n += 1
        el = time.perf_counter() - t0
        if (el >= seconds and n >= 2) or n >= 2000:
            break
    return {"value": round(n / el, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} decode tokens through one config-2 layer (router + 8 experts + shared), "
                      f"{el:.1f} s on {threads} host threads"}


def bench_reference(args, world, rank, local):
    """--impl reference: the CPU restatement of the reference kernels."""
    import torch

    import oracle as O
    from glm53_flash_mlx_b200 import synthetic as S

    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    layer = build_layers(1, 1000, dev)[0]
    hl = host_layer(layer)
    xs = S.random_bf16((POOL, H), seed=77, device=dev)
    xs_bits = xs.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    del layer
    threads = O.default_threads()
    # each step is one decode token through the CPU restatement (~13 ms on 16
    # threads); warm-up and timed tokens are capped by time so that any
    # --steps / --warmup finishes within a few minutes
    warm_budget_s, timed_budget_s = 10.0, 120.0
    w0 = time.perf_counter()
    warm = 0
    while warm < args.warmup and time.perf_counter() - w0 < warm_budget_s:
        cpu_token(O, hl, xs_bits[warm % POOL], threads)
        warm += 1
    t0 = time.perf_counter()
    done = 0
    while done < args.steps and (done == 0 or time.perf_counter() - t0 < timed_budget_s):
        cpu_token(O, hl, xs_bits[done % POOL], threads)
        done += 1
    el = time.perf_counter() - t0
    value = done / el
    return {
        "metric": "FP8 MoE decode layer tokens/s (L=1, batch 1)", "value": round(value, 3), "unit": "tokens/s",
        "impl": "reference", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / done * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3xbf16->f32", "data": "synthetic",
        "config": config_block(args, 1),
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{done} timed decode tokens of the {args.steps} requested (one config-2 layer "
                                   f"each; at most {timed_budget_s:.0f} s) after {warm} warm-up tokens "
                                   f"(at most {warm_budget_s:.0f} s), {threads} host threads"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def config_block(args, world, graph=None):
    workload = ("config2: packed decode MoE layer, L=1, batch 1 (router + top-8 of 288 + shared)" if world == 1 else
                f"config2 layer expert-parallel over {world} GPUs (config 4 at batch 1 per rank): {E // world} "
                "experts per GPU, router and shared expert replicated; dispatch and combine as NVLink peer-memory "
                "stores with arrival counters (CUDA IPC buffers)")
    return {"workload": workload,
            "hidden": H, "moe_intermediate": I, "experts": E, "top_k": TOP_K, "swiglu_limit": LIMIT,
            "weights": "E4M3 + FP32 128x128 block scales, seeded N(0,0.02) amax/448",
            "global_batch": 1 * world, "seq_len": 1,
            "l2": f"inputs larger than L2: {args.layers} distinct layers rotated "
                  f"({args.layers * 5.44 / world:.1f} GB of experts per GPU) and a {POOL}-vector activation pool; "
                  "no flush",
            "graph": graph or f"{GRAPH_STEPS} decode steps (router + decode each, stream-ordered) per CUDA graph",
            "parallelism": f"ep{world}" if world > 1 else "single"}


def main():
    args = parse_args()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(bench_reference(args, world, rank, local)), flush=True)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    if args.linear_only:
        import torch

        if rank == 0:
            print(json.dumps({"linear_config1_5": bench_linear(torch.device("cuda", local), args)}), flush=True)
        return
    if args.batched_only:
        import torch

        dev = torch.device("cuda", local)
        layers = build_layers(args.layers, 1000 + 101 * rank, dev, args.experts)
        if rank == 0:
            res = {"batched_decode": bench_batched(layers, dev, args),
                   "ep_batched": {f"B{B}": bench_ep_batched(layers, dev, args, 1, 0, int(B))
                                  for B in args.batched_tokens.split(",") if int(B) in (16, 64)}}
            print(json.dumps(res), flush=True)
        return
    if args.hc_only:
        import torch

        if rank == 0:
            print(json.dumps({"ffn_boundary": bench_hc(torch.device("cuda", local), args)}), flush=True)
        return
    if args.prefill_only:
        import torch

        dev = torch.device("cuda", local)
        layers = build_layers(args.layers, 1000 + 101 * rank, dev, args.experts)
        if rank == 0:
            res = {}
            for T in (int(t) for t in args.prefill_tokens.split(",")):
                if args.prefill_mma in ("f16", "both"):
                    res[f"prefill_{T}"] = bench_prefill(layers, dev, args, T)
                if args.prefill_mma in ("f8", "both"):
                    res[f"prefill_{T}_f8"] = bench_prefill(layers, dev, args, T, "f8")
            print(json.dumps(res), flush=True)
        return
    if world > 1:
        res = bench_ep(args, world, rank, local)
        layers = xs = None
    else:
        res, layers, xs = bench_b200(args, world, rank, local)
    line = {
        "metric": "FP8 MoE decode layer tokens/s (L=1, batch 1)",
        "value": round(res["value"], 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(res["t_ms"] / args.steps, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3xbf16->f32",
        "data": "synthetic (seeded random-init weights of the config-2 shapes)",
        "config": config_block(args, world, res.get("graph")),
        "clocks": res["clocks"],
        "roofline": res["roofline"],
        "e2e": res["e2e"],
        "gpu_launches": res["gpu_launches"],
    }
    base = {"value", "t_ms", "clocks", "roofline", "e2e", "gpu_launches", "graph"}
    for k, v in res.items():  # secondary measurements (stages, prefill, sweeps, batched, boundary)
        if k not in base:
            line[k] = v
    if rank == 0 and world == 1 and not args.no_cpu:
        import torch

        hl = host_layer(layers[0])
        xs_bits = xs.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        line["cpu_baseline"] = cpu_baseline(hl, xs_bits, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
