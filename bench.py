"""Benchmark of the B200 EXL3 routed-MoE path (48-layer MoE decode stack).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch T] [--impl ours|reference]

One step = one decode token batch (T tokens) through 48 MoE layers: per layer the router (x . Wr^T + Zipf(1.1)
logit bias, softmax top-10), the device expert cache step (8,000 slots over 24,576 (layer, expert) keys, LRU,
tier mask: picks in neither VRAM nor RAM get weight 0 and are logged), and the fused-dequant gate/up, SwiGLU, down
and weighted combine.  The whole step is captured once in a CUDA graph and replayed.  Inputs are resident in HBM
for `value`; `e2e` repeats the step through the public op API with the 48 layer inputs copied from pinned host
memory and the outputs copied back inside the timed region.  Synthetic data: seeded hash-generated EXL3 blobs,
N(0,1) activations.  Decode does not shard: under torchrun each rank runs an independent replica.

Further legs of the same line: decode at batch 2 and 4; a decode leg where cache misses fill
(`fill`: an 8-layer stack whose experts are all RAM-resident, so a miss is copied from pinned host memory into an LRU
slot inside the step); one prefill layer at 8,192 tokens (configs[2], with and without the router); the expert-parallel
prefill stack; the mixed-bitrate layer with the gated shared expert (configs[4]: decode T=1 and 4, prefill
T=2048); CPU baselines of decode and prefill.

--impl reference times the reference path's CPU restatement (oracle/, plain C) on the host cores on a bounded
sample of the same workload (the reference itself is SYCL for an Intel GPU and cannot run here).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen38-flash-next-b70-offload_b200"))

METRIC = "MoE decode tok/s bs1/4 & prefill tok/s @8k; % HBM / tensor-core roofline"
H, I, E, TOPK, K, L, S = 2048, 768, 512, 10, 3, 48, 8000
SEED = 0
GU_BYTES = (H // 16) * (2 * I // 16) * 8 * K * 4     # gate|up codes per expert: 1,179,648 B
BLOB = 1786368
PF_T = 8192          # configs[2] prefill chunk
# DRAM bytes (read + write) of one decode gate-up launch at batch 1, from one ncu capture of gu_cluster_kernel<3> on
# the same per-layer work (4-layer stack): dram__bytes_read.sum + dram__bytes_write.sum
GU_TRAFFIC_BS1 = 11997696
PF_KEY0 = 1 << 20    # blob keys of the prefill layer (distinct from the decode stack's)
# DRAM bytes (read + write) of one prefill gate-up GEMM launch (prefill_gemm_kernel<0>) on the configs[2] layer at
# 8,192 tokens, from one ncu capture of the bench's own prefill run (997,299,968 read + 124,593,664 written)
PF_GU_TRAFFIC = 1121893632
# router weight std: x . Wr then has the std of a standard Gumbel variable (pi / sqrt(6) = 1.28), so -1.1 ln(rank) +
# router noise makes each layer's top-10 a Zipf(1.1)-like Plackett-Luce sample and picks miss the 8,000-slot cache
WR_STD = 1.2825498 / (2048 ** 0.5)


def per_layer_slots(li: int, slots: int, layers: int) -> int:
    """Slots the decode stack gives layer li: its hottest Zipf ranks, slots / layers each (the first slots % layers
    layers one more)."""
    return slots // layers + (1 if li < slots % layers else 0)


def decode_config(T: int, world: int) -> dict:
    """The decode workload as both arms report it (same keys, same values)."""
    return {"workload": f"configs[1]: 48-layer MoE decode stack, batch {T}", "tokens_per_step": T, "layers": L,
            "H": H, "I": I, "experts": E, "topk": TOPK, "K": K, "slots": S, "keys": L * E,
            "parallelism": f"replicas x{world}",
            "router": "in the step: logits x . Wr^T + per-layer Zipf(1.1) bias, softmax top-10",
            "tier": "ram_res = 0 except each layer's safe expert: a pick in neither VRAM nor RAM is masked (safe "
                    "expert, weight 0) and logged, no fill runs in the timed step (the 'fill' leg times fills)"}


def cpu_info() -> dict:
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    import torch
    return {"cpu_model": model, "os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads()}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region (clock record for the JSON line)."""

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.p = None
        fd, self.path = tempfile.mkstemp(prefix="exl3b_clocks_", suffix=".csv")
        os.close(fd)

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        time.sleep(0.25)
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                c = [v.strip() for v in line.split(",")]
                if len(c) >= 9:
                    rows.append(c)
        os.unlink(self.path)
        if not rows:
            return None
        sm = sorted(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        reasons = set()
        for r in rows:
            for name, v in (("hw_slowdown", r[5]), ("hw_thermal_slowdown", r[6]), ("sw_thermal_slowdown", r[7]),
                            ("sw_power_cap", r[8])):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": float(rows[0][2]), "samples": len(rows),
                "reasons": sorted(reasons)}


# ------------------------------------------------------------------------------------------------ setup
def build_stack(dev, T):
    """Device state of the 48-layer decode stack: warm 8,000-slot cache (each layer's hottest experts by Zipf rank,
    the layer's safe expert pinned), tier flags (RAM tier empty: non-cached picks are masked), routers, inputs."""
    import torch
    from exl3b200 import ExpertStore, synth
    from exl3b200 import ops as X

    st = ExpertStore(H, I, K, E, S, device=dev, max_layers=L)
    # layer tables without a host arena: non-resident experts are never RAM-resident here (ram_res = 0), so the
    # tier mask guarantees no kernel dereferences their table entry (exl3_moe.a8.sycl:762-765 contract)
    per = [per_layer_slots(li, S, L) for li in range(L)]
    keys, slot = [], 0
    ptrs = torch.zeros(L * E, dtype=torch.int64)
    slot_of = torch.full((L * E,), -1, dtype=torch.int32)
    slot_key = torch.full((S,), -1, dtype=torch.int32)
    slot_last = torch.zeros(S, dtype=torch.int32)
    safe = torch.zeros(L, dtype=torch.int32)
    for li in range(L):
        st.layer_index[f"model.layers.{li}.mlp"] = li
        rank = synth.zipf_rank(E, li, SEED)
        safe[li] = int(rank[0])
        for j in range(per[li]):
            e = int(rank[j])
            key = li * E + e
            keys.append(key)
            slot_of[key] = slot
            slot_key[slot] = key
            ptrs[key] = st.slot_base + slot * st.blob
            if j == 0:
                slot_last[slot] = 0x7FFFFFFF          # safe expert pinned in VRAM
            slot += 1
    synth.fill_blobs(st.slots, SEED, keys, H, I, K)
    st.ptrs_all.copy_(ptrs.to(dev))
    st.slot_of_dev.copy_(slot_of.to(dev))
    st.slot_key.copy_(slot_key.to(dev))
    st.slot_last.copy_(slot_last.to(dev))
    ram_res = torch.zeros(L * E, dtype=torch.uint8)
    for li in range(L):
        ram_res[li * E + int(safe[li])] = 1
    ring = torch.zeros(1 + (1 << 16), dtype=torch.int32, device=dev)
    X.moe_set_tier(ram_res.to(dev), ring, safe.to(dev))
    wr = torch.stack([synth.router_weight(E, H, WR_STD, SEED + 17 * li) for li in range(L)]).to(dev)
    bias = torch.stack([synth.zipf_bias(E, li, SEED) for li in range(L)]).to(dev)
    xs = torch.stack([synth.activations(T, H, 1000 + li) for li in range(L)]).to(dev)
    torch.cuda.synchronize(dev)
    return st, wr, bias, xs, ring


def step_fn(st, wr, bias, xs, outs, routes, routed=False):
    """One decode step through the public API, per layer: the router op then ExpertStore.forward_cached (the
    plugin's two calls), or with routed=True ExpertStore.forward_cached_routed (router and cached MoE in one call);
    outputs written into the step's output buffer.  routes receives each layer's (ids, w) after the tier mask's
    rewrite."""
    import torch
    keys = list(st.layer_index)
    routes.clear()
    for li in range(L):
        if routed:
            _, ids, w = st.forward_cached_routed(keys[li], xs[li], wr[li], bias[li], TOPK, out=outs[li])
        else:
            ids, w = torch.ops.exl3b200_moe.router_topk(xs[li], wr[li], bias[li], TOPK)
            st.forward_cached(keys[li], xs[li], ids, w, out=outs[li])
        routes.append((ids, w))


def measure_decode(st, wr, bias, xs, ring, args, dev, local, clocks=True, routed=False):
    """Graph-captured decode step timed over args.steps replays (device time), then end to end through the public
    ops with pinned-host inputs and outputs, then the per-phase device time of an eager pass (profile events)."""
    import ctypes
    import torch
    from exl3b200 import _lib
    T = xs.shape[1]
    outs = torch.empty_like(xs)
    routes = []
    # warm-up (also the cache's LRU history), then capture
    for _ in range(max(args.warmup, 3)):
        step_fn(st, wr, bias, xs, outs, routes, routed)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        step_fn(st, wr, bias, xs, outs, routes, routed)
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    graph_routes = []
    with torch.cuda.graph(g):
        step_fn(st, wr, bias, xs, outs, graph_routes, routed)
    for _ in range(args.warmup):
        g.replay()
    ring0 = int(ring[0].item())
    torch.cuda.synchronize(dev)
    clk = Clocks(local) if clocks else None
    if clk:
        clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    clk_rec = clk.stop() if clk else None
    ms = e0.elapsed_time(e1) / args.steps
    masked = (int(ring[0].item()) - ring0) / (args.steps * L * T * TOPK)
    id_buf = torch.stack([r[0] for r in graph_routes])
    w_buf = torch.stack([r[1] for r in graph_routes])
    ids_np, w_np = id_buf.cpu().numpy(), w_buf.cpu().numpy()
    distinct = [len({int(e) for e, ww in zip(ids_np[li].ravel(), w_np[li].ravel()) if ww != 0.0}) for li in range(L)]
    # e2e: host inputs -> device, graph replay, outputs -> host, every step
    hx = xs.cpu().pin_memory()
    ho = torch.empty_like(outs, device="cpu").pin_memory()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e2.record()
    for _ in range(args.steps):
        xs.copy_(hx, non_blocking=True)
        g.replay()
        ho.copy_(outs, non_blocking=True)
    e3.record()
    torch.cuda.synchronize(dev)
    ms_e2e = e2.elapsed_time(e3) / args.steps
    # per-phase device time: events recorded by the library around its kernels on the launch stream, in an eager pass
    # of the same step queued behind a GPU sleep so that no launch gap is timed
    L_ = _lib.lib()
    keys = list(st.layer_index)
    gu_ms, dn_ms, rp_ms = [], [], []
    for _ in range(2):
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(L)]
        for row in evs:
            for ev in row:
                ev.record()
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(int(40e6))
        for li in range(L):
            ids, w = torch.ops.exl3b200_moe.router_topk(xs[li], wr[li], bias[li], TOPK)
            L_.exl3b_set_profile_events(*[ctypes.c_void_p(ev.cuda_event) for ev in evs[li]])
            st.forward_cached(keys[li], xs[li], ids, w)
        L_.exl3b_set_profile_events(None, None, None, None)
        torch.cuda.synchronize(dev)
        for li in range(L):
            rp_ms.append(evs[li][0].elapsed_time(evs[li][1]))
            gu_ms.append(evs[li][1].elapsed_time(evs[li][2]))
            dn_ms.append(evs[li][2].elapsed_time(evs[li][3]))
    del g
    return {"T": T, "ms": ms, "ms_e2e": ms_e2e, "masked": masked, "distinct": distinct, "id_buf": id_buf,
            "w_buf": w_buf, "gu_ms": gu_ms, "dn_ms": dn_ms, "rp_ms": rp_ms, "clocks": clk_rec,
            "h2d": int(xs.numel() * 2), "d2h": int(outs.numel() * 2)}


def prefill_cpu_baseline(arena, x, ids, w, T, seconds=20.0):
    """The CPU restatement (oracle/, C, prefill semantics: pick outputs rounded to fp16) on the host cores: the first
    tokens of the same layer (same blobs, routing and inputs), experts on parallel threads, as many tokens as fit the
    time budget (at least 256); tok/s of that sample."""
    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.lib()
    threads = os.cpu_count() or 1
    blobs_np = arena.cpu().numpy()
    blobs = [blobs_np[e] for e in range(E)]
    xb = x.cpu().view(torch.int16).numpy().view(np.uint16)
    idn, wn = ids.cpu().numpy(), w.cpu().numpy()
    t0 = time.perf_counter()
    O.moe_layer_fast(xb, idn, wn, blobs, H, I, K, y_half=True, threads=threads, rows=np.arange(64))
    probe = time.perf_counter() - t0
    n = int(min(T, max(256, 64 * seconds / max(probe, 1e-3) / 2)))
    n = 64 * max(1, n // 64)
    t0 = time.perf_counter()
    O.moe_layer_fast(xb, idn, wn, blobs, H, I, K, y_half=True, threads=threads, rows=np.arange(n))
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 2), "unit": "tok/s (one layer)", "cores": threads, "kind": "port",
            "sample": f"first {n} of the {T} tokens of the configs[2] layer (same blobs, routing and inputs), experts on "
                      f"{threads} threads, {dt:.1f} s wall; a rate, not extrapolated", **cpu_info()}


def measure_prefill(dev, local, iters=10, warmup=3, T=PF_T, cpu_leg=False):
    """one MoE layer, 8192-token prefill chunk, all 512 experts resident, router logits ~ N(0,1) plus a
    per-expert N(0,1.5) bias.  The layer (moe_forward on the router's picks: the grouped tcgen05 GEMM path) is timed
    with device events; e2e adds the host -> device copy of x and the device -> host copy of the output per call."""
    import ctypes
    import torch
    from exl3b200 import _lib, synth
    arena = torch.empty((E, BLOB), dtype=torch.uint8, device=dev)
    synth.fill_blobs(arena, SEED, [PF_KEY0 + e for e in range(E)], H, I, K)
    ptrs = (arena.data_ptr() + torch.arange(E, dtype=torch.int64) * BLOB).to(dev)
    x = synth.activations(T, H, 3000).to(dev)
    wr = synth.router_weight(E, H, 1.0 / H ** 0.5, SEED + 999).to(dev)
    bias = synth.normal_bias(E, 1.5, SEED).to(dev)
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(2):   # warm: the first call loads the kernels
        ids, w = torch.ops.exl3b200_moe.router_topk(x, wr, bias, TOPK)
    torch.cuda.synchronize(dev)
    r0.record()
    for _ in range(5):
        ids, w = torch.ops.exl3b200_moe.router_topk(x, wr, bias, TOPK)
    r1.record()
    torch.cuda.synchronize(dev)
    router_ms = r0.elapsed_time(r1) / 5
    fwd = torch.ops.exl3b200_moe.moe_forward
    for _ in range(warmup):
        out = fwd(x, ids, w, ptrs, I, K, E)
    torch.cuda.synchronize(dev)
    clk = Clocks(local)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        out = fwd(x, ids, w, ptrs, I, K, E)
    e1.record()
    torch.cuda.synchronize(dev)
    clk_rec = clk.stop()
    ms = e0.elapsed_time(e1) / iters
    hx = x.cpu().pin_memory()
    ho = torch.empty_like(out, device="cpu").pin_memory()
    torch.cuda.synchronize(dev)
    e0.record()
    for _ in range(iters):
        x.copy_(hx, non_blocking=True)
        out = fwd(x, ids, w, ptrs, I, K, E)
        ho.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    ms_e2e = e0.elapsed_time(e1) / iters
    # phase times of the library's launches (align .. input transform | gate-up GEMM | down GEMM + combine)
    L_ = _lib.lib()
    ph = [[], [], []]
    for _ in range(3):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        for ev in evs:
            ev.record()
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(int(20e6))
        L_.exl3b_set_profile_events(*[ctypes.c_void_p(ev.cuda_event) for ev in evs])
        fwd(x, ids, w, ptrs, I, K, E)
        L_.exl3b_set_profile_events(None, None, None, None)
        torch.cuda.synchronize(dev)
        for k in range(3):
            ph[k].append(evs[k].elapsed_time(evs[k + 1]))
    ph = [sum(v) / len(v) for v in ph]
    # the layer with its router, as one call sequence (router then MoE), device time
    e0.record()
    for _ in range(iters):
        ids_r, w_r = torch.ops.exl3b200_moe.router_topk(x, wr, bias, TOPK)
        out = fwd(x, ids_r, w_r, ptrs, I, K, E)
    e1.record()
    torch.cuda.synchronize(dev)
    ms_router = e0.elapsed_time(e1) / iters
    cnt = torch.bincount(ids.flatten().long(), minlength=E)
    _, tc, src = peaks()
    flops = 2.0 * T * TOPK * 3 * H * I
    gu_flops = 2.0 * T * TOPK * 2 * H * I
    gu_ach = gu_flops / (ph[1] * 1e-3) / 1e12
    cpu = prefill_cpu_baseline(arena, x, ids, w, T) if cpu_leg else None
    del arena
    return {"tokens": T, "value": round(T * 1000.0 / ms, 1), "unit": "tok/s (one layer)", "ms_per_layer": round(ms, 4),
            "with_router": {"value": round(T * 1000.0 / ms_router, 1), "unit": "tok/s (one layer, router included)",
                            "ms_per_layer": round(ms_router, 4), "router_ms": round(router_ms, 3)},
            "cpu_baseline": cpu,
            "tflops": round(flops / (ms * 1e-3) / 1e12, 1), "layer_frac_of_peak": round(flops / (ms * 1e-3) / 1e12 / tc, 4),
            "e2e": {"value": round(T * 1000.0 / ms_e2e, 1), "unit": "tok/s (one layer)",
                    "h2d_bytes_per_step": int(x.numel() * 2), "d2h_bytes_per_step": int(out.numel() * 2)},
            "roofline": {"bound": "tensor", "achieved": round(gu_ach, 1), "peak": tc, "unit": "TFLOP/s",
                         "frac": round(gu_ach / tc, 4), "traffic": PF_GU_TRAFFIC if T == PF_T else None,
                         "kernel": "prefill_gemm_kernel<0>",
                         "peak_source": src + " bf16 burst", "algorithmic_flops_per_launch": gu_flops,
                         "avg_launch_us": round(ph[1] * 1e3, 1)},
            "phase_us": {"align_transform": round(ph[0] * 1e3, 1), "gateup_gemm": round(ph[1] * 1e3, 1),
                         "down_gemm_combine": round(ph[2] * 1e3, 1)},
            "router_ms": round(router_ms, 3), "active_experts": int((cnt > 0).sum()), "max_picks": int(cnt.max()),
            "launches_per_layer": 8, "clocks": clk_rec,
            "config": "configs[2]: 1 layer, 8192 tokens, 512 experts resident, top-10, K=3, logits N(0,1) + bias N(0,1.5)"}


def measure_prefill_ep(dev, local, world, rank, T_total, layers=48, iters=3, warmup=3, chunks=1):
    """expert-parallel prefill of the 48-layer stack, T_total tokens per batch split evenly over the ranks
    (strong scaling), the 512 experts sharded contiguously (rank d holds experts [d 512/N, (d+1) 512/N)); NCCL
    all-to-all dispatch and combine around each rank's grouped GEMMs (exl3b200.ep.EPPrefill).  Every layer has its
    own router, bias and inputs; the layers share one synthetic set of 512 experts (915 MB per layer, far above the
    126 MB L2, so sharing the bytes does not change what a layer costs).  Routing is computed before timing.  With
    one GPU the same stack runs through the single-GPU prefill.  With chunks > 1 each layer's batch is split into
    that many token ranges whose all-to-alls overlap the other chunks' expert GEMMs.  Device time, max over ranks."""
    import torch
    import torch.distributed as dist
    from exl3b200 import synth
    from exl3b200 import ops as X
    per = E // world
    arena = torch.empty((per, BLOB), dtype=torch.uint8, device=dev)
    synth.fill_blobs(arena, SEED, [PF_KEY0 + rank * per + e for e in range(per)], H, I, K)
    ptrs_local = (arena.data_ptr() + torch.arange(per, dtype=torch.int64) * BLOB).to(dev)
    T = T_total // world
    xs, routes = [], []
    for li in range(layers):
        x = synth.activations(T, H, 5000 + 97 * li + rank).to(dev)
        wr = synth.router_weight(E, H, 1.0 / H ** 0.5, SEED + 3000 + li).to(dev)
        bias = synth.normal_bias(E, 1.5, SEED + li).to(dev)
        ids, w = X.router_topk(x, wr, bias, TOPK)
        xs.append(x)
        routes.append((ids, w))
    torch.cuda.synchronize(dev)
    if world > 1:
        from exl3b200.ep import EPPrefill
        ep = EPPrefill(dist.group.WORLD, E, H, I, K, ptrs_local, max_tokens=T, chunks=chunks)
        run = lambda li: ep.forward(xs[li], *routes[li])
    else:
        run = lambda li: X.moe_prefill(xs[li], routes[li][0], routes[li][1], ptrs_local, I, K, E)
    for _ in range(warmup):
        for li in range(layers):
            run(li)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        for li in range(layers):
            run(li)
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / iters
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    phases, loads = None, None
    if world > 1:
        # one more pass, unchunked, with per-phase device events (outside the timed region), and each rank's expert
        # load: the picks it received over the stack
        ep.profile, ep.chunks = True, 1
        acc, picks = {}, 0
        for li in range(layers):
            run(li)
            for kname, v in ep.phase_ms().items():
                acc[kname] = acc.get(kname, 0.0) + v
            picks += ep.stats()["recv_picks"]
        ep.profile, ep.chunks = False, chunks
        t = torch.tensor([acc[kname] for kname in sorted(acc)] + [float(picks)], dtype=torch.float64, device=dev)
        allt = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allt, t)
        names = sorted(acc)
        phases = {n: round(max(float(a[i]) for a in allt) / layers * 1e3, 1) for i, n in enumerate(names)}
        loads = [int(a[-1]) for a in allt]
    flops = 2.0 * T_total * TOPK * 3 * H * I * layers
    _, tc, _ = peaks()
    out = {"tokens_per_batch": T_total, "layers": layers, "value": round(T_total * 1000.0 / ms, 1),
           "unit": "tok/s (48-layer stack)", "ms_per_step": round(ms, 3), "n_gpus": world, "scaling": "strong",
           "tflops_per_gpu": round(flops / (ms * 1e-3) / 1e12 / world, 1),
           "frac_of_peak_per_gpu": round(flops / (ms * 1e-3) / 1e12 / world / tc, 4),
           "parallelism": f"expert-parallel x{world} (NCCL all-to-all, {chunks} pipelined chunks per layer)"
           if world > 1 else "one GPU",
           "phase_us_per_layer_max_over_ranks": phases, "picks_received_per_rank": loads,
           "config": "configs[3]: 48 layers, logits N(0,1) + bias N(0,1.5), top-10, K=3, experts sharded by id"}
    del arena, xs, routes
    return out


def measure_fill(dev, args, layers=8):
    """Decode with cache fills: an 8-layer stack of configs[1] layers (H=2048, I=768, 512 experts, top-10, K=3,
    Zipf(1.1) routing), the same slots per layer as the 48-layer stack (1,333 here), every expert RAM-resident (the
    RAM tier holds all keys), so a pick that misses VRAM is copied from its pinned host copy into the LRU slot inside
    the step (write-through read of the host copy in the same call).  The step is one CUDA graph of router + cached
    MoE call per layer; the cache state evolves from replay to replay."""
    import numpy as np
    import torch
    from exl3b200 import ExpertStore, synth
    from exl3b200 import ops as X
    Sf = round(S * layers / L)
    st = ExpertStore(H, I, K, E, Sf, device=dev, max_layers=layers)
    stage = torch.empty((E, BLOB), dtype=torch.uint8, device=dev)
    synth.fill_blobs(stage, SEED, list(range(E)), H, I, K)
    host = stage.cpu()
    del stage
    keys = []
    for li in range(layers):
        key = f"model.layers.{li}.mlp"
        st.add_layer(key).copy_(host)   # the layers share one set of expert bytes (timing does not depend on them)
        keys.append(key)
    del host
    for li, key in enumerate(keys):
        st.make_resident(key, synth.zipf_rank(E, li, SEED)[:per_layer_slots(li, Sf, layers)].tolist())
    ram_res = torch.ones(layers * E, dtype=torch.uint8, device=dev)
    ring = torch.zeros(1 + 4096, dtype=torch.int32, device=dev)
    safe = torch.tensor([int(synth.zipf_rank(E, li, SEED)[0]) for li in range(layers)], dtype=torch.int32, device=dev)
    X.moe_set_tier(ram_res, ring, safe)
    wr = torch.stack([synth.router_weight(E, H, WR_STD, SEED + 17 * li) for li in range(layers)]).to(dev)
    bias = torch.stack([synth.zipf_bias(E, li, SEED) for li in range(layers)]).to(dev)
    # new tokens every step (16 rotating input sets, copied into the step's input buffer before each replay): with
    # fixed inputs the routing would repeat and every pick would hit after the first step
    pool = torch.stack([torch.stack([synth.activations(1, H, 20000 + 97 * j + li) for li in range(layers)])
                        for j in range(16)]).to(dev)
    xs = pool[0].clone()
    outs = torch.empty_like(xs)

    def step():
        for li, key in enumerate(keys):
            ids, w = torch.ops.exl3b200_moe.router_topk(xs[li], wr[li], bias[li], TOPK)
            st.forward_cached(key, xs[li], ids, w, out=outs[li])

    try:
        for j in range(3):
            xs.copy_(pool[j])
            step()
        torch.cuda.synchronize(dev)
        # fills per layer call over a few eager steps (the fill list of each call, read after it)
        nf = []
        for j in range(4):
            xs.copy_(pool[3 + j])
            for li, key in enumerate(keys):
                ids, w = torch.ops.exl3b200_moe.router_topk(xs[li], wr[li], bias[li], TOPK)
                st.forward_cached(key, xs[li], ids, w, out=outs[li])
                nf.append(int(st.fill_list[0].item()))
        g = torch.cuda.CUDAGraph()
        s2 = torch.cuda.Stream(dev)
        s2.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s2):
            step()
        torch.cuda.current_stream(dev).wait_stream(s2)
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g):
            step()
        for j in range(args.warmup):
            xs.copy_(pool[j % 16])
            g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for j in range(args.steps):
            xs.copy_(pool[(7 + j) % 16])   # 8 KB device copy per step, inside the timed region
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / args.steps
        del g
    finally:
        X.moe_set_tier(torch.zeros(0, dtype=torch.uint8), torch.zeros(0, dtype=torch.int32),
                       torch.zeros(0, dtype=torch.int32))
    per_layer = ms / layers
    return {"value": round(1000.0 / ms, 2), "unit": f"tok/s ({layers}-layer stack, batch 1)", "ms_per_step": round(ms, 4),
            "us_per_layer": round(per_layer * 1e3, 2), "fills_per_layer_call": round(float(np.mean(nf)), 3),
            "config": f"{layers} configs[1] layers, {Sf} slots ({Sf // layers} per layer, as in the 48-layer stack), "
                      "every expert RAM-resident (misses fill from pinned host memory in the step), Zipf(1.1) routing, "
                      "router in the step, one CUDA graph per step, new tokens every step"}


def measure_config5(dev, iters=20):
    """one MoE layer, 512 routed experts with per-tensor K drawn from {2, 3, 4, 5} plus the always-on
    shared expert (K = 4) behind a sigmoid gate, hidden 2048, intermediate 768, top-10, N(0,1) activations, seed 7:
    decode at T = 1 and 4 and prefill at T = 2048.  A call is router + shared gate + MoE (moe_forward_shared, which
    runs the decode kernels below 256 tokens and the prefill GEMMs from 256).  Each call is timed alone with device
    events after a 256 MB write that evicts L2, with new tokens every call, so its codes come from HBM as in a stack.
    Roofline: decode on HBM bytes (the K-scaled blobs of the distinct experts read, shared expert included), prefill
    on tensor FLOPs (2 T (top-k + 1) 3 H I)."""
    import math
    import numpy as np
    import torch
    from exl3b200 import synth
    from exl3b200 import ops as X
    seed = 7
    kin = [synth.mixed_k(seed, e) for e in range(E)] + [(4, 4, 4)]
    sizes = [synth.blob_geometry(H, I, *k)["blob"] for k in kin]
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)
    arena = torch.empty(int(sum(sizes)), dtype=torch.uint8, device=dev)
    for e, (k, o, sz) in enumerate(zip(kin, offs, sizes)):
        synth.fill_blob(arena[int(o):int(o) + sz], seed, e, H, I, *k)
    ptrs = (arena.data_ptr() + torch.from_numpy(offs)).to(dev)
    kinfo = torch.tensor([synth.kinfo_pack(*k) for k in kin], dtype=torch.int32, device=dev)
    gate = synth.router_weight(1, H, 1.0 / math.sqrt(H), seed + 2).reshape(H).to(dev)
    wr = synth.router_weight(E, H, 1.0 / math.sqrt(H), seed + 3).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    hbm, tc, src = peaks()
    mean_bpw = float(sum(sizes[:E])) / E / BLOB * K
    res = {"config": "configs[4]: one layer, 512 routed experts with per-tensor K in {2,3,4,5} (P = .2/.6/.1/.1) plus "
                     "the shared expert (K=4, sigmoid gate), H=2048, I=768, top-10, seed 7; router and gate in the call; "
                     "L2 evicted before every call",
           "mean_routed_code_bits_per_weight_vs_K3_blob": round(mean_bpw, 3)}
    for T in (1, 4, 2048):
        xs = [synth.activations(T, H, seed + 100 + 7 * i).to(dev) for i in range(iters + 3)]
        times, byts = [], []
        for i, x in enumerate(xs):
            flush.fill_(i & 255)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            ids, w = X.router_topk(x, wr, None, TOPK)
            torch.ops.exl3b200_moe.moe_forward_shared(x, ids, w, ptrs, kinfo, gate, I, E)
            e1.record()
            torch.cuda.synchronize(dev)
            if i >= 3:
                times.append(e0.elapsed_time(e1))
                used = set(int(v) for v in ids.flatten().tolist()) | {E}
                byts.append(sum(sizes[e] for e in used))
        ms = float(np.mean(times))
        leg = {"value": round(T * 1000.0 / ms, 1), "unit": "tok/s (one layer)", "ms_per_layer": round(ms, 4)}
        if T < 256:
            b = float(np.mean(byts))
            leg["roofline"] = {"bound": "hbm", "achieved": round(b / (ms * 1e-3) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                               "frac": round(b / (ms * 1e-3) / 1e9 / hbm, 4), "bytes_per_call": int(b),
                               "peak_source": src}
        else:
            fl = 2.0 * T * (TOPK + 1) * 3 * H * I
            leg["roofline"] = {"bound": "tensor", "achieved": round(fl / (ms * 1e-3) / 1e12, 1), "peak": tc,
                               "unit": "TFLOP/s", "frac": round(fl / (ms * 1e-3) / 1e12 / tc, 4),
                               "flops_per_call": fl, "peak_source": src + " bf16 burst"}
        res[("decode_T" if T < 256 else "prefill_T") + str(T)] = leg
    del arena, flush
    return res


def run_ours(args):
    import torch
    import torch.distributed as dist
    from exl3b200 import synth
    from exl3b200 import ops as X

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    X.register()
    T = args.batch
    if args.only in ("prefill", "ep"):
        pf = measure_prefill(dev, local, T=args.pf_tokens) if args.only == "prefill" else \
            measure_prefill_ep(dev, local, world, rank, args.ep_tokens, chunks=args.ep_chunks)
        if rank == 0:
            print(json.dumps({"metric": METRIC, args.only if args.only == "prefill" else "prefill_ep": pf}), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    st, wr, bias, xs, ring = build_stack(dev, T)
    if world > 1:
        dist.barrier()
    d = measure_decode(st, wr, bias, xs, ring, args, dev, local)
    ms, ms_e2e = d["ms"], d["ms_e2e"]
    # the same step through the routed entry (router and cached MoE in one call per layer)
    d2 = measure_decode(st, wr, bias, xs, ring, args, dev, local, clocks=False, routed=True)
    routed_step = {"value": round(world * T * 1000.0 / d2["ms"], 2), "unit": "tok/s", "ms_per_step": round(d2["ms"], 4),
                   "e2e": {"value": round(world * T * 1000.0 / d2["ms_e2e"], 2), "unit": "tok/s"},
                   "step": "ExpertStore.forward_cached_routed per layer (picks selected inside the decode kernels)"}
    batches = {}
    if T == 1 and not args.no_bs4:
        for Tb in (2, 4):
            xb = torch.stack([synth.activations(Tb, H, 1000 + li) for li in range(L)]).to(dev)
            db = measure_decode(st, wr, bias, xb, ring, args, dev, local, clocks=False)
            hbm, _, _ = peaks()
            sb = sum(db["distinct"]) * BLOB
            batches[f"bs{Tb}"] = {
                "value": round(world * Tb * 1000.0 / db["ms"], 2), "unit": "tok/s", "ms_per_step": round(db["ms"], 4),
                "e2e": {"value": round(world * Tb * 1000.0 / db["ms_e2e"], 2), "unit": "tok/s",
                        "h2d_bytes_per_step": db["h2d"], "d2h_bytes_per_step": db["d2h"]},
                "distinct_experts_per_layer": round(sum(db["distinct"]) / L, 2),
                "layer_hbm": {"bytes_per_step": sb, "frac": round(sb / (db["ms"] * 1e-3) / 1e9 / hbm, 4)},
                "masked_pick_fraction": round(db["masked"], 4),
                "phase_us": {"route_prep": round(1e3 * sum(db["rp_ms"]) / len(db["rp_ms"]), 2),
                             "gateup": round(1e3 * sum(db["gu_ms"]) / len(db["gu_ms"]), 2),
                             "down_combine": round(1e3 * sum(db["dn_ms"]) / len(db["dn_ms"]), 2)}}
            del xb
    X.moe_set_tier(torch.zeros(0, dtype=torch.uint8), torch.zeros(0, dtype=torch.int32), torch.zeros(0, dtype=torch.int32))
    del st
    torch.cuda.empty_cache()
    fill = cfg5 = None
    if T == 1 and not args.no_fill:
        fill = measure_fill(dev, args)
        torch.cuda.empty_cache()
    if T == 1 and not args.no_config5:
        cfg5 = measure_config5(dev)
        torch.cuda.empty_cache()
    pf = pf_ep = None
    if not args.no_prefill:
        if world == 1:
            pf = measure_prefill(dev, local, T=args.pf_tokens, cpu_leg=rank == 0 and not args.no_cpu)
        pf_ep = measure_prefill_ep(dev, local, world, rank, args.ep_tokens, chunks=args.ep_chunks)
    hbm, tc, src = peaks()
    distinct = d["distinct"]
    avg_distinct = sum(distinct) / L
    gu_bytes = avg_distinct * GU_BYTES
    gu_s = (sum(d["gu_ms"]) / len(d["gu_ms"])) * 1e-3
    ach = gu_bytes / gu_s / 1e9
    # max over ranks; value = all ranks' tokens / slowest rank
    if world > 1:
        t = torch.tensor([ms, ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
    step_bytes = sum(distinct) * BLOB
    line = {
        "metric": METRIC, "value": round(world * T * 1000.0 / ms, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u32 codes -> fp16 (fp32 accumulate)",
        "data": "synthetic (seeded hash EXL3 blobs, N(0,1) bf16 activations, Zipf(1.1) router bias)",
        "config": decode_config(T, world),
        "step": "router_topk op + ExpertStore.forward_cached per layer (the plugin's two calls; the one-call routed entry "
                "is reported as 'routed')",
        "workload_stats": {"l2": f"working set per step {step_bytes / 1e6:.0f} MB of codes > 126 MB L2 (no flush "
                                 "needed)", "masked_pick_fraction": round(d["masked"], 4),
                           "distinct_experts_per_layer": round(avg_distinct, 2)},
        "e2e": {"value": round(world * T * 1000.0 / ms_e2e, 2), "unit": "tok/s",
                "h2d_bytes_per_step": d["h2d"], "d2h_bytes_per_step": d["d2h"]},
        "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s", "frac": round(ach / hbm, 4),
                     "traffic": GU_TRAFFIC_BS1 if T == 1 else None, "kernel": "gu_cluster_kernel<3> (decode gate-up)",
                     "peak_source": src,
                     "algorithmic_bytes_per_launch": int(gu_bytes), "avg_launch_us": round(gu_s * 1e6, 2)},
        "layer_hbm": {"bytes_per_step": step_bytes, "achieved_gbs": round(step_bytes / (ms * 1e-3) / 1e9, 1),
                      "frac": round(step_bytes / (ms * 1e-3) / 1e9 / hbm, 4),
                      "phase_us": {"route_prep": round(1e3 * sum(d["rp_ms"]) / len(d["rp_ms"]), 2),
                                   "gateup": round(1e3 * sum(d["gu_ms"]) / len(d["gu_ms"]), 2),
                                   "down_combine": round(1e3 * sum(d["dn_ms"]) / len(d["dn_ms"]), 2)}},
        "gpu_launches": args.steps * L * 4,
        "clocks": d["clocks"],
    }
    line["routed"] = routed_step
    line.update(batches)
    if fill is not None:
        line["fill"] = fill
    if cfg5 is not None:
        line["config5"] = cfg5
    if pf is not None:
        line["prefill"] = pf
    if pf_ep is not None:
        line["prefill_ep"] = pf_ep
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(d["id_buf"], d["w_buf"], T, seconds=args.cpu_seconds)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ CPU oracle
def cpu_baseline(id_buf, w_buf, T, seconds=20.0):
    """The CPU restatement (oracle/, C) on the host cores: layers of the bench step (the GPU run's routing after the
    cache mask; inputs and blobs regenerated from the same seeds) run in parallel threads (the C code releases the
    GIL), until about `seconds` of wall time; tok/s extrapolated to the 48-layer step."""
    import concurrent.futures as cf
    import numpy as np
    import torch
    from exl3b200 import synth
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.lib()
    threads = os.cpu_count() or 1
    ids_np, w_np = id_buf.cpu().numpy(), w_buf.cpu().numpy()
    nlay = max(1, min(L, 2 * threads))
    jobs = []
    for li in range(nlay):
        blobs = [None] * E
        for e in set(int(v) for v in ids_np[li].ravel()):
            blobs[e] = synth.make_blob(SEED, li * E + e, H, I, K).numpy()
        xb = synth.activations(T, H, 1000 + li).view(torch.int16).numpy().view(np.uint16)
        jobs.append((xb, ids_np[li].copy(), w_np[li].copy(), blobs))
    done = 0
    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(threads) as ex:
        while time.perf_counter() - t0 < seconds and done < 4 * L:
            batch = [jobs[(done + i) % nlay] for i in range(threads)]
            list(ex.map(_oracle_fast_job, batch))
            done += len(batch)
    dt = time.perf_counter() - t0
    tok_s = T * done / L / dt
    return {"value": round(tok_s, 5), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{done} layer calls of the bench step ({T} token(s), top-{TOPK}, the GPU run's masked routing), "
                      f"{threads} threads, {dt:.1f} s wall, extrapolated to 48 layers", **cpu_info()}


def tier_mask(ids, w, li):
    """The decode stack's tier mask on one layer's routing (in place): the stack holds each layer's hottest
    per_layer_slots Zipf ranks in VRAM and nothing else in RAM, so a pick of a colder expert becomes (safe expert,
    weight 0), safe = the layer's rank-0 expert; returns the number masked."""
    import numpy as np
    from exl3b200 import synth
    rank_order = synth.zipf_rank(E, li, SEED).numpy()
    rank = np.empty(E, np.int64)
    rank[rank_order] = np.arange(E)
    m = rank[ids] >= per_layer_slots(li, S, L)
    ids[m] = int(rank_order[0])
    w[m] = 0.0
    return int(m.sum())


def _oracle_fast_job(args):
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    x, ids, w, blobs = args
    ids = np.where(w == 0.0, -1, ids).astype(np.int32)   # weight-0 picks contribute exactly 0: not computed (as on the GPU)
    return O.moe_layer_fast(x, ids, w, blobs, H, I, K, threads=1)


def run_reference(args):
    """--impl reference: the reference path's CPU restatement (oracle/, C) on the host cores, rank 0 only.  A step
    runs one layer per host thread (up to 48), each layer one decode call of the bench's stack: the router
    restatement on the same seeded inputs, the stack's tier mask, the MoE layer.  ms_per_step is the time of those
    layers; value is tok/s of the 48-layer step, extrapolated from them (also given as its own field)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from exl3b200 import synth
    O.lib()
    T = args.batch
    threads = os.cpu_count() or 1
    nlay = max(1, min(L, threads))
    jobs, masked = [], 0
    for li in range(nlay):
        x = synth.activations(T, H, 1000 + li).view(torch.int16).numpy().view(np.uint16)
        wr = synth.router_weight(E, H, WR_STD, SEED + 17 * li).view(torch.int16).numpy().view(np.uint16)
        ids, w, _ = O.router(x, wr, synth.zipf_bias(E, li, SEED).numpy(), TOPK)
        ids, w = np.ascontiguousarray(ids, np.int32), np.ascontiguousarray(w, np.float32)
        masked += tier_mask(ids, w, li)
        blobs = [None] * E
        for e in set(int(v) for v, ww in zip(ids.ravel(), w.ravel()) if ww != 0.0):
            blobs[e] = synth.make_blob(SEED, li * E + e, H, I, K).numpy()
        jobs.append((x, ids, w, blobs))
    import concurrent.futures as cf
    times = []
    t_run = time.perf_counter()
    with cf.ThreadPoolExecutor(threads) as ex:
        for it in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            list(ex.map(_oracle_fast_job, jobs))
            dt = time.perf_counter() - t0
            if it >= args.warmup:
                times.append(dt)
    step_s = sum(times) / len(times)
    full_s = step_s * L / nlay
    v = T / full_s
    print(json.dumps({
        "metric": METRIC, "value": round(v, 5), "unit": "tok/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u32 codes -> fp16 (fp64 accumulate)", "impl": "reference",
        "data": "synthetic (same seeded workload)", "config": decode_config(T, int(os.environ.get("WORLD_SIZE", "1"))),
        "step": {"layers_per_step": nlay, "ms_per_48_layer_step_extrapolated": round(full_s * 1e3, 1),
                 "masked_pick_fraction": round(masked / (nlay * T * TOPK), 4),
                 "run_s": round(time.perf_counter() - t_run, 1)},
        "cpu_baseline": {"value": round(v, 5), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{nlay} of the 48 layers per step ({threads} threads, one layer each), "
                                   "tok/s extrapolated to 48 layers", **cpu_info()},
        "e2e": {"value": round(v, 5), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-bs4", action="store_true", help="skip the batch 2 and 4 decode legs")
    ap.add_argument("--no-fill", action="store_true", help="skip the decode leg whose misses fill")
    ap.add_argument("--no-config5", action="store_true", help="skip the configs[4] mixed-bitrate layer")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--ep-tokens", type=int, default=8192, help="configs[3] tokens per batch (8192 or 32768)")
    ap.add_argument("--ep-chunks", type=int, default=1, help="configs[3] pipelined token chunks per layer")
    ap.add_argument("--only", choices=["all", "decode", "prefill", "ep"], default="all",
                    help="decode: skip both prefill measurements; prefill: only the configs[2] layer; ep: only the "
                         "configs[3] expert-parallel stack (small profiling runs)")
    ap.add_argument("--layers", type=int, default=48, help="decode stack depth (48; fewer only for small profiling runs)")
    ap.add_argument("--slots", type=int, default=8000, help="device cache slots (8000; fewer for small profiling runs)")
    ap.add_argument("--pf-tokens", type=int, default=8192, help="configs[2] prefill tokens")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    global L, S
    L, S = args.layers, args.slots
    if args.only == "decode":
        args.no_prefill = True
    if L != 48 or S != 8000:   # small profiling stacks: the headline legs only
        args.no_fill = args.no_config5 = True
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
