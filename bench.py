#!/usr/bin/env python
"""Benchmark of the Qwen3-MoE layer hot path (BASELINE.json metric: MoE-layer tokens/s and the
fraction of the HBM roofline), one JSON line on stdout.

Workload ("C2"): a Qwen3-30B-A3B-shaped MoE layer at decode batch T
(default 64): hidden 2048, 128 experts, top-8 renormalised, moe_intermediate 768, gate/up Q4_K,
down Q6_K, weights ~N(0, 0.02) before quantisation, router f32 ~N(0, 0.02), activations ~N(0, 1).
A step is one pass over the MoE layers of a 48-layer model (48 distinct, resident layers of that
shape, the same T tokens into each), so every step streams ~48 x the distinct-expert bytes through
HBM (far above the 126 MB L2).  `value` = layer-tokens per second (T x layers x steps / time),
device-resident inputs, the 48 layer calls replayed as one CUDA graph.  `e2e` = the same through
the C-ABI calls from the host, per step the T x H f32 input copied host->device from pinned memory
and the last layer's output read back.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl ours|reference]

--impl reference times the CPU oracle (the stand-in for ggml's CPU mul_mat_id path, which is not
present in the reference tree) on the host cores, one layer call per step.
Under torchrun (N > 1) every rank runs an independent replica (weak scaling); rank 0 prints.
"""
from __future__ import annotations

import argparse
import datetime
import faulthandler
import hashlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
_T0 = time.time()


def log(msg):
    """Progress on stderr (stdout carries only the JSON line)."""
    print(f"[bench {time.time() - _T0:7.1f}s] {msg}", file=sys.stderr, flush=True)

H, I, E, K_USED = 2048, 768, 128, 8
Q4K, Q6K = 12, 14
DOWN_T = Q6K                                                      # Q4_K_M promotes ffn_down to Q6_K
PREPACK = True  # Q6_K down tensors repacked once at load by tmoe_prepack (TYPE_Q6_K_R8); --no-prepack


def down_type_gpu():
    """The down type the GPU arm's layers are created with (the packed type when --prepack)."""
    return 270 if PREPACK and DOWN_T == Q6K else DOWN_T
EXPERT_BYTES = 2 * I * (H // 256) * 144 + H * (I // 256) * 210  # 3,059,712
GATE_UP_BYTES = 2 * I * (H // 256) * 144                          # 1,769,472
DOWN_BYTES = H * (I // 256) * 210                                 # 1,290,240
ROUTER_BYTES = E * H * 4                                          # 1,048,576


def set_shape(name):
    """c2: the Qwen3-30B-A3B layer (the metric's config); 235b: the Qwen3-235B-A22B layer of config 4
    (hidden 4096, moe_intermediate 1536, 128 experts, top-8, all Q4_K)."""
    global H, I, DOWN_T, EXPERT_BYTES, GATE_UP_BYTES, DOWN_BYTES, ROUTER_BYTES
    H, I, DOWN_T = (4096, 1536, Q4K) if name == "235b" else (2048, 768, Q6K)
    down_block = 210 if DOWN_T == Q6K else 144
    GATE_UP_BYTES = 2 * I * (H // 256) * 144
    DOWN_BYTES = H * (I // 256) * down_block
    EXPERT_BYTES = GATE_UP_BYTES + DOWN_BYTES
    ROUTER_BYTES = E * H * 4


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--tokens", type=int, default=64)
    p.add_argument("--layers", type=int, default=48)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--seed", type=int, default=20261201)
    p.add_argument("--cpu-sample-s", type=float, default=15.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-sweep", dest="sweep", action="store_false",
                   help="decode mode at N = 1: skip the extra key that times T in {1, 4, 16, 64}")
    p.add_argument("--ctx", type=int, default=4096, help="model mode: the context each sequence decodes at")
    p.add_argument("--prefill", type=int, default=2048,
                   help="model mode: also time the prefill of one prompt of this many random tokens (0: skip)")
    p.add_argument("--mode", choices=["decode", "prefill", "streamed", "gguf", "model"], default="decode",
                   help="decode: C2 at T tokens (the metric's config); prefill: C2-shaped layer at T=8192 "
                        "(tensor roofline); streamed: config 5, skewed routing over 64 device slots of 128 experts; "
                        "gguf: loading the expert tensors of a C2-shaped GGUF file into HBM; model: config 3, the "
                        "whole Qwen3-30B-A3B-shaped model decoding --tokens sequences at --ctx context")
    p.add_argument("--slots", type=int, default=64)
    p.add_argument("--routing", default=None,
                   help="streamed mode: replay the layer steps of this tetraeder-routing v1 trace instead of the "
                        "Zipf routing (cyclically, one recorded step per bench step)")
    p.add_argument("--routing-layer", type=int, default=-1, help="the trace layer to replay (-1: the first one)")
    p.add_argument("--record-trace", default=None,
                   help="streamed mode: also write the routing of --steps steps as a tetraeder-routing v1 trace")
    p.add_argument("--shape", choices=["c2", "235b"], default="c2",
                   help="c2: the Qwen3-30B-A3B layer (the metric's config); 235b: config 4's layer shape")
    p.add_argument("--no-prepack", dest="prepack", action="store_false",
                   help="keep the Q6_K down tensors in ggml's layout (default: repacked once at load with "
                        "tmoe_prepack, the optional explicit repack of the boundary; the products are bit for bit "
                        "those of the ggml layout, and a one-GPU decode line also times the ggml layout)")
    p.add_argument("--no-c4", action="store_true",
                   help="decode mode: skip the config-4 line (the 235B-shaped layer, expert-parallel over the ranks "
                        "at N > 1) added to the C2 line")
    p.add_argument("--ep", choices=["a2a", "allreduce"], default="a2a",
                   help="N > 1: a2a = each rank its own --tokens, dispatched to the experts' ranks (all-to-all); "
                        "allreduce = the reference's EP mode, the same tokens on every rank, outputs summed")
    a = p.parse_args()
    global PREPACK
    # the large-batch modes and the reference arm (the CPU oracle on ggml's bytes) keep ggml's layout
    PREPACK = a.prepack and a.mode == "decode" and a.impl == "ours"
    set_shape(a.shape)
    if a.mode in ("prefill", "streamed") and a.tokens == 64:
        a.tokens = 8192
    if a.mode == "prefill" and a.layers == 48:
        a.layers = 4
    return a


def workload(args, n_gpus):
    if args.shape == "235b":
        name = {"decode": "C4 Qwen3-235B-A22B-shaped MoE layer, decode",
                "prefill": "C4 Qwen3-235B-A22B-shaped MoE layer, prefill",
                "streamed": "C4-shaped layer, streamed"}[args.mode]
        return {"workload": name, "tokens_per_layer_call": args.tokens, "n_embd": H, "n_ff": I, "n_expert": E,
                "n_expert_used": K_USED, "types": "gate/up/down Q4_K (this repo's quantiser)",
                "layers_per_step": args.layers,
                "l2": f"inputs larger than L2: {args.layers} distinct resident layers rotated each step",
                "parallelism": f"replicas x{n_gpus}" if n_gpus > 1 else "single GPU", "seed": args.seed}
    name = {"decode": "C2 Qwen3-30B-A3B MoE layer, decode",
            "prefill": "C2-shaped Qwen3-30B-A3B MoE layer, prefill (north-star tensor target)",
            "streamed": "C5 skewed large-batch stress, 64 of 128 experts in device slots"}[args.mode]
    types = "gate/up Q4_K, down Q6_K (this repo's quantiser)"
    if down_type_gpu() != DOWN_T:
        types += ("; down repacked once at load by tmoe_prepack (Q6_K_R8, 8-row fragment order, outside the timed "
                  "region)")
    return {"workload": name, "tokens_per_layer_call": args.tokens,
            "n_embd": H, "n_ff": I, "n_expert": E, "n_expert_used": K_USED,
            "types": types, "layers_per_step": args.layers,
            "l2": f"inputs larger than L2: {args.layers} distinct resident layers rotated each step",
            "parallelism": f"replicas x{n_gpus}" if n_gpus > 1 else "single GPU", "seed": args.seed}


# ---------------------------------------------------------------------------------------- clocks
class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        rows = []
        for line in open(self.path):
            f = [c.strip() for c in line.split(",")]
            if len(f) >= 9 and f[1].isdigit():
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [int(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": int(statistics.median(sm)), "sm_max_mhz": int(rows[0][2]), "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()) if rows else None,
                "reasons": reasons}


# ---------------------------------------------------------------------------------------- ours
def make_layers(torch, moe, n_layers, seed, device, world=1, rank=0, ggml_down=None):
    """n_layers C2 layers.  With world > 1 (expert parallelism) every rank draws the same router
    (the routing is replicated) and holds only its contiguous share of each layer's experts.  When
    the down tensors are repacked, ggml_down (a list) receives the ggml-layout originals."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    ge = torch.Generator(device=device)
    ge.manual_seed(seed + 1000003 * (rank + 1))
    per = E // world
    layers = []
    for _ in range(n_layers):
        rw = torch.randn((E, H), generator=g, device=device) * 0.02
        gate = moe.quantize(Q4K, torch.randn((per, I, H), generator=ge, device=device) * 0.02)
        up = moe.quantize(Q4K, torch.randn((per, I, H), generator=ge, device=device) * 0.02)
        down = moe.quantize(DOWN_T, torch.randn((per, H, I), generator=ge, device=device) * 0.02)
        if down_type_gpu() != DOWN_T:
            if ggml_down is not None:
                ggml_down.append(down)
            down = moe.prepack(down)
        layers.append((rw, moe.ExpertWeights(gate, up, down)))
    torch.cuda.synchronize()
    return layers


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import tetraeder_b200 as tb
    from tetraeder_b200 import moe

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    T, L = args.tokens, args.layers
    ep = world > 1
    a2a = ep and args.ep == "a2a"
    # N = 1: the layer on one GPU.  N > 1: the reference's EP mode, experts split contiguously over
    # the ranks, the same tokens on every rank, partial outputs summed with NCCL (strong scaling)
    # one GPU, decode, repacked down tensors: the ggml layout is timed too (key "ggml_layout")
    ggml_down = [] if world == 1 and args.mode == "decode" and down_type_gpu() != DOWN_T else None
    layers = make_layers(torch, moe, L, args.seed, dev, world, rank, ggml_down)
    log(f"{L} layers generated ({E // world} experts each on this rank)")
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed + 1 + (rank if a2a else 0))  # a2a: every rank has tokens of its own
    x_dev = torch.randn((T, H), generator=gen, device=dev)
    # e2e: every layer call takes its own input from pinned host memory and returns its output there
    x_host = torch.randn((L, T, H), generator=torch.Generator().manual_seed(args.seed + 2)).pin_memory()
    out_host = torch.empty((L, T, H), dtype=torch.float32).pin_memory()
    x_call = [torch.empty((T, H), device=dev) for _ in range(L)]
    layer = tb.MoeLayer(H, I, E, K_USED, gate_type=Q4K, up_type=Q4K, down_type=down_type_gpu(),
                        max_tokens=world * T if a2a else T, device=local_rank)
    outs = [torch.empty((T, H), device=dev) for _ in range(L)]
    ids = [torch.empty((T, K_USED), dtype=torch.int32, device=dev) for _ in range(L)]
    ws = [torch.empty((T, K_USED), dtype=torch.float32, device=dev) for _ in range(L)]
    comm, table = None, None
    if ep:
        uid = [moe.EPComm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = moe.EPComm(uid[0], world, rank, device=local_rank, timeout_s=120.0)
        table = torch.tensor(moe.ep_id_map(E, world, rank), dtype=torch.int32, device=dev)

    def call(li, x):
        rw, wts = layers[li]
        if a2a:
            moe.ep_a2a_moe_ffn(layer, comm, x, wts, router_w=rw, out=outs[li], ids_out=ids[li], w_out=ws[li])
        elif ep:
            moe.ep_moe_ffn(layer, comm, x, wts, table, router_w=rw, out=outs[li], ids_out=ids[li], w_out=ws[li])
        else:
            layer.moe_ffn(x, wts, router_w=rw, out=outs[li], ids_out=ids[li], w_out=ws[li])

    def one_step(x):
        for li in range(L):
            call(li, x)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # eager warm-up (sets kernel attributes), checks the device flag
    one_step(x_dev)
    layer.check()
    log("eager warm-up ok")
    # one CUDA graph for the 48 layer calls
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        one_step(x_dev)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=s):
            one_step(x_dev)
    torch.cuda.synchronize()
    log("graph captured")

    def timed(fn, K, W):
        for _ in range(W):
            fn()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(K):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1))

    with Clocks(local_rank) as clk:
        ms = timed(graph.replay, args.steps, max(args.warmup, 3))
    clocks = clk.summary()
    layer.check()
    log(f"graph timed: {ms / args.steps:.3f} ms/step")
    # all-reduce EP: the ranks process the same tokens jointly; a2a and replicas: T tokens per rank
    units = (1 if ep and not a2a else world) * args.steps * L * T
    value = units / (ms / 1e3)

    # e2e: per layer call, the H2D of its input and the D2H of its output, on two copy streams
    # pipelined with the calls (call l+1's input lands while call l computes; call l's output leaves
    # while call l+1 computes); events keep each buffer's reuse in order across steps
    h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    ev_in, ev_done, ev_out = [ev() for _ in range(L)], [ev() for _ in range(L)], [ev() for _ in range(L)]
    for li in range(L):  # recorded once, so the first step's waits are satisfied
        ev_done[li].record()
        ev_out[li].record()

    def e2e_step():
        main = torch.cuda.current_stream()
        for li in range(L):
            with torch.cuda.stream(h2d_s):
                h2d_s.wait_event(ev_done[li])  # the last step's call li no longer reads x_call[li]
                x_call[li].copy_(x_host[li], non_blocking=True)
                ev_in[li].record(h2d_s)
        for li in range(L):
            main.wait_event(ev_in[li])
            main.wait_event(ev_out[li])  # the last step's output li has left the device
            call(li, x_call[li])
            ev_done[li].record(main)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(ev_done[li])
                out_host[li].copy_(outs[li], non_blocking=True)
                ev_out[li].record(d2h_s)
        main.wait_stream(d2h_s)

    e2e_ms = timed(e2e_step, args.steps, max(args.warmup, 3))
    e2e_value = units / (e2e_ms / 1e3)

    ggml_line = None
    if ggml_down:
        # the same step over the down tensors in ggml's Q6_K layout (no repack): its own handle and
        # graph; the outputs of the two layouts are compared bit for bit
        graph.replay()
        torch.cuda.synchronize()
        want = [o.clone() for o in outs]
        layer_g = tb.MoeLayer(H, I, E, K_USED, gate_type=Q4K, up_type=Q4K, down_type=DOWN_T, max_tokens=T,
                              device=local_rank)
        layers_g = [(rw, moe.ExpertWeights(w.gate, w.up, d)) for (rw, w), d in zip(layers, ggml_down)]

        def step_g():
            for li in range(L):
                rw, wts = layers_g[li]
                layer_g.moe_ffn(x_dev, wts, router_w=rw, out=outs[li], ids_out=ids[li], w_out=ws[li])

        step_g()
        layer_g.check()
        same = all(torch.equal(a.view(torch.int32), b.view(torch.int32)) for a, b in zip(outs, want))
        graph_g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            step_g()
            torch.cuda.synchronize()
            with torch.cuda.graph(graph_g, stream=s):
                step_g()
        torch.cuda.synchronize()
        ms_g = timed(graph_g.replay, args.steps, max(args.warmup, 3))
        layer_g.check()
        ggml_line = {"value": round(units / (ms_g / 1e3), 1), "unit": "tokens/s",
                     "ms_per_step": round(ms_g / args.steps, 4), "outputs_bitwise_equal": same,
                     "note": "the same step with the down tensors in ggml's Q6_K layout (no tmoe_prepack)"}
        log(f"ggml layout: {ms_g / args.steps:.3f} ms/step, outputs equal: {same}")
        del graph_g, layers_g, want
        layer_g.close()
    log(f"e2e timed: {e2e_ms / args.steps:.3f} ms/step")

    # distinct experts per layer (the D of the roofline bytes); a2a: over every rank's tokens
    if a2a:
        all_ids = []
        for li in range(L):
            parts = [torch.empty_like(ids[li]) for _ in range(world)]
            dist.all_gather(parts, ids[li])
            all_ids.append(torch.cat(parts))
    else:
        all_ids = ids
    distinct = [int(torch.unique(all_ids[li]).numel()) for li in range(L)]
    if ep:  # this rank's GEMVs read only the experts it holds
        lo, hi = rank * (E // world), (rank + 1) * (E // world)
        local = [int(((u >= lo) & (u < hi)).sum()) for u in (torch.unique(all_ids[li]) for li in range(L))]
    else:
        local = distinct

    # per-kernel device time of the same workload (events around each kernel)
    # (a 1 ms device sleep first lets the host queue the 4 layer calls, so no event waits on it)
    layer.profile(True)
    for _ in range(2):
        for l0 in range(0, L, 4):
            torch.cuda._sleep(2_000_000)
            for li in range(l0, min(L, l0 + 4)):
                call(li, x_dev)
            prof = layer.profile_collect()
    layer.profile(False)
    log("per-kernel profile done")
    n_calls = 2 * L
    phase_ms = {k: v[0] / v[1] for k, v in prof.items()}
    total_phase = sum(v[0] for v in prof.values())
    shares = {k: round(v[0] / total_phase, 4) for k, v in prof.items()}
    d_mean = sum(distinct) / L
    d_local = sum(local) / L
    # weights of the distinct experts + the Q8_K activation rows read (qs, d, and the split
    # sub-block sums: 2 u32 words x 2 planes per super-block for Q4_K, 4 x 2 for Q6_K) + the f32
    # outputs written
    gate_up_bytes = d_local * GATE_UP_BYTES + T * (H + (H // 256) * (4 + 16)) + T * K_USED * I * 4
    down_bytes = d_local * DOWN_BYTES + T * K_USED * (I + (I // 256) * (4 + 32)) + T * K_USED * H * 4
    peaks = load_peaks()
    dom = max(("gate_up", "down"), key=lambda k: prof.get(k, (0, 1))[0])
    dom_bytes = gate_up_bytes if dom == "gate_up" else down_bytes
    achieved = dom_bytes / (phase_ms[dom] / 1e3) / 1e9
    layer_bytes = d_mean * EXPERT_BYTES + ROUTER_BYTES + T * H * 8
    layer_ms = ms / (args.steps * L)
    roofline = {"bound": "hbm", "kernel": f"gemv_kernel ({dom})", "achieved": round(achieved, 1),
                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "peak_source": peaks["source"],
                "traffic": None if ep or args.shape != "c2" else traffic_from_profiles(dom),
                "algorithmic_bytes_per_launch": int(dom_bytes), "avg_launch_us": round(phase_ms[dom] * 1e3, 2)}
    layer_roof = {"bytes_per_layer_call": int(layer_bytes), "distinct_experts_mean": round(d_mean, 2),
                  "us_per_layer_call": round(layer_ms * 1e3, 2),
                  "achieved_gbs": round(layer_bytes / (layer_ms / 1e3) / 1e9, 1),
                  "frac": round(layer_bytes / (layer_ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
                  "kernel_us": {k: round(v * 1e3, 2) for k, v in phase_ms.items()}, "kernel_share": shares}
    dtype = "int8 x u4/u6 integer MMA (Q8_K activations, Q4_K/Q6_K weights), f32 scales"
    if args.mode == "prefill":
        # tensor bound: the routed GEMM flops (no dequant, no padding); gate/up is the dominant kernel
        gu_flops = 2 * T * K_USED * 2 * H * I
        layer_flops = 2 * T * K_USED * 3 * H * I
        ach = gu_flops / (phase_ms["gate_up"] / 1e3) / 1e12
        roofline = {"bound": "tensor", "kernel": "prefill_gateup_kernel (tcgen05, exact Q8_K x Q4_K in fp16)",
                    "achieved": round(ach, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": round(ach / peaks["bf16_tflops"], 4), "peak_source": peaks["source"] + ", burst bf16",
                    "traffic": None, "algorithmic_flops_per_launch": int(gu_flops),
                    "avg_launch_us": round(phase_ms["gate_up"] * 1e3, 2)}
        lt = layer_flops / (layer_ms / 1e3) / 1e12
        layer_roof = {"flops_per_layer_call": int(layer_flops), "us_per_layer_call": round(layer_ms * 1e3, 2),
                      "achieved_tflops": round(lt, 1), "frac": round(lt / peaks["bf16_tflops"], 4),
                      "distinct_experts_mean": round(d_mean, 2),
                      "kernel_us": {k: round(v * 1e3, 2) for k, v in phase_ms.items()}, "kernel_share": shares}
        dtype = ("gate/up: Q8_K int8 x Q4_K integer values carried exactly in fp16 on tcgen05 (f32 TMEM "
                 "accumulators per super-block); down: fp16 x fp16 tcgen05")
    launches_per_call = sum(v[1] for v in prof.values()) / n_calls
    result = {
        "metric": "moe_layer_tokens_per_s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic",
        "config": workload(args, world), "roofline": roofline, "layer_roofline": layer_roof,
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": L * T * H * 4,
                "d2h_bytes_per_step": L * T * H * 4, "ms_per_step": round(e2e_ms / args.steps, 4),
                "path": f"{L} tmoe_layer C-ABI calls (ctypes, eager) per step, each with its own pinned H2D input "
                        "and D2H output, copies pipelined with the calls on two copy streams"},
        "gpu_launches": int(launches_per_call * L * args.steps), "clocks": clocks,
    }
    if ggml_line:
        result["ggml_layout"] = ggml_line
    if a2a:
        result["config"]["parallelism"] = (f"ep{world} all-to-all (experts split contiguously, {T} tokens per rank "
                                           "dispatched to the experts' ranks and combined back; the messages are "
                                           "written into the peers' buffers over NVLink, NCCL if those cannot be "
                                           "mapped)")
    elif ep:
        result["config"]["parallelism"] = f"ep{world} (experts split contiguously, tokens replicated, NCCL all-reduce)"
        result["scaling"] = "strong"
    if args.sweep and args.mode == "decode" and rank == 0 and not ep:
        result["sweep"] = sweep_tokens(torch, tb, layers, dev)
    del graph
    torch.cuda.synchronize()
    if comm is not None:
        comm.close()
    return result


def c4_line(args, rank, world, local_rank):
    """Config 4 beside the C2 line: the Qwen3-235B-A22B-shaped layer (H 4096, I 1536, 128 experts
    top-8, all Q4_K), the experts split contiguously over the ranks and the tokens dispatched
    all-to-all at N > 1 (the same EP mode as the C2 line):
      decode: T = --tokens per rank, 16 distinct layers (21.7 GB of experts over the ranks, above L2);
      prefill (key "prefill"): T = 4096 per rank, 2 distinct layers, 5 timed steps (the grouped
      tcgen05 GEMMs; tensor roofline)."""
    import copy
    keep = ("metric", "value", "unit", "n_gpus", "steps", "ms_per_step", "scaling", "config", "roofline",
            "layer_roofline", "e2e", "gpu_launches", "clocks")
    set_shape("235b")
    try:
        a = copy.copy(args)
        a.shape, a.layers, a.sweep = "235b", 16, False
        r = run_ours(a, rank, world, local_rank)
        line = {k: r[k] for k in keep if k in r}
        p = copy.copy(args)
        p.shape, p.mode, p.tokens, p.layers, p.sweep, p.steps, p.warmup = "235b", "prefill", 4096, 2, False, 5, 3
        rp = run_ours(p, rank, world, local_rank)
        line["prefill"] = {k: rp[k] for k in keep if k in rp}
    finally:
        set_shape("c2")
    return line


def zipf_bias(torch, E_, seed, s_=1.2):
    """A Zipf(s) bias over a seeded expert permutation: expert perm[r] gets -s * ln(r + 1)."""
    g = np.random.default_rng(seed)
    perm = g.permutation(E_)
    bias = np.empty(E_, np.float32)
    bias[perm] = -s_ * np.log(np.arange(1, E_ + 1, dtype=np.float64))
    return torch.from_numpy(bias), perm


def run_streamed(args, local_rank):
    """Config 5: T tokens with router logits ~N(0,1) plus a Zipf(1.2) bias over a seeded expert
    permutation, `--slots` of the 128 experts in device slots and all 128 in a pinned host store;
    every step is one streamed layer step (device plan, paging of the misses over the host link,
    chunked grouped expert products, combine).  The slot table carries over between steps, as in a
    running model; it starts with the `--slots` most-routed experts of the bias resident."""
    import torch

    import tetraeder_b200 as tb
    from tetraeder_b200 import moe

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    T, NS = args.tokens, args.slots
    (rw, wts), = make_layers(torch, moe, 1, args.seed, dev)
    store = moe.ExpertWeights(*(t.cpu().pin_memory() for t in (wts.gate, wts.up, wts.down)))
    slots = moe.ExpertWeights(*(torch.zeros((NS,) + tuple(t.shape[1:]), dtype=torch.uint8, device=dev)
                                for t in (wts.gate, wts.up, wts.down)))
    del wts, rw
    torch.cuda.synchronize()
    bias, perm = zipf_bias(torch, E, args.seed + 5)
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed + 1)
    replay = None
    if args.routing:  # recorded routing: the logits of each step reproduce its recorded choice
        from tetraeder_b200.trace import LayerStep, TraceReader
        with TraceReader(args.routing) as tr:
            if tr.header.n_expert != E or tr.header.n_used != K_USED:
                raise SystemExit(f"{args.routing}: {tr.header.n_expert} experts, top-{tr.header.n_used}; "
                                 f"the bench layer has {E}, top-{K_USED}")
            steps = [r for r in tr if isinstance(r, LayerStep)]
        layer_id = args.routing_layer if args.routing_layer >= 0 else (steps[0].layer if steps else 0)
        steps = [r for r in steps if r.layer == layer_id]
        if not steps:
            raise SystemExit(f"{args.routing}: no steps of layer {layer_id}")
        T = args.tokens = steps[0].n_tokens
        steps = [r for r in steps if r.n_tokens == T]
        replay = [torch.from_numpy(r.logits(E)).to(dev) for r in steps]
    x = torch.randn((T, H), generator=gen, device=dev)
    lg = replay[0] if replay else torch.randn((T, E), generator=gen, device=dev) + bias.to(dev)
    layer = tb.MoeLayer(H, I, E, K_USED, gate_type=Q4K, up_type=Q4K, down_type=down_type_gpu(),
                        max_tokens=T, device=local_rank)
    cache = tb.SlotCache(layer, slots, store)
    cache.make_resident([int(e) for e in perm[:NS]])
    out = torch.empty((T, H), device=dev)
    x_host, out_host = x.cpu().pin_memory(), torch.empty((T, H)).pin_memory()

    cursor = [0]

    def step():
        logits = lg
        if replay:
            logits = replay[cursor[0] % len(replay)]
            cursor[0] += 1
        layer.moe_ffn_streamed(x, cache, logits=logits, out=out)

    step()
    layer.check()
    _, st0, _ = cache.state()
    W = max(args.warmup, 3)

    def timed(fn):
        for _ in range(W):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    _, sa, _ = cache.state()
    with Clocks(local_rank) as clk:
        ms = timed(step)
    clocks = clk.summary()
    _, sb, _ = cache.state()
    layer.check()
    misses_per_step = (sb[1] - sa[1]) / (W + args.steps)
    hits_per_step = (sb[0] - sa[0]) / (W + args.steps)

    def e2e():
        x.copy_(x_host, non_blocking=True)
        step()
        out_host.copy_(out, non_blocking=True)

    e2e_ms = timed(e2e)
    layer.profile(True)
    step()
    prof = layer.profile_collect()
    layer.profile(False)
    n_chunks, _, loads = cache.last_plan()
    phase_ms = {k: v[0] for k, v in prof.items()}
    if args.record_trace:  # the routing of --steps further steps, as a trace (untimed)
        from tetraeder_b200.trace import TraceHeader, TraceWriter
        th = TraceHeader(1, E, K_USED, model="bench streamed C5", vram_slots=NS, ram_slots=E, ubatch=T,
                         hot_source="profile", expert_bytes=[EXPERT_BYTES])
        ids = torch.empty((T, K_USED), dtype=torch.int32, device=dev)
        with TraceWriter(args.record_trace, th) as tw:
            for i in range(args.steps):
                logits = replay[(cursor[0] + i) % len(replay)] if replay else lg
                layer.moe_ffn_streamed(x, cache, logits=logits, out=out, ids_out=ids)
                tw.layer_step(i, 0, ids.cpu().numpy())
    peaks = load_peaks()
    gu_flops = 2 * T * K_USED * 2 * H * I
    ach = gu_flops / (phase_ms["gate_up"] / 1e3) / 1e12
    page_bytes = sum(len(c) for c in loads) * EXPERT_BYTES
    value = args.steps * T / (ms / 1e3)
    res = {
        "metric": "moe_layer_tokens_per_s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": W, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "gate/up exact Q8_K x Q4_K on tcgen05 (fp16-carried integers), down fp16 tcgen05", "data": "synthetic",
        "config": dict(workload(args, 1), slots=NS,
                       routing=(f"recorded: {os.path.basename(args.routing)}, {len(replay)} steps of one layer, "
                                "replayed in order" if replay else
                                "logits ~N(0,1) + Zipf(1.2) bias over a seeded permutation"),
                       store="all 128 experts in pinned host memory, paged in by a copy kernel"),
        "roofline": {"bound": "tensor", "kernel": "prefill_gateup_kernel (all chunks)", "achieved": round(ach, 1),
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": round(ach / peaks["bf16_tflops"], 4),
                     "peak_source": peaks["source"] + ", burst bf16", "traffic": None,
                     "algorithmic_flops_per_launch": int(gu_flops), "avg_launch_us": round(phase_ms["gate_up"] * 1e3, 2)},
        "slots": {"hits_per_step": hits_per_step, "misses_per_step": misses_per_step,
                  "miss_bytes_per_step": int(misses_per_step * EXPERT_BYTES), "chunks_last_step": n_chunks,
                  "miss_bytes_last_step": int(page_bytes),
                  "paging_on_stream_us": round(phase_ms.get("slot_page", 0) * 1e3, 1),
                  "note": "misses of chunks >= 1 are paged on a side stream, overlapping the previous chunk's "
                          "compute; paging_on_stream_us is what stays on the layer's stream (chunk 0's pages, "
                          "the staging-to-slot copies)",
                  "host_link_gbs_lower_bound": round(page_bytes / (ms / args.steps / 1e3) / 1e9, 1)},
        "kernel_us": {k: round(v * 1e3, 2) for k, v in phase_ms.items()},
        "e2e": {"value": round(args.steps * T / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4,
                "ms_per_step": round(e2e_ms / args.steps, 4), "path": "tmoe_streamed_layer C-ABI call + pinned H2D/D2H"},
        "gpu_launches": int(sum(v[1] for v in prof.values()) * args.steps), "clocks": clocks,
    }
    cache.close()
    layer.close()
    return res


def run_gguf(args, local_rank):
    """Expert loading from a GGUF file (load_weights, qwen3moe.rs:2498-2584): a synthetic C2-shaped
    file of --layers layers (128 experts of random bytes per layer; default 4 layers, 1.57 GB of
    experts) is written to a temporary directory, then each step loads every layer's three stacked
    expert tensors into preallocated HBM through tmoe_gguf_load (pinned double buffering).  Page
    cache warm (the file was just written); `cold_gbs` is the same load after
    posix_fadvise(DONTNEED) on the file (no effect where the directory is RAM-backed).
    `reference_pattern_gbs`: the reference's loop for the same bytes (16 MB reads into a pageable
    buffer, each copied to the device synchronously), in this process."""
    import shutil
    import tempfile

    import torch

    from tests.gguf_fixture import write_moe_gguf
    from tetraeder_b200.gguf import EXPERT_TENSORS, GgufFile

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    L = args.layers if args.layers != 48 else 4
    tmp = tempfile.mkdtemp(prefix="tmoe_gguf_")
    try:
        path = os.path.join(tmp, "c2.gguf")
        log(f"writing a {L}-layer C2-shaped GGUF")
        write_moe_gguf(path, n_layer=L, n_embd=H, n_ff=I, n_expert=E, n_used=K_USED, gate_type=Q4K,
                       down_type=DOWN_T, quantise=False, extra_kv=False, n_vocab=256, seed=args.seed)
        f = GgufFile(path)
        names = [f"blk.{il}.{n}.weight" for il in range(L) for n in EXPERT_TENSORS]
        outs = [torch.empty(f.tensor(n).nbytes, dtype=torch.uint8, device=dev) for n in names]
        step_bytes = sum(o.numel() for o in outs)

        def step():
            for n, o in zip(names, outs):
                f.load(n, o)

        def timed(fn, n_steps, before=None):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ms = 0.0
            for _ in range(n_steps):
                if before:
                    before()
                torch.cuda.synchronize()
                e0.record()
                fn()
                e1.record()
                torch.cuda.synchronize()
                ms += e0.elapsed_time(e1)
            return ms / n_steps

        for _ in range(max(args.warmup, 3)):
            step()
        with Clocks(local_rank) as clk:
            ms = timed(step, args.steps)

        def drop():
            fd = os.open(path, os.O_RDONLY)
            os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
            os.close(fd)

        cold_ms = timed(step, 1, before=drop)
        buf = bytearray(16 << 20)

        def reference_pattern():
            with open(path, "rb") as fh:
                for n, o in zip(names, outs):
                    t = f.tensor(n)
                    fh.seek(t.offset)
                    done = 0
                    while done < t.nbytes:
                        k = min(len(buf), t.nbytes - done)
                        fh.readinto(memoryview(buf)[:k])
                        o[done:done + k].copy_(torch.frombuffer(buf, dtype=torch.uint8, count=k))
                        done += k

        ref_ms = timed(reference_pattern, 1)
        checks = [torch.equal(outs[i][:4096].cpu(), torch.from_numpy(f.read(names[i], 0, 4096)))
                  for i in (0, len(names) - 1)]
        if not all(checks):
            raise RuntimeError("loaded bytes differ from the file")
        f.close()
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    gbs = step_bytes / (ms / 1e3) / 1e9
    return {
        "metric": "gguf_expert_load_gbs", "value": round(gbs, 2), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": f"C2-shaped GGUF, {L} layers x {E} experts (gate/up Q4_K, down Q6_K shapes, random "
                               "bytes), every expert tensor into HBM", "bytes_per_step": step_bytes,
                   "page_cache": "warm", "loader": "tmoe_gguf_load: pread into two pinned 64 MB buffers, "
                                                   "cudaMemcpyAsync per chunk"},
        "cold_gbs": round(step_bytes / (cold_ms / 1e3) / 1e9, 2),
        "reference_pattern_gbs": round(step_bytes / (ref_ms / 1e3) / 1e9, 2),
        "e2e": {"value": round(gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": step_bytes, "d2h_bytes_per_step": 0,
                "path": "GgufFile.load -> tmoe_gguf_load (file -> HBM is the whole path)"},
        "gpu_launches": 0, "clocks": clk.summary(),
    }


def run_model(args, local_rank):
    """Config 3: decode steps of the whole Qwen3-30B-A3B-shaped model (48 layers, 32 query / 4 KV
    heads of 128, 128 experts top-8 of 768, vocabulary 151936), synthetic Q4_K_M-typed weights
    (attention q/k/o and experts gate/up Q4_K, v and expert down Q6_K, token embedding Q4_K, output
    Q6_K), B = --tokens sequences each at --ctx positions of context (the F16 KV caches filled with
    random values up to there: the step's cost does not depend on them).  One step = one CUDA graph
    replay: every sequence gets one token (the previous step's greedy token) at its next position."""
    import torch

    from tetraeder_b200.gguf import Hparams
    from tetraeder_b200.model import Qwen3MoeModel

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    B, ctx = args.tokens, args.ctx
    W = max(args.warmup, 3)
    hp = Hparams(name="Qwen3-30B-A3B-shaped", n_layer=48, n_ctx_train=40960, n_embd=2048, n_head=32, n_head_kv=4,
                 head_dim=128, n_rot=128, n_expert=128, n_expert_used=8, n_ff_exp=768, n_vocab=151936, rms_eps=1e-6,
                 rope_freq_base=1e6, tied_output=False)
    n_ctx = max(ctx + W + args.steps + 1, args.prefill)
    log(f"model: synthetic weights, B={B}, context {ctx}")
    m = Qwen3MoeModel.synthetic(hp, max_batch=B, n_ctx=n_ctx, device=local_rank, seed=args.seed)
    gen = torch.Generator(device=dev)
    gen.manual_seed(args.seed + 3)
    prefill = None
    if args.prefill > 0:  # pp: one prompt of random token ids into sequence 0, then its first token
        S = args.prefill
        prompt = torch.randint(0, hp.n_vocab, (S,), dtype=torch.int32, device=dev, generator=gen)
        m.prefill(prompt, seq=0)
        m.check()
        for _ in range(W):
            m.prefill(prompt, seq=0)
        torch.cuda.synchronize()
        n_pp = max(2, min(args.steps, 5))
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local_rank) as pclk:
            p0.record()
            for _ in range(n_pp):
                m.prefill(prompt, seq=0)
            p1.record()
            torch.cuda.synchronize()
        pms = p0.elapsed_time(p1) / n_pp
        m.check()
        # routed FLOPs of one prompt: projections (q, k, v, o), router, experts, causal attention
        d_, nh_, nkv_, H_ = hp.head_dim, hp.n_head, hp.n_head_kv, hp.n_embd
        per_tok = (2 * H_ * (nh_ * d_ + 2 * nkv_ * d_) + 2 * nh_ * d_ * H_ + 2 * H_ * hp.n_expert
                   + 2 * hp.n_expert_used * 3 * H_ * hp.n_ff_exp)
        attn_fl = 4 * nh_ * d_ * S * (S + 1) / 2
        fl = hp.n_layer * (S * per_tok + attn_fl)
        prefill = {"tokens": S, "ms": round(pms, 3), "tokens_per_s": round(S / (pms / 1e3), 1), "runs": n_pp,
                   "flops": int(fl), "tflops": round(fl / (pms / 1e3) / 1e12, 1), "clocks": pclk.summary(),
                   "path": "Qwen3MoeModel.prefill: one multi-token step per run (eager C-ABI calls), the head on the "
                           "last row"}
        log(f"prefill of {S} tokens: {pms:.2f} ms ({S / (pms / 1e3):.0f} tokens/s)")
    for c in m.kc + m.vc:
        c[:, :ctx].normal_(0.0, 1.0, generator=gen)
    tokens = torch.randint(0, hp.n_vocab, (B,), dtype=torch.int32, device=dev, generator=gen)
    pos = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    m.decode(tokens, pos)
    m.check()
    g = m.graph(tokens, pos)

    def step():
        g.replay()
        tokens.copy_(m.next_tokens[:B])
        pos.add_(1)

    for _ in range(W):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local_rank) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    m.check()
    # bytes a step must read: every weight it touches (all experts at this B: about 126 of 128 per
    # layer for B >= 64, fewer below; counted from the expected distinct experts), the KV caches up
    # to the positions, the output matrix
    exp_d = hp.n_expert * (1 - (1 - hp.n_expert_used / hp.n_expert) ** B)
    w = m.w
    attn = sum(w[f"blk.0.{n}.weight"].data.numel() for n in ("attn_q", "attn_k", "attn_v", "attn_output"))
    expert = sum(w[f"blk.0.{n}.weight"].data.numel() for n in ("ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"))
    expert //= hp.n_expert
    kv = B * (ctx + W + args.steps // 2) * hp.n_head_kv * hp.head_dim * 2 * 2
    per_layer = attn + exp_d * expert + hp.n_expert * hp.n_embd * 4 + kv
    step_bytes = hp.n_layer * per_layer + w["output.weight"].data.numel()
    peaks = load_peaks()
    achieved = step_bytes / (ms / 1e3) / 1e9
    g = None
    m.close()
    return {
        "metric": "decode_tokens_per_s", "value": round(B / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": W, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "Q4_K/Q6_K weights x Q8_K activations (integer MMA); attention in f16 MMAs with "
                                  "f32 accumulation over an F16 KV cache", "data": "synthetic",
        "config": {"workload": "C3 Qwen3-30B-A3B-shaped model, batched decode", "sequences": B, "context": ctx,
                   "n_layer": hp.n_layer, "n_embd": hp.n_embd, "n_head": hp.n_head, "n_head_kv": hp.n_head_kv,
                   "head_dim": hp.head_dim, "n_expert": hp.n_expert, "n_expert_used": hp.n_expert_used,
                   "n_ff_exp": hp.n_ff_exp, "n_vocab": hp.n_vocab, "types": "Q4_K_M-like (attn q/k/o, experts gate/up, "
                   "token_embd Q4_K; attn v, experts down, output Q6_K)", "seed": args.seed,
                   "l2": "inputs larger than L2: every step reads all weights and the KV caches"},
        "roofline": {"bound": "hbm", "kernel": "the whole decode step", "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": peaks["source"], "traffic": None,
                     "algorithmic_bytes_per_step": int(step_bytes),
                     "note": "weights touched (expected distinct experts) + KV caches + output matrix"},
        "gpu_launches": None, "clocks": clk.summary(), "prefill": prefill,
    }


def sweep_tokens(torch, tb, layers, dev):
    """tokens/s and layer roofline fraction at T in {1, 4, 16, 64} (graph of 48 layer calls)."""
    peaks = load_peaks()
    res = {}
    for T in (1, 4, 16, 64):
        log(f"sweep T={T}")
        layer = tb.MoeLayer(H, I, E, K_USED, gate_type=Q4K, up_type=Q4K, down_type=down_type_gpu(), max_tokens=T,
                            device=dev.index)
        x = torch.randn((T, H), device=dev)
        out = torch.empty((T, H), device=dev)
        ids = [torch.empty((T, K_USED), dtype=torch.int32, device=dev) for _ in layers]

        def step():
            for li, (rw, wts) in enumerate(layers):
                layer.moe_ffn(x, wts, router_w=rw, out=out, ids_out=ids[li])
        step()
        torch.cuda.synchronize()  # the handle's workspace is shared: never two streams at once
        s = torch.cuda.Stream(device=dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            step()
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s):
                step()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 20
        e0.record()
        for _ in range(n):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (n * len(layers))
        d = sum(int(torch.unique(i).numel()) for i in ids) / len(layers)
        by = d * EXPERT_BYTES + ROUTER_BYTES + T * H * 8
        res[str(T)] = {"tokens_per_s": round(T / (ms / 1e3), 1), "us_per_layer": round(ms * 1e3, 2),
                       "distinct_experts": round(d, 2), "hbm_frac": round(by / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4)}
        del g
        layer.close()
    return res


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d.get("bf16_tflops"), "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback (profiling recipe)"}


def gemv_source_sha16():
    """The first 16 hex digits of sha256(csrc/gemv.cu): the source the committed ncu figures are of."""
    with open(os.path.join(ROOT, "tetraeder_b200", "csrc", "gemv.cu"), "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()[:16]


def traffic_from_profiles(kernel):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, used only when
    the summary was taken of the gemv.cu that is built now (its `source_sha16` line); else None."""
    path = os.path.join(ROOT, "profiles", "gemv_decode_c2.md")
    if not os.path.exists(path):
        return None
    traffic, sha = None, None
    for line in open(path):
        if line.startswith(f"traffic_bytes_per_launch[{kernel}]:"):
            try:
                traffic = int(float(line.split(":", 1)[1].strip()))
            except ValueError:
                return None
        elif line.startswith("source_sha16[gemv.cu]:"):
            sha = line.split(":", 1)[1].strip()
    return traffic if sha == gemv_source_sha16() else None


# ---------------------------------------------------------------------------------------- CPU
def host_layer(seed, T):
    """One C2 layer on the host, quantised with the oracle's fit (the same algorithm as the device
    quantiser)."""
    import oracle as O
    rng = np.random.default_rng(seed)
    gate = O.quantize(O.TYPE_Q4_K, (rng.standard_normal((E, I, H), dtype=np.float32) * 0.02))
    up = O.quantize(O.TYPE_Q4_K, (rng.standard_normal((E, I, H), dtype=np.float32) * 0.02))
    down = O.quantize(DOWN_T, (rng.standard_normal((E, H, I), dtype=np.float32) * 0.02))
    rw = (rng.standard_normal((E, H), dtype=np.float32) * 0.02)
    x = rng.standard_normal((T, H), dtype=np.float32)
    return gate, up, down, rw, x


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(args):
    import oracle as O
    O.build()
    T = args.tokens
    gate, up, down, rw, x = host_layer(args.seed, T)
    threads = cpu_threads()
    t0 = time.perf_counter()
    O.layer(x, K_USED, gate, up, down, H, I, E, router_w=rw, down_type=DOWN_T, nthreads=threads)
    first = time.perf_counter() - t0
    n = max(1, int(args.cpu_sample_s / max(first, 1e-3)))
    t0 = time.perf_counter()
    for _ in range(n):
        O.layer(x, K_USED, gate, up, down, H, I, E, router_w=rw, down_type=DOWN_T, nthreads=threads)
    dt = time.perf_counter() - t0
    return {"value": round(n * T / dt, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} C2 layer calls of T={T} tokens (router, Q8_K expert dots, combine), one layer's weights"}


def run_reference(args):
    """The reference arm: the CPU oracle (stand-in for ggml's CPU mul_mat_id path) on the host cores,
    one C2 layer call of T tokens per step, wall-clock timed."""
    import oracle as O
    O.build()
    T = args.tokens
    gate, up, down, rw, x = host_layer(args.seed, T)
    threads = cpu_threads()
    for _ in range(args.warmup):
        O.layer(x, K_USED, gate, up, down, H, I, E, router_w=rw, down_type=DOWN_T, nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.layer(x, K_USED, gate, up, down, H, I, E, router_w=rw, down_type=DOWN_T, nthreads=threads)
    dt = time.perf_counter() - t0
    value = args.steps * T / dt
    sample = f"{args.steps} C2 layer calls of T={T} tokens, one layer's weights, {threads} threads"
    return {"metric": "moe_layer_tokens_per_s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 (Q8_K activations x Q4_K/Q6_K weights)", "data": "synthetic",
            "config": workload(args, 1), "impl": "reference",
            "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "ggml's CPU mul_mat_id (llama.cpp b12426) is not in the reference tree and cannot be built "
                    "here; the oracle/ C restatement of its semantics is timed instead"}


_JSON_FD = None  # the original stdout: it carries only the JSON line


def emit(obj):
    os.write(_JSON_FD if _JSON_FD is not None else 1, (json.dumps(obj) + "\n").encode())


def main():
    global _JSON_FD
    args = parse()
    # stdout carries the one JSON line; anything else written to file descriptor 1 (NCCL's version
    # banner, library output) goes to stderr
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    faulthandler.dump_traceback_later(int(os.environ.get("TMOE_BENCH_WATCHDOG_S", "420")), exit=False)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return 0
        emit(run_reference(args))
        return 0
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    if args.mode in ("gguf", "model"):
        if world > 1:
            raise SystemExit(f"--mode {args.mode} runs on one GPU")
        emit(run_gguf(args, local_rank) if args.mode == "gguf" else run_model(args, local_rank))
        return 0
    res = run_streamed(args, local_rank) if args.mode == "streamed" else run_ours(args, rank, world, local_rank)
    if args.mode == "decode" and args.shape == "c2" and not args.no_c4:
        res["c4"] = c4_line(args, rank, world, local_rank)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline(args)
        emit(res)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
