#!/usr/bin/env python3
"""Benchmark: Qwen3-30B-A3B-shaped MoE decode (Q4_0 experts) on B200.

Workload (benchmark configs[1]): decode batch of 64 tokens through a stack of 48 distinct
MoE layers (hidden 2048, 128 experts, top-8, intermediate 768, Q4_0 experts, f32 router whose
rows are scaled so the expert load follows Zipf(1.1)). One step = one batch through all 48
layers (router, experts, combine, residual), weights resident in HBM.

  value   tok/s with activations already on the device (CUDA graph of the 48 layers)
  e2e     tok/s through the host-buffer C entry point cpg_run_moe_layers: each step copies
          the batch from pinned host memory, runs the layers, copies the result back
  roofline  the expert kernel (gate/up and down items in one launch, the dominant kernel),
          algorithmic bytes / its measured duration (CUDA events inside the decode graph),
          against MEASURED_PEAKS.json
  cpu_baseline  the reference engine (oracle/_ref: the reference's own C sources) on the host
          cores, a bounded sample of the same workload
  decode_q8_batch1  configs[0]: one token through 48 stacked layers with Q8_0 experts (plain
          N(0,0.02) router), tok/s and HBM GB/s against the measured copy bandwidth, with the
          reference engine's time on the same workload (bounded sample) beside it
  expert_parallel  configs[4]: 2048 tokens (2048/N per rank) through the 48 stacked layers with
          the 128 experts sharded 128/N per GPU (cpg_moe_ep: NCCL dispatch and combine), uniform
          top-8 routing; tok/s, ms per layer, and the binding roof (HBM, tensor or NVLink)
  full_model  configs[2]: the whole 48-layer model (attention + MoE, vocab 151936, Q4_0 attention
          and experts, Q8_0 embed and lm_head): 512-token prompt, then 128 greedy decode steps;
          decode tok/s and HBM GB/s of the bytes a token must read
  batched_decode  64 sequences of the same model decoded together (cpg_qwen3_batch, continuous
          batching), each with its own prompt and KV cache: tok/s over all sequences, and two of
          them checked against the single-sequence path
  prefill   configs[3]: 4096 Zipf(1.2)-routed tokens through one Q4_0 MoE block per step on the
          tcgen05 grouped GEMM (cpg_moe_apply), tok/s and TFLOP/s, roofline of the gate/up GEMM
          against the measured tensor peak

--impl reference times the reference engine alone (rank 0), on the same metric and config.
Multi-GPU: one process per GPU under torchrun; every rank runs its own replica (decode does not
shard: 22 MB of weights per layer per token), value = all ranks' tokens / max-over-ranks time.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s & MoE-layer HBM GB/s (Qwen3-30B-A3B shape, Q4) at 1/2/4/8 B200"
D, F, E, K = 2048, 768, 128, 8
ENC_Q4, ENC_Q8 = 4, 8
MAT_BYTES = F * D // 32 * 18                     # 884,736
MAT_BYTES_Q8 = F * D // 32 * 34                  # 1,671,168
REGION_BYTES = 3 * MAT_BYTES                     # 2,654,208 per expert (Wg | Wu | Wd)
ROUTER_BYTES = E * D * 4
LN_BYTES = D * 4


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--zipf", type=float, default=1.1)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--cpu-sample-layers", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefill-tokens", type=int, default=4096, help="0 skips the prefill section")
    ap.add_argument("--no-q8", action="store_true", help="skip the Q8 batch-1 section")
    ap.add_argument("--ep-tokens", type=int, default=2048, help="0 skips the expert-parallel section")
    ap.add_argument("--no-full-model", action="store_true", help="skip the whole-model section")
    ap.add_argument("--full-prompt", type=int, default=512)
    ap.add_argument("--full-new", type=int, default=128)
    ap.add_argument("--batch-seqs", type=int, default=64, help="0 skips the several-sequence decode section")
    ap.add_argument("--batch-prompt", type=int, default=32)
    ap.add_argument("--batch-new", type=int, default=32)
    return ap.parse_args()


def physical_cores() -> int:
    """Distinct (physical id, core id) pairs among the CPUs this process may run on: hyper-threads
    share a core (the reference's cp_physical_cores, engine/api/cachepotato.c:59-80, restated; it
    also falls back to the online CPU count)."""
    allowed = os.sched_getaffinity(0) if hasattr(os, "sched_getaffinity") else None
    seen, proc, pkg = set(), None, 0
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                k, _, v = line.partition(":")
                k, v = k.strip(), v.strip()
                if k == "processor":
                    proc = int(v)
                elif k == "physical id":
                    pkg = int(v)
                elif k == "core id" and (allowed is None or proc in allowed):
                    seen.add((pkg, int(v)))
    except (OSError, ValueError):
        seen = set()
    if seen:
        return len(seen)
    return len(allowed) if allowed else (os.cpu_count() or 1)


def headline_config(args) -> dict:
    """The headline workload, identical in both arms' JSON lines."""
    return {"workload": "Qwen3-30B-A3B MoE decode: 64-token batch through 48 stacked MoE layers "
                        "(configs[1], Q4_0 experts, Zipf(1.1)-calibrated f32 router)",
            "tokens_per_step_per_gpu": args.tokens, "layers": args.layers, "d_model": D, "d_exp": F, "experts": E,
            "topk": K, "expert_encoding": "Q4_0",
            "l2": "inputs larger than L2: each step streams ~13 GB of distinct expert weights"}


def profiled_traffic():
    """DRAM bytes of one captured launch of the headline expert kernel and the algorithmic bytes of
    that same launch, from the committed ncu summary (profiles/k_experts_q4_decode_T64.md)."""
    import re
    path = os.path.join(ROOT, "profiles", "k_experts_q4_decode_T64.md")
    try:
        txt = open(path).read()
    except OSError:
        return None, None
    t = re.search(r"traffic_bytes_per_launch:\s*(\d+)", txt)
    a = re.search(r"algorithmic_bytes_same_launch:\s*(\d+)", txt)
    return (int(t.group(1)) if t else None), (int(a.group(1)) if a else None)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """fp16/bf16 dense tensor throughput (TFLOP/s): the measured burst figure (a kernel timed alone)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (bf16 cuBLAS burst)"
    return 1590.0, "fallback"


# ------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, dev: int):
        self.dev, self.p, self.path = dev, None, None

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        self.path = f"/tmp/cpg_clocks_{os.getpid()}.csv"
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.dev}", f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.p = None

    def stop(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        self.p.wait()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons)}


# ------------------------------------------------------------------ device memory views
class DevPtr:
    """A raw device range as a torch tensor (via __cuda_array_interface__)."""

    def __init__(self, ptr: int, nbytes: int, typestr: str = "|u1"):
        item = int(typestr[-1])
        self.__cuda_array_interface__ = {"shape": (nbytes // item,), "typestr": typestr,
                                         "data": (ptr, False), "version": 2, "strides": None}


def moe_launches_per_layer(T: int) -> int:
    """Kernels one cpg_moe_forward enqueues (moe.cu): the router, k_group when the T*K pairs are
    too many for the expert kernel to group itself (> 1024), the expert kernel(s) (one launch
    when the gate/up items (token chunks x d_exp/64) outnumber the SMs, else gate/up and down),
    and the combine."""
    import torch
    chunks = min(T * K, E) + T * K // 16
    experts = 1 if chunks * (F // 64) > torch.cuda.get_device_properties(0).multi_processor_count else 2
    return 1 + (1 if T * K > 1024 else 0) + experts + 1


def view(torch, ptr, nbytes, dtype="f4"):
    ts = {"f4": "<f4", "u1": "|u1"}[dtype]
    return torch.as_tensor(DevPtr(ptr, nbytes, ts), device="cuda")


# ------------------------------------------------------------------ our implementation
def expert_blob(torch, lib, Q, seed, l, out_ptr=None):
    """Layer l's 128 experts as the benchmark's stack holds them: Wg | Wu | Wd per expert,
    N(0, 0.02) from a seeded device generator, quantised to Q4_0 on the device. Written to
    out_ptr, or returned as a new device tensor."""
    out = None
    if out_ptr is None:
        out = torch.empty(E * REGION_BYTES, dtype=torch.uint8, device="cuda")
        out_ptr = out.data_ptr()
    g = torch.Generator(device="cuda")
    w32 = torch.randn(E * 3 * F * D, generator=g.manual_seed(seed * 1000 + 2 * l + 2), device="cuda")
    w32.mul_(0.02)
    Q.check(lib.cpg_quantize(out_ptr, w32.data_ptr(), ENC_Q4, w32.numel(), None))
    del w32
    return out


def full_model_parts(torch, lib, Q, seed, L, V=151936, n_prompt=512):
    """configs[2]'s weights besides the experts (attention Q4_0, fresh f32 routers, Q8_0 embed and
    lm_head, unit norms) and its prompt, from the benchmark's seeds."""
    H, KVH, HD = 32, 4, 128
    QD, KD = H * HD, KVH * HD
    g = torch.Generator(device="cuda")

    def quant(rows, cols, s, enc=ENC_Q4):
        gb = 18 if enc == ENC_Q4 else 34
        out = torch.empty(rows * cols // 32 * gb, dtype=torch.uint8, device="cuda")
        w = torch.randn(rows * cols, generator=g.manual_seed(s), device="cuda").mul_(0.02)
        Q.check(lib.cpg_quantize(out.data_ptr(), w.data_ptr(), enc, w.numel(), None))
        return out
    ones_d, ones_h = torch.ones(D, device="cuda"), torch.ones(HD, device="cuda")
    attn, routers = [], []
    for l in range(L):
        b = seed * 5000 + 10 * l
        attn.append(dict(ln1=ones_d, q_norm=ones_h, k_norm=ones_h, wq=quant(QD, D, b + 1), wk=quant(KD, D, b + 2),
                         wv=quant(KD, D, b + 3), wo=quant(D, QD, b + 4)))
        routers.append(torch.randn((E, D), generator=g.manual_seed(b + 5), device="cuda") * 0.02)
    embed = quant(V, D, seed * 5000 + 901, ENC_Q8)
    head = quant(V, D, seed * 5000 + 902, ENC_Q8)
    prompt = np.random.default_rng(seed + 3).integers(0, V, n_prompt).astype(np.int32)
    return dict(attn=attn, routers=routers, embed=embed, head=head, final_norm=ones_d, ln2=ones_d,
                prompt=prompt, V=V, H=H, KVH=KVH, HD=HD)


def build_stack(torch, L, T, zipf, seed, lib, Q):
    """48 layers in the HBM region store, routers calibrated on the chained activations."""
    from cachepotato_b200.workload import calibrate_router_scales, load_stats
    layer_bytes = LN_BYTES + ROUTER_BYTES + E * REGION_BYTES
    lib.cpg_store_close()
    Q.check(lib.cpg_store_open(L * layer_bytes))
    base = int(lib.cpg_store_base())
    g = torch.Generator(device="cuda")
    layers, stats = [], []
    x = torch.randn((T, D), generator=g.manual_seed(seed), device="cuda", dtype=torch.float32)
    x0 = x.clone()
    for l in range(L):
        off = l * layer_bytes
        r_ln = lib.cpg_store_add_region(off, LN_BYTES, 0)
        r_wg = lib.cpg_store_add_region(off + LN_BYTES, ROUTER_BYTES, 0)
        r_ex = [lib.cpg_store_add_region(off + LN_BYTES + ROUTER_BYTES + e * REGION_BYTES, REGION_BYTES, 1)
                for e in range(E)]
        ln2 = view(torch, lib.cpg_store_region_get(r_ln), LN_BYTES)
        ln2.fill_(1.0)
        wg = view(torch, lib.cpg_store_region_get(r_wg), ROUTER_BYTES).view(E, D)
        wg.copy_(torch.randn((E, D), generator=g.manual_seed(seed * 1000 + 2 * l + 1), device="cuda") * 0.02)
        expert_blob(torch, lib, Q, seed, l, lib.cpg_store_region_get(r_ex[0]))
        # Zipf calibration on this layer's actual input
        xn = x * torch.rsqrt((x * x).mean(-1, keepdim=True) + 1e-6)
        z = (xn @ wg.T).double().cpu().numpy()
        s = calibrate_router_scales(z, K, zipf, seed=seed + l)
        wg.mul_(torch.from_numpy(s).cuda()[:, None])
        ptrs = []
        for e in range(E):
            b = lib.cpg_store_region_get(r_ex[e])
            ptrs += [b, b + MAT_BYTES, b + 2 * MAT_BYTES]
        layer = Q.MoELayer(ln2, wg, ENC_Q4, D, F, E, K, blob=None, expert_ptrs=ptrs)
        layer.ptr_list = ptrs
        out = layer.forward(x)
        stats.append(load_stats(out.topk_idx.cpu().numpy(), E))
        x = out.x_out
        layers.append(layer)
    torch.cuda.synchronize()
    return layers, x0, stats


def run_ours(args, rank, world, torch, dist):
    from cachepotato_b200 import _lib
    from cachepotato_b200 import qwen3 as Q
    lib = _lib.lib()
    T, L = args.tokens, args.layers
    layers, x0, stats = build_stack(torch, L, T, args.zipf, args.seed, lib, Q)
    ctx = Q.DecodeContext(layers[0], max_T=T, device=torch.cuda.current_device())
    arr = ctx.layer_array(layers)
    s = torch.cuda.ExternalStream(ctx.stream_ptr())
    xbuf = view(torch, ctx.x_ptr(), T * D * 4).view(T, D)
    xbytes = T * D * 4

    def device_step():
        with torch.cuda.stream(s):
            xbuf.copy_(x0)                     # this step's batch enters the stack
        ctx.run_device(arr, L, T)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- value: device-resident steps
    for _ in range(args.warmup):
        device_step()
    barrier()
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(args.steps):
        device_step()
    e1.record(s)
    barrier()
    ms = e0.elapsed_time(e1)
    # ---- the same steps with per-phase events inside the graph (roofline of each kernel)
    ctx.profile(True)
    phase = np.zeros(4)
    for _ in range(max(1, args.warmup // 2)):
        device_step()
    for _ in range(args.steps):
        device_step()
        phase += np.array(ctx.phase_ms())
    ctx.profile(False)
    barrier()
    clk = clocks.stop()
    # ---- e2e: host buffers through cpg_run_moe_layers (H2D + layers + D2H each step)
    pinned = [torch.empty((T, D), dtype=torch.float32).pin_memory() for _ in range(args.steps + args.warmup)]
    x0h = x0.cpu()
    for p in pinned:
        p.copy_(x0h)
    for i in range(args.warmup):
        ctx.run_host_ptr(arr, L, pinned[i].data_ptr(), T)
    barrier()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record(s)
    for i in range(args.steps):
        ctx.run_host_ptr(arr, L, pinned[args.warmup + i].data_ptr(), T)
    h1.record(s)
    barrier()
    ms_e2e = h0.elapsed_time(h1)
    # same final activations on both paths (the host path is the same graph)
    dev_out = xbuf.cpu()
    assert torch.equal(dev_out, pinned[-1]), "host-buffer path disagrees with the device path"

    # ---- batch-1 decode on the same stack (the north-star decode target: one token per step)
    x1 = x0[:1].clone()
    xb1 = xbuf[:1]

    def step1():
        with torch.cuda.stream(s):
            xb1.copy_(x1)
        ctx.run_device(arr, L, 1)

    for _ in range(args.warmup):
        step1()
    barrier()
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record(s)
    for _ in range(args.steps):
        step1()
    b1.record(s)
    barrier()
    ms_b1 = b0.elapsed_time(b1)

    # ---- batch-1 decode with Q8_0 experts (its own 48-layer stack)
    q8 = None if args.no_q8 else q8_batch1_bench(args, torch, lib, Q, barrier)
    ms_q8 = q8.pop("_ms") if q8 else 0.0

    # ---- the whole model, prompt + greedy decode
    fm = None if args.no_full_model else full_model_bench(args, layers, torch, lib, Q, barrier)
    ms_fm = fm.pop("_ms") if fm else 0.0
    bt = fm.pop("_batched") if fm else None
    ms_bt = bt.pop("_ms") if bt else 0.0

    # ---- expert parallelism across the ranks (a collective: every rank takes part)
    ep = ep_bench(args, layers, torch, lib, Q, dist, rank, world, barrier) if args.ep_tokens > 0 else None
    ms_ep = ep.pop("_ms") if ep else 0.0

    # ---- prefill: Zipf(1.2)-routed tokens through one MoE block per step
    pf = prefill_bench(args, layers, torch, lib, Q, s, barrier) if args.prefill_tokens > 0 else None
    ms_pf = pf.pop("_ms") if pf else 0.0

    # max over ranks
    ep_par = ep.pop("_parity") if ep else 0.0
    t = torch.tensor([ms, ms_e2e, ms_b1, ms_pf, ms_q8, ms_ep, ms_fm, ep_par], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e, ms_b1, ms_pf, ms_q8, ms_ep, ms_fm, ep_par = (float(v) for v in t.tolist())
    if ep is not None:
        ep["parity"] = {"max_rel_vs_single_gpu_apply": ep_par, "tolerance": 1e-3, "ranks": world,
                        "layers": "0 and last", "reference": "cpg_moe_apply of the whole layer on each rank's GPU"}
        if ep_par > 1e-3:
            raise SystemExit(f"expert-parallel parity failed: max_rel {ep_par:.3e} > 1e-3")
    if rank != 0:
        return None

    U = [st["distinct_experts"] for st in stats]
    step_bytes = sum(LN_BYTES + ROUTER_BYTES + u * REGION_BYTES + 2 * T * D * 4 for u in U)
    # expert launch: the active experts' three matrices, xn read (fp16 hi + lo: 4 B a value), h
    # written and read back (4 B a value each way), y written (f32)
    expert_bytes = sum(u * 3 * MAT_BYTES + T * D * 4 + 2 * T * K * F * 4 + T * K * D * 4 for u in U)
    ms_step = ms / args.steps
    hbm, kind = peaks()
    expert_ms_per_step = (phase[1] + phase[2]) / args.steps
    b1_bytes = L * (LN_BYTES + ROUTER_BYTES + K * REGION_BYTES + 2 * D * 4)
    achieved = expert_bytes / (expert_ms_per_step * 1e-3) / 1e9
    traffic, traffic_alg = profiled_traffic()
    tok_s = world * T * args.steps / (ms * 1e-3)
    e2e_tok_s = world * T * args.steps / (ms_e2e * 1e-3)
    res = {
        "metric": METRIC, "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q4_0 x f32 (f32 activations as fp16 hi + lo halves, exact q on mma.sync, fp32 accumulate)",
        "data": "synthetic",
        "config": headline_config(args), "parallelism": f"replicas x{world}",
        "moe_layer_hbm_gbs": round(step_bytes / (ms_step * 1e-3) / 1e9, 1),
        "routing": {"distinct_experts_per_layer_mean": round(float(np.mean(U)), 1),
                    "distinct_experts_per_layer": [int(u) for u in U],
                    "max_expert_load_mean": round(float(np.mean([st["max_load"] for st in stats])), 1)},
        "phase_ms_per_step": {"router": round(phase[0] / args.steps, 4),
                              "experts": round((phase[1] + phase[2]) / args.steps, 4),
                              "combine": round(phase[3] / args.steps, 4)},
        "roofline": {"bound": "hbm", "kernel": "k_experts<Q4,BOTH> (gate/up then down items, one launch)",
                     "achieved": round(achieved, 1),
                     "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_kind": kind,
                     "algorithmic_bytes_per_launch": int(expert_bytes / L),
                     "traffic": traffic,
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of this "
                                        "kernel (profiles/k_experts_q4_decode_T64.md); its algorithmic bytes: "
                                        f"{traffic_alg}") if traffic else None},
        "e2e": {"value": round(e2e_tok_s, 1), "unit": "tok/s", "h2d_bytes_per_step": xbytes,
                "d2h_bytes_per_step": xbytes},
        "decode_batch1": {"value": round(world * args.steps / (ms_b1 * 1e-3), 1), "unit": "tok/s",
                          "ms_per_step": round(ms_b1 / args.steps, 4),
                          "hbm_gbs": round(b1_bytes / (ms_b1 / args.steps * 1e-3) / 1e9, 1),
                          "frac": round(b1_bytes / (ms_b1 / args.steps * 1e-3) / 1e9 / hbm, 4),
                          "bytes_per_step": b1_bytes},
        "gpu_launches": moe_launches_per_layer(T) * L * args.steps,
        "clocks": clk,
    }
    if q8:
        per = ms_q8 / args.steps
        q8["value"] = round(world * args.steps / (ms_q8 * 1e-3), 1)
        q8["ms_per_step"] = round(per, 4)
        q8["hbm_gbs"] = round(q8["bytes_per_step"] / (per * 1e-3) / 1e9, 1)
        q8["frac"] = round(q8["hbm_gbs"] / hbm, 4)
        res["decode_q8_batch1"] = q8
    if fm:
        per_tok = ms_fm / args.full_new
        fm["value"] = round(world * args.full_new / (ms_fm * 1e-3), 1)
        fm["ms_per_token"] = round(per_tok, 4)
        fm["hbm_gbs"] = round(fm["bytes_per_token"] / (per_tok * 1e-3) / 1e9, 1)
        fm["frac"] = round(fm["hbm_gbs"] / hbm, 4)
        res["full_model"] = fm
    if bt:
        bt["value"] = round(world * bt["sequences"] * bt["steps"] / (ms_bt * 1e-3), 1)
        bt["vs_one_sequence"] = round(bt["value"] / fm["value"], 2)
        res["batched_decode"] = bt
    if ep:
        per_layer = ms_ep / args.steps / L
        ep["value"] = round(args.ep_tokens * args.steps / (ms_ep * 1e-3), 1)
        ep["ms_per_step"] = round(ms_ep / args.steps, 4)
        ep["ms_per_layer"] = round(per_layer, 5)
        roof = ep.pop("_roof_ms")
        bind = max(roof, key=roof.get)
        ep["roofline"] = {"bound": bind, "roof_ms_per_layer": {k: round(v, 5) for k, v in roof.items()},
                          "frac": round(roof[bind] / per_layer, 4),
                          "peaks": {"hbm_gbs": hbm, "tensor_tflops": tensor_peak()[0], "nvlink_gbs": 770.0}}
        res["expert_parallel"] = ep
    if pf:
        pf["value"] = round(world * args.prefill_tokens * args.steps / (ms_pf * 1e-3), 1)
        pf["ms_per_step"] = round(ms_pf / args.steps, 4)
        pf["tflops"] = round(pf["flops_per_step"] / (ms_pf / args.steps * 1e-3) / 1e12, 1)
        res["prefill"] = pf
    return res


def q8_batch1_bench(args, torch, lib, Q, barrier):
    """one token per step through args.layers distinct layers whose 128 experts are
    Q8_0 (weights ~N(0,0.02) quantised on the device by cpg_quantize), f32 router ~N(0,0.02),
    ln2 = 1. The layer stack (30.8 GB for 48 layers) is larger than L2, so every step streams the
    8 selected experts of each layer from HBM."""
    L = args.layers
    g = torch.Generator(device="cuda")
    layers = []
    for l in range(L):
        blob = torch.empty(E * 3 * MAT_BYTES_Q8, dtype=torch.uint8, device="cuda")
        w32 = torch.randn(E * 3 * F * D, generator=g.manual_seed(args.seed * 3000 + l), device="cuda")
        w32.mul_(0.02)
        Q.check(lib.cpg_quantize(blob.data_ptr(), w32.data_ptr(), ENC_Q8, w32.numel(), None))
        del w32
        ln2 = torch.ones(D, device="cuda")
        wg = torch.randn((E, D), generator=g.manual_seed(args.seed * 3000 + 500 + l), device="cuda") * 0.02
        layers.append(Q.MoELayer(ln2, wg, ENC_Q8, D, F, E, K, blob=blob))
    ctx = Q.DecodeContext(layers[0], max_T=1, device=torch.cuda.current_device())
    arr = ctx.layer_array(layers)
    s = torch.cuda.ExternalStream(ctx.stream_ptr())
    xbuf = view(torch, ctx.x_ptr(), D * 4).view(1, D)
    x1 = torch.randn((1, D), generator=g.manual_seed(args.seed + 91), device="cuda")

    def step():
        with torch.cuda.stream(s):
            xbuf.copy_(x1)
        ctx.run_device(arr, L, 1)

    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(args.steps):
        step()
    e1.record(s)
    barrier()
    ms = e0.elapsed_time(e1)
    del ctx
    return {"_ms": ms, "unit": "tok/s",
            "bytes_per_step": L * (LN_BYTES + ROUTER_BYTES + K * 3 * MAT_BYTES_Q8 + 2 * D * 4),
            "config": {"workload": f"configs[0]: decode batch 1 through {L} stacked Q8_0 MoE layers "
                                   "(plain N(0,0.02) f32 router)", "expert_encoding": "Q8_0"}}


def full_model_bench(args, layers, torch, lib, Q, barrier):
    """the whole Qwen3-30B-A3B-shaped model (48 layers, hidden 2048, 32 query / 4 KV
    heads of 128, QK-RMSNorm, RoPE theta 1e6, 128 experts top-8 of width 768, vocab 151936) with
    random weights N(0,0.02): attention and experts Q4_0, embed and lm_head Q8_0, norms 1, f32
    routers (not Zipf-scaled: the experts are the region store's, the routers are fresh). A prompt
    of args.full_prompt uniform ids in one pass, then args.full_new greedy steps through
    cpg_qwen3_generate (each step embeds the previous argmax on the device and reads its id back)."""
    L = len(layers)
    P = full_model_parts(torch, lib, Q, args.seed, L, n_prompt=args.full_prompt)
    V, H, KVH, HD, prompt = P["V"], P["H"], P["KVH"], P["HD"], P["prompt"]
    QD, KD = H * HD, KVH * HD
    moe = [Q.MoELayer(P["ln2"], P["routers"][l], ENC_Q4, D, F, E, K, blob=None, expert_ptrs=ly.ptr_list)
           for l, ly in enumerate(layers)]
    max_ctx = args.full_prompt + args.full_new + 1
    m = Q.Qwen3Model(d_model=D, n_heads=H, n_kv=KVH, head_dim=HD, vocab=V, max_ctx=max_ctx, attn=P["attn"],
                     moe=moe, attn_enc=ENC_Q4, embed=P["embed"], embed_enc=ENC_Q8, lm_head=P["head"],
                     head_enc=ENC_Q8, final_norm=P["final_norm"])
    s = torch.cuda.ExternalStream(m.stream_ptr())
    m.generate(prompt[:8], 4)                           # warm-up (small)
    barrier()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record(s)
    nxt = m.prefill(prompt)
    e1.record(s)
    ids = [nxt]
    for _ in range(args.full_new):
        nxt = m.step(nxt)
        ids.append(nxt)
    e2.record(s)
    barrier()
    ms_prefill, ms_decode = e0.elapsed_time(e1), e1.elapsed_time(e2)
    bt = batched_decode_bench(args, m, V, torch, Q, barrier) if args.batch_seqs > 0 else None
    m.close()
    avg_pos = args.full_prompt + args.full_new / 2
    per_layer = (2 * QD * D + 2 * KD * D) // 32 * 18 + ROUTER_BYTES + K * REGION_BYTES + 2 * D * 4 + 2 * HD * 4
    bytes_tok = L * (per_layer + 2 * KD * 4 * avg_pos) + V * D // 32 * 34 + D // 32 * 34 + D * 4
    return {"_ms": ms_decode, "_batched": bt, "unit": "tok/s", "bytes_per_token": int(bytes_tok),
            "prefill_ms": round(ms_prefill, 3), "prefill_tok_s": round(args.full_prompt / (ms_prefill * 1e-3), 1),
            "tokens_head": [int(v) for v in ids[:8]],
            "config": {"workload": f"configs[2]: whole model, {L} layers, vocab {V}, prompt {args.full_prompt} uniform "
                                   f"ids, {args.full_new} greedy steps (host reads each argmax)",
                       "attention": "32 query / 4 KV heads x 128, QK-RMSNorm, RoPE theta 1e6, f32 KV cache",
                       "bytes_per_token": "48 x (attention 10.6 MB + router 1 MiB + 8 experts 21.2 MB + KV reads "
                                          "at the mean position) + lm_head 330.6 MB + embed row"}}


def batched_decode_bench(args, m, V, torch, Q, barrier):
    """Several sequences through the same whole model at once (cpg_qwen3_batch; the reference
    decodes one sequence at a time). args.batch_seqs sequences, each with its own prompt of
    args.batch_prompt uniform ids and its own KV cache, are prefilled one by one; then
    args.batch_new steps advance all of them together (one new token per sequence per step, each
    argmax fed back on the device, the ids read back at the end). The first and last sequences
    are checked against the single-sequence path (cpg_qwen3_generate on the same prompt)."""
    S, n_p, n_new = args.batch_seqs, args.batch_prompt, args.batch_new
    rng = np.random.default_rng(args.seed + 5)
    prompts = [rng.integers(0, V, n_p).astype(np.int32) for _ in range(S)]
    b = Q.Qwen3Batch(m, S, n_p + n_new + 2)
    s = torch.cuda.ExternalStream(m.stream_ptr())
    first = [b.prefill(j, p) for j, p in enumerate(prompts)]
    slots = np.arange(S, dtype=np.int32)
    warm = b.generate(slots, first, 1)[0]               # warm-up step (captures the step of S sequences)
    barrier()
    e0, e1 = (torch.cuda.Event(enable_timing=True) for _ in range(2))
    e0.record(s)
    out = b.generate(slots, warm, n_new)
    e1.record(s)
    barrier()
    ms = e0.elapsed_time(e1)
    b.close()
    match = []
    for j in (0, S - 1):
        want = m.generate(prompts[j], n_new + 1)
        match.append([first[j], int(warm[j])] + out[:, j].tolist() == want.tolist())
    return {"_ms": ms, "unit": "tok/s", "sequences": S, "steps": n_new,
            "ms_per_step": round(ms / n_new, 4), "ids_match_single_sequence": match,
            "config": {"workload": f"{S} sequences of the configs[2] model, each its own {n_p}-id uniform prompt "
                                   f"and KV cache, then {n_new} steps of all {S} together (greedy, ids fed back "
                                   "on the device)"}}


def ep_bench(args, layers, torch, lib, Q, dist, rank, world, barrier):
    """args.ep_tokens tokens split evenly over the ranks go through the stacked layers;
    rank r holds experts [r*128/N, (r+1)*128/N) of every layer (pointers into its region store)
    and runs x += MoE(x) per layer with cpg_moe_ep (NCCL dispatch of fp16 rows to the expert
    owners, tcgen05 experts there, f32 partial rows back). Routing: 8 distinct experts per token
    drawn uniformly (seeded per layer), weights uniform in [0.1, 1.1) renormalised."""
    G = world
    assert E % G == 0 and args.ep_tokens % G == 0
    T, E_l, L = args.ep_tokens // G, E // G, len(layers)
    ln2 = torch.ones(D, device="cuda")
    wg = torch.zeros((E_l, D), device="cuda")
    local = [Q.MoELayer(ln2, wg, ENC_Q4, D, F, E_l, K, blob=None,
                        expert_ptrs=l.ptr_list[rank * E_l * 3:(rank + 1) * E_l * 3]) for l in layers]
    idx_l, wt_l, remote_rows = [], [], 0
    for l in range(L):
        rng = np.random.default_rng(args.seed * 7 + l)
        idx = np.argsort(rng.random((args.ep_tokens, E)), axis=1)[:, :K].astype(np.int32)
        wt = rng.random((args.ep_tokens, K)).astype(np.float32) + 0.1
        wt /= wt.sum(1, keepdims=True)
        mine = slice(rank * T, (rank + 1) * T)
        idx_l.append(torch.from_numpy(idx[mine].copy()).cuda())
        wt_l.append(torch.from_numpy(wt[mine].copy()).cuda())
        owners = idx[mine] // E_l                       # distinct remote owners per token
        remote_rows += sum(len(set(o.tolist()) - {rank}) for o in owners)
    uid = [Q.ExpertParallel.unique_id() if rank == 0 else None]
    if dist is not None:
        dist.broadcast_object_list(uid, src=0)
    ep = Q.ExpertParallel(G, rank, uid[0])
    ws = ep.workspace(local[0], T)
    g = torch.Generator(device="cuda").manual_seed(args.seed * 11 + rank)
    x0 = torch.randn((T, D), generator=g, device="cuda")
    x = x0.clone()

    def step():
        x.copy_(x0)
        for l in range(L):
            ep.forward(local[l], x, idx_l[l], wt_l[l], mlp=x, ws=ws, check_status=False)

    for _ in range(max(3, args.warmup)):
        step()
    ep.wait()
    Q.check(lib.cpg_moe_ep_check(ws.data_ptr(), None))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    barrier()
    ms = e0.elapsed_time(e1)
    ep.wait()
    Q.check(lib.cpg_moe_ep_check(ws.data_ptr(), None))
    # per-phase device times (events inside cpg_moe_ep; every rank takes the same calls)
    n_ph = min(L, 8)
    phase = np.zeros(5)
    x.copy_(x0)
    for l in range(n_ph):
        ph = [0.0] * 5
        ep.forward(local[l], x, idx_l[l], wt_l[l], mlp=x, ws=ws, check_status=False, phase_ms=ph)
        phase += np.array(ph)
    phase /= n_ph
    # parity: this rank's tokens through layers 0 and L-1 by expert parallelism against the whole
    # layer applied on this GPU alone (cpg_moe_apply, all 128 experts), same rows and routing
    parity = 0.0
    for l in sorted({0, L - 1}):
        got = ep.forward(local[l], x0, idx_l[l], wt_l[l], ws=ws)
        want = Q.moe_apply(layers[l], x0, idx_l[l], wt_l[l])
        parity = max(parity, float((got - want).abs().max() / want.abs().max()))
    ep.close()
    pairs = args.ep_tokens * K / G                      # per GPU, uniform routing
    link_bytes = remote_rows / L * D * (2 + 4)          # per layer: fp16 rows out, f32 rows back
    roof = {"hbm": E_l * REGION_BYTES / (peaks()[0] * 1e9) * 1e3,
            "tensor": pairs * 3 * 2 * F * D / (tensor_peak()[0] * 1e12) * 1e3,
            "nvlink": link_bytes / 770e9 * 1e3}
    return {"_ms": ms, "_roof_ms": roof, "_parity": parity, "unit": "tok/s",
            "phase_ms_per_layer_rank": {k: round(float(v), 5) for k, v in
                                        zip(("plan_pack", "dispatch", "owner_experts", "return", "combine"), phase)},
            "config": {"workload": f"configs[4]: {args.ep_tokens} tokens x {L} stacked Q4_0 MoE layers, experts "
                                   f"sharded {E_l} per GPU over {G} GPU(s), uniform top-8 routing",
                       "tokens_per_rank": T, "experts_per_rank": E_l, "scaling": "strong",
                       "remote_rows_per_layer_rank0": round(remote_rows / L, 1),
                       "transfer": "fixed capacity: T fp16 rows + metadata out and T f32 rows back per peer"},
            "gpu_launches_per_layer": 9}


def prefill_bench(args, layers, torch, lib, Q, s, barrier):
    """T tokens (default 4096) whose expert assignment is drawn Zipf-Mandelbrot(1.2)
    go through one Q4_0 MoE block per step (token sort, tcgen05 gate/up and down grouped GEMMs,
    combine: cpg_moe_apply). Steps rotate over the 48 stacked layers, so each step reads a
    different layer's 340 MB of experts (larger than L2)."""
    from cachepotato_b200.workload import zipf_assignment
    T, n = args.prefill_tokens, len(layers)
    idx, wt = zipf_assignment(T, E, K, 1.2, 20.0, args.seed + 77)
    counts = np.bincount(idx.ravel(), minlength=E)
    g = torch.Generator(device="cuda").manual_seed(args.seed + 78)
    x = torch.randn((T, D), generator=g, device="cuda")
    xn = x * torch.rsqrt((x * x).mean(-1, keepdim=True) + 1e-6)
    idx_d, wt_d = torch.from_numpy(idx).cuda(), torch.from_numpy(wt).cuda()
    ws = torch.empty(int(lib.cpg_moe_apply_workspace_bytes(layers[0].handle, T)), dtype=torch.uint8, device="cuda")
    mlp = torch.zeros((T, D), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def step(i, phase=None):
        Q.moe_apply(layers[i % n], xn, idx_d, wt_d, ws=ws, mlp=mlp, stream=s, check_status=False,
                    phase_ms=phase)

    for i in range(max(3, args.warmup)):
        step(i)
    Q.check(lib.cpg_moe_apply_check(ws.data_ptr(), s.cuda_stream))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(args.steps):
        step(i)
    e1.record(s)
    barrier()
    ms = e0.elapsed_time(e1)
    Q.check(lib.cpg_moe_apply_check(ws.data_ptr(), s.cuda_stream))
    # per-phase times (events inside the call; synchronising, so a separate pass)
    phase, ph = np.zeros(4), [0.0] * 4
    for i in range(args.steps):
        step(i, ph)
        phase += np.array(ph)
    phase /= args.steps
    P = T * K
    fl_gu, fl_dn = 2.0 * P * D * 2 * F, 2.0 * P * F * D
    peak, kind = tensor_peak()
    ach = fl_gu / (phase[1] * 1e-3) / 1e12
    return {
        "_ms": ms, "unit": "tok/s", "flops_per_step": fl_gu + fl_dn,
        "config": {"workload": "configs[3]: 4096-token prefill through one Q4_0 MoE block, expert assignment "
                               "Zipf-Mandelbrot(s=1.2, q=20) Gumbel-top-8, steps rotate over 48 layers",
                   "tokens": T, "expert_tokens_min": int(counts.min()), "expert_tokens_max": int(counts.max()),
                   "dtype": "q4_0 decoded to f16 in SMEM x f16 activations -> f32 (tcgen05 kind::f16)"},
        "phase_ms": {"sort": round(phase[0], 4), "gate_up": round(phase[1], 4), "down": round(phase[2], 4),
                     "combine": round(phase[3], 4)},
        "roofline": {"bound": "tensor", "kernel": "k_gemm_tc<0> (gate/up)", "achieved": round(ach, 1),
                     "peak": peak, "unit": "TFLOP/s", "frac": round(ach / peak, 4), "peak_kind": kind,
                     "algorithmic_flops_per_launch": fl_gu,
                     "down_tflops": round(fl_dn / (phase[2] * 1e-3) / 1e12, 1)},
        "gpu_launches_per_step": 5,
    }


# ------------------------------------------------------------------ reference (CPU)
_REF = {}


def reference_engine():
    """The reference engine (oracle/_ref), its thread pool on the host's physical cores (the pool
    is process-global: the first initialisation fixes it, engine/kernels/parallel.c:126-132)."""
    if "ref" not in _REF:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        _REF["O"] = O
        _REF["ref"] = O.Reference(threads=physical_cores())
        _REF["orc"] = O.Oracle()
    return _REF["O"], _REF["ref"], _REF["orc"]


def reference_sample(n_layers: int, T: int, zipf, seed: int, steps: int, warmup: int, enc: int = ENC_Q4):
    """The reference engine on n_layers distinct layers, T tokens per pass (one sampled step =
    those layers in sequence, x += mlp after each, as run_layers does); routers Zipf-calibrated on
    the chained activations unless zipf is None. Returns (per-step seconds of the timed steps,
    threads)."""
    O, ref, orc = reference_engine()
    from cachepotato_b200.workload import calibrate_router_scales, rmsnorm_rows
    x = orc.normal(T * D, seed, 1.0).reshape(T, D)
    layers = []
    xi = x
    for l in range(n_layers):          # routers calibrated on the chained activations
        L0 = O.SynthLayer(D, F, E, K, enc, seed=seed + 17 * l, oracle=orc)
        if zipf is not None:
            s = calibrate_router_scales(rmsnorm_rows(xi) @ L0.wgate.T, K, zipf, seed=seed + l)
            L0.wgate *= s[:, None]
        layers.append(L0)
        xi = xi + ref.qwen3_moe(L0, xi)["mlp"]
    times = []
    for i in range(warmup + steps):
        xi = x.copy()
        t0 = time.perf_counter()
        for L0 in layers:
            r = ref.qwen3_moe(L0, xi)
            xi = xi + r["mlp"]
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    return times, ref.threads


def reference_line(args, times, threads, n_layers):
    """tok/s of the 48-layer step from the sampled steps (per-layer time x 48)."""
    per_layer = float(np.mean(times)) / n_layers
    return args.tokens / (per_layer * args.layers), per_layer


def run_reference(args, rank):
    if rank != 0:
        return None
    T, L, n = args.tokens, args.layers, args.cpu_sample_layers
    times, threads = reference_sample(n, T, args.zipf, args.seed, args.steps, args.warmup)
    tok_s, per_layer = reference_line(args, times, threads, n)
    sample = (f"{n} of {L} distinct layers per timed step (T={T}); ms_per_step is that sampled step, value "
              f"scales its per-layer time to the {L}-layer step; {threads} threads = physical cores")
    return {
        "metric": METRIC, "impl": "reference", "value": round(tok_s, 3), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(float(np.mean(times)) * 1e3, 2),
        "layers_timed": n, "ms_per_layer": round(per_layer * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q4_0 x f32 (AVX2 FMA)",
        "data": "synthetic", "config": headline_config(args),
        "parallelism": f"reference engine, 1 process, {threads} threads",
        "cpu_baseline": {"value": round(tok_s, 3), "unit": "tok/s", "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(tok_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    import torch
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    res = run_ours(args, rank, world, torch, dist)
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        n = args.cpu_sample_layers
        times, threads = reference_sample(n, args.tokens, args.zipf, args.seed, 5, 1)
        tok_s, per_layer = reference_line(args, times, threads, n)
        res["cpu_baseline"] = {"value": round(tok_s, 3), "unit": "tok/s", "cores": threads, "kind": "reference",
                               "sample": f"reference engine, {n} of {args.layers} distinct layers x 5 timed reps, "
                                         f"T={args.tokens}, per-layer time x {args.layers}; threads = physical cores",
                               "ms_per_layer": round(per_layer * 1e3, 3)}
        if "decode_q8_batch1" in res:
            t8, th8 = reference_sample(n, 1, None, args.seed + 5, 5, 1, ENC_Q8)
            pl8 = float(np.mean(t8)) / n
            res["decode_q8_batch1"]["cpu_baseline"] = {
                "value": round(1.0 / (pl8 * args.layers), 3), "unit": "tok/s", "cores": th8, "kind": "reference",
                "sample": f"reference engine, Q8_0 experts, {n} layers x 5 timed reps, T=1, "
                          f"per-layer time x {args.layers}"}
    if res is not None:
        print(json.dumps(res), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
