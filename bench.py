#!/usr/bin/env python
"""Benchmark of the MoE hot path on B200: batch-1 decode through a Qwen3-30B-A3B-shape MoE stack.

One step = one decode token through 48 MoE layers (H 2048, 128 experts, top-8 + renorm, expert
intermediate 768, gate/up Q4_K, down Q6_K on even layers and Q4_K on odd layers = the Q4_K_M
rule), every expert resident in HBM (17.6 GB of expert bytes), each layer = router -> experts ->
weighted combine into the residual, through one call of the public C ABI (hoard_moe_layers).
Weights are seeded N(0, 0.02) quantized on the device by hoard_b200.quant; the token activations
are seeded N(0,1), RMS-normalised, one distinct row per step. A step touches 1.2 GB of distinct
weights, far above the 126 MB L2, so no flush is needed between steps.

`python bench.py --impl reference` times the CPU restatement of hoard's ggml CPU path (the oracle,
C++ with OpenMP over all host threads) on a bounded sample of the same workload: the reference
itself (C++/Win32 over ggml + Vulkan, neither vendored nor buildable here) cannot run.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, E, K_USED, I, N_LAYER = 2048, 128, 8, 768, 48
Q4_K, Q6_K = 12, 14
SEED = 20241201
METRIC = "decode tok/s b=1 (Qwen3-30B-A3B shape, 48 MoE layers, experts HBM-resident)"
WORKLOAD = "qwen3-30b-a3b MoE stack: 48 layers x (router + top-8 of 128 experts + combine), T=1 decode"


def down_type(layer: int) -> int:
    return Q6_K if layer % 2 == 0 else Q4_K


def expert_bytes(layer: int) -> int:
    g = I * (H // 256) * 144
    d = H * (I // 256) * (210 if down_type(layer) == Q6_K else 144)
    return 2 * g + d


def algorithmic_bytes_per_token(sel_layers) -> int:
    """Bytes the hot path must move for one token: distinct experts' bytes per layer + f32 router
    weight [E][H] + ffn_norm [H] + residual in/out (f32)."""
    total = 0
    for layer, sel in enumerate(sel_layers):
        total += len(set(int(e) for e in sel.reshape(-1))) * expert_bytes(layer)
        total += E * H * 4 + H * 4 + 2 * H * 4
    return total


def c2_layer_bytes(sel, T: int) -> int:
    """Bytes one C2 layer call must move: the distinct selected experts' bytes (layer 0: Q6_K down),
    the f32 router weight [E][H] and ffn_norm [H], and the T residual rows in and out (f32)."""
    return (len(set(int(e) for e in sel.reshape(-1))) * expert_bytes(0) + E * H * 4 + H * 4 + 2 * T * H * 4)


# --------------------------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0:   # nvidia-smi's first sample
                time.sleep(0.01)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = max(mx, float(p[2]))
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------------------------
def build_model(ctx, device, n_layer: int):
    """Seeded router + expert weights for every layer, generated and quantized on the device."""
    import torch
    from hoard_b200 import quant
    g = torch.Generator(device=device)
    for layer in range(n_layer):
        g.manual_seed(SEED + 7919 * layer)
        w_router = torch.randn(E, H, generator=g, device=device) * 0.02
        w_norm = 1.0 + 0.1 * torch.randn(H, generator=g, device=device)
        ctx.set_router(layer, w_router, w_norm)
        dt = down_type(layer)
        for e0 in range(0, E, 16):
            n = min(16, E - e0)
            gate = quant.quantize_q4k(torch.randn(n, I, H, generator=g, device=device) * 0.02)
            up = quant.quantize_q4k(torch.randn(n, I, H, generator=g, device=device) * 0.02)
            down = quant.quantize(torch.randn(n, H, I, generator=g, device=device) * 0.02, dt)
            for i in range(n):
                ctx.upload_expert(layer, e0 + i, gate[i].contiguous(), up[i].contiguous(), down[i].contiguous())
        torch.cuda.synchronize(device)


def token_rows(n: int, device):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 1)
    x = torch.randn(n, 1, H, generator=g, device=device)
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-6)


CPU_POOL = 64   # distinct experts per sampled layer on the CPU: 64 x ~3 MB, well above any LLC


def cpu_sample(max_seconds: float, nthreads: int):
    """Times the oracle (ggml CPU semantics, C++ + OpenMP) on a bounded sample of the workload:
    single-token MoE layers (router over all 128 experts, then the 8 selected experts + combine),
    alternating an even (Q6_K down) and an odd (Q4_K down) layer, until ~max_seconds.
    Expert e is served by pool expert e mod 64 (64 distinct seeded experts per layer, ~190 MB, so
    the sample streams from DRAM like the full model would). Returns (tok/s, sample text)."""
    import torch
    from hoard_b200 import quant
    from oracle import oracle as orc
    orc.lib()
    g = torch.Generator().manual_seed(SEED)
    layers = []
    for layer in range(2):
        dt = down_type(layer)
        layers.append(dict(
            w_router=(torch.randn(E, H, generator=g) * 0.02).numpy(),
            w_norm=(1.0 + 0.1 * torch.randn(H, generator=g)).numpy(),
            gate=quant.quantize_q4k(torch.randn(CPU_POOL, I, H, generator=g) * 0.02).numpy(),
            up=quant.quantize_q4k(torch.randn(CPU_POOL, I, H, generator=g) * 0.02).numpy(),
            down=quant.quantize(torch.randn(CPU_POOL, H, I, generator=g) * 0.02, dt).numpy(), dt=dt))
    x = token_rows(64, "cpu").numpy()
    t0 = time.perf_counter()
    n = 0
    while True:
        L = layers[n % 2]
        xt = x[n % 64]
        fx, _, sel, w = orc.route(xt, L["w_norm"], L["w_router"], K_USED, True, 1e-6, nthreads)
        orc.experts(H, CPU_POOL, K_USED, I, (Q4_K, Q4_K, L["dt"]), L["gate"], L["up"], L["down"], fx, xt,
                    sel % CPU_POOL, w, orc.MODE_GGML, nthreads)
        n += 1
        el = time.perf_counter() - t0
        if el >= max_seconds and n >= 2:
            break
    per_layer = el / n
    tok_s = 1.0 / (per_layer * N_LAYER)
    return tok_s, (f"{n} single-token MoE layers (router over 128 experts + 8 experts + combine; even/odd "
                   f"down types alternating; 64 distinct experts per layer) in {el:.1f}s; "
                   f"tok/s = 1/(48 x mean layer time)")


# the persistent kernel's phase stamps, in the order a layer passes them
TRACE_STAMPS = [(19, "router_sums_read"), (1, "topk_selected"), (2, "gate_up_copies_issued"), (3, "weights"),
                (5, "down_copies_issued"), (6, "first_gate_up_chunk"), (7, "h_published"),
                (8, "first_expert_h_ready"), (9, "first_expert_h_quantised"), (10, "first_expert_down_landed"),
                (11, "down_done"), (14, "combined"), (15, "router_weights_landed"), (12, "router_partials"),
                (16, "barrier_arrive"), (17, "barrier_passed"),
                (13, "layer_end")]


def trace_breakdown(ctx, x_row, device):
    """One extra (untimed) decode step with the persistent kernel's phase stamps on; returns, per stamp,
    the time from the layer's start (us): the median and the max over CTAs, averaged over layers."""
    import torch
    ctas, nph = ctx.trace_layout()
    buf = torch.zeros(ctas * N_LAYER * nph, dtype=torch.int64, device=device)
    ctx.set_trace(buf)
    x = x_row.clone()
    ctx.layers(0, N_LAYER, x)
    torch.cuda.synchronize(device)
    ctx.set_trace(None)
    t = buf.view(ctas, N_LAYER, nph).cpu().numpy().astype(np.float64)
    if not t.any():
        return None
    out = {}
    for ph, name in TRACE_STAMPS:              # layers 0 .. N-2 (the last layer has no router partials)
        v = (t[:, :-1, ph] - t[:, :-1, 0]) / 1e3
        if (t[:, :-1, ph] == 0).any():
            continue
        out[name] = {"median": round(float(np.median(v, axis=0).mean()), 3), "max": round(float(v.max(axis=0).mean()), 3)}
    out["layer_total"] = round(float(np.median(t[:, 1:, 0] - t[:, :-1, 0]) / 1e3), 3)
    return out


# --------------------------------------------------------------------------------------------
def run_reference(args, rank, world):
    """The reference arm: the CPU restatement of hoard's ggml-CPU path, all host threads."""
    if rank != 0:
        return
    from oracle import oracle as orc
    threads = orc.max_threads()
    budget = max(2.0, min(20.0, 2.0 * args.steps))
    tok_s, sample = cpu_sample(budget, threads)
    line = {"metric": METRIC, "value": round(tok_s, 4), "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 / tok_s, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot (Q8_K) + f32",
            "data": "synthetic (seeded N(0,0.02) weights quantized Q4_K/Q6_K; seeded N(0,1) activations)",
            "config": {"workload": WORKLOAD, "T": 1, "layers": N_LAYER, "H": H, "E": E, "k": K_USED, "I": I},
            "cpu_baseline": {"value": round(tok_s, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(tok_s, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "hoard's own path (C++/Win32 over ggml b9660 Vulkan/CPU) is not vendored and cannot be "
                    "built here; this is the oracle's C++ restatement of its ggml CPU arithmetic"}
    print(json.dumps(line), flush=True)


PREFILL_T = 4096          # tokens per call of the prefill measurement (the C2 sweep's largest T)
C4_TOKENS = 64 * 2048     # C4: 64 sequences x 2048 tokens per prefill step, split over the ranks
C2_TS = (16, 512, 4096)   # isolated-layer sweep (C2: T in {1, 16, 512, 4096}; T = 1 is the decode line)


def layer_flops(T: int) -> float:
    """Algorithmic FLOPs of the expert FFN of one layer for T tokens: k experts x 3 matmuls x 2HI."""
    return 2.0 * T * K_USED * 3 * H * I


def measure_c2(ctx, x0, Ts, timed):
    """Isolated layer 0 of the context (C2: Q6_K down) at each T in Ts on the rows x0[:T]: us per layer
    call (events around 20 calls after 3), tok/s, expert-FFN TFLOP/s and the HBM roofline of the call's
    algorithmic bytes (the distinct experts its routing selects)."""
    try:
        hbm_peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"])
    except Exception:
        hbm_peak = 6650.0                                                    # the pool's fallback figure
    sweep = []
    for T in Ts:
        xt = x0[:T].clone()
        sel_t, _ = ctx.route(0, xt)
        nbytes = c2_layer_bytes(sel_t.cpu(), T)
        ms_l = timed(lambda: ctx.layer(0, xt), reps=20, warm=3)
        gbs = nbytes / (ms_l * 1e-3) / 1e9
        sweep.append({"T": T, "us_per_layer": round(ms_l * 1e3, 1), "tok_s": round(T / ms_l * 1e3, 1),
                      "expert_tflops": round(layer_flops(T) / (ms_l * 1e-3) / 1e12, 1),
                      "roofline": {"bound": "hbm", "algorithmic_bytes": int(nbytes), "achieved": round(gbs, 1),
                                   "peak": hbm_peak, "unit": "GB/s", "frac": round(gbs / hbm_peak, 4)}})
    return sweep


def run_c2_only(args, local_rank):
    """`--c2-only T,T,...`: the isolated C2 layer alone (one MoE layer, Q6_K down) at the given token
    counts, one JSON line; the command that the small-batch kernel profiles are taken with."""
    import torch
    from hoard_b200 import moe
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    Ts = [int(t) for t in args.c2_only.split(",")]
    ctx = moe.MoEContext(n_embd=H, n_expert=E, n_expert_used=K_USED, n_ff=I, n_layer=1, norm_topk=True, eps=1e-6,
                         resid_dtype=torch.float32, gate_types=[Q4_K], up_types=[Q4_K], down_types=[Q6_K],
                         max_tokens=max(Ts), device=local_rank)
    build_model(ctx, device, 1)
    if args.gemm_min_tokens is not None:
        ctx.set_gemm_min_tokens(args.gemm_min_tokens)
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 4096)
    x0 = torch.randn(max(Ts), H, generator=g, device=device)
    x0 = x0 / torch.sqrt((x0 * x0).mean(-1, keepdim=True) + 1e-6)
    stream = torch.cuda.current_stream(device)

    def timed(fn, reps, warm):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        b.record(stream)
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) / reps

    # bring the clocks up before the first timed call: ~0.5 s of layer calls at the largest T
    xw = x0.clone()
    t_end = time.time() + 0.5
    while time.time() < t_end:
        for _ in range(10):
            ctx.layer(0, xw)
        torch.cuda.synchronize(device)
    sweep = measure_c2(ctx, x0, Ts, timed)
    ctx.sync_status()
    ctx.close()
    print(json.dumps({"metric": "C2 isolated MoE layer (Qwen3-30B-A3B shape)", "c2_layer": sweep}))


def measure_prefill(ctx, device, stream, dist, rank=0, world=1, ep_chunks=1, ep_gemm_ctas=0, ep_transport="p2p"):
    """Batched tokens through the tensor-core expert path: the 48-layer stack at T = PREFILL_T tokens per
    call and rank (prefill tok/s; with world > 1 expert-parallel: experts [g*E/G, (g+1)*E/G) computed on
    rank g, tokens exchanged by NCCL all-to-all, weak scaling) and the isolated layer 0 (Q6_K down) at
    the C2 token counts. Inputs are seeded RMS-normalised rows resident in HBM, distinct per rank; every
    call streams all experts' weights of a layer (391 MB > 126 MB L2), so no flush is needed."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 4096 + 7 * rank)
    x0 = torch.randn(PREFILL_T, H, generator=g, device=device)
    x0 = x0 / torch.sqrt((x0 * x0).mean(-1, keepdim=True) + 1e-6)
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        tpeak, tsrc = float(peaks["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        tpeak, tsrc = 1400.0, "fallback (sustained)"

    def timed(fn, reps, warm):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize(device)
        if dist:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        b.record(stream)
        torch.cuda.synchronize(device)
        ms = a.elapsed_time(b) / reps
        if dist:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    x = x0.clone()
    # C4 as specified: 131,072 tokens per step through the 48 MoE layers, split evenly over the ranks
    # (strong scaling), each rank running its share as calls of PREFILL_T tokens; with G > 1 the experts
    # [g*E/G, (g+1)*E/G) are computed on rank g. `local_ms` times one call of PREFILL_T tokens with every
    # expert on this rank (the single-GPU rate) in the same run, for the efficiency figure.
    n_calls = max(1, C4_TOKENS // (world * PREFILL_T))
    local_ms = timed(lambda: ctx.layers(0, N_LAYER, x), reps=3, warm=1)
    x = x0.clone()
    imbalance = None
    if world > 1:
        from hoard_b200.ep import ExpertParallel
        sel, _ = ctx.route(0, x0)
        per_rank = torch.bincount((sel.view(-1) // (E // world)).long(), minlength=world).float()
        if dist:
            dist.all_reduce(per_rank)
        imbalance = float(per_rank.max() / per_rank.mean())
        ep = ExpertParallel(ctx, experts_per_rank=E // world, slot_base=rank * (E // world),
                            max_rows=PREFILL_T * K_USED * world, chunks=ep_chunks, transport=ep_transport)
        ctx.set_gemm_ctas(ep_gemm_ctas if ep_chunks > 1 and ep_transport == "nccl" else 0)

        def step():
            for _ in range(n_calls):
                ep.layers(0, N_LAYER, x)
        ms = timed(step, reps=2, warm=1)
        ctx.set_gemm_ctas(0)
        ep.close()
    else:
        def step():
            for _ in range(n_calls):
                ctx.layers(0, N_LAYER, x)
        ms = timed(step, reps=2, warm=1)
    ctx.sync_status()
    sweep = measure_c2(ctx, x0, C2_TS, timed)
    ctx.sync_status()
    achieved = layer_flops(PREFILL_T) * N_LAYER * n_calls / (ms * 1e-3) / 1e12    # per GPU
    traffic = None
    try:
        traffic = json.load(open(os.path.join(ROOT, "profiles", "traffic.json"))).get("prefill_gateup_T4096_bytes")
    except Exception:
        pass
    tok_s = C4_TOKENS / ms * 1e3 if n_calls * world * PREFILL_T == C4_TOKENS else PREFILL_T * n_calls * world / ms * 1e3
    local_tok_s = PREFILL_T / local_ms * 1e3
    return {"metric": f"prefill tok/s (C4: {C4_TOKENS} tokens per step through {N_LAYER} MoE layers, split over the "
                      f"GPUs; {PREFILL_T} tokens per call)",
            "value": tok_s, "unit": "tok/s", "ms_per_step": round(ms, 3), "scaling": "strong",
            "tokens_per_step": C4_TOKENS, "calls_per_rank": n_calls,
            "single_gpu_tok_s": round(local_tok_s, 1),
            "efficiency_vs_single_gpu": round(tok_s / (world * local_tok_s), 4),
            "speedup_vs_single_gpu": round(tok_s / local_tok_s, 3),
            "expert_load_imbalance": None if imbalance is None else round(imbalance, 4),
            "imbalance_note": "entries received by the busiest rank / the mean over ranks (one call's routing)",
            "parallelism": (("ep{} (dispatch/combine by the library's kernels over NVLink peer memory)".format(world)
                             if ep_transport == "p2p" else
                             f"ep{world} (NCCL all-to-all dispatch/combine, {ep_chunks} micro-batches"
                             f"{f', GEMMs on {ep_gemm_ctas} CTAs' if ep_chunks > 1 and ep_gemm_ctas else ''})")
                            if world > 1 else "single GPU"),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": tpeak, "unit": "TFLOP/s",
                         "frac": round(achieved / tpeak, 4), "peak_source": tsrc,
                         "flops": "expert FFN only: 2*T*k*3*H*I per layer (router, dispatch, combine excluded)",
                         "timing": "whole prefill step (all kernels of 48 layers), not the GEMM alone",
                         "traffic": traffic,
                         "traffic_kernel": "k_tc_experts<0> (gate/up GEMM), DRAM bytes per launch at T=4096"},
            "c2_layer": sweep}


C1_PROMPT, C1_GEN = 16, 64


def measure_c1_decode(device):
    """C1: the OLMoE-shape model (16 layers, MHA 16 x 128 with QK norm over the whole projection, 64
    experts top-8 without renorm, I 1024, vocab 50304, Q4_K_M, f16 KV cache), seeded weights, greedy
    decode of 64 tokens after a 16-token prompt through the device driver (hoard_b200.harness): one
    captured CUDA graph per token (embedding, 16 x (attention + MoE layer), lm-head, argmax), timed
    with CUDA events around the 64 replays."""
    import torch
    from hoard_b200 import harness as hx
    cfg = hx.C1_OLMOE
    model = hx.DecodeModel(cfg, hx.seeded_tensors(cfg, seed=SEED + 101, device=device), device=device.index,
                           max_ctx=C1_PROMPT + C1_GEN + 8)
    try:
        g = torch.Generator().manual_seed(SEED + 102)
        prompt = torch.randint(0, cfg.n_vocab, (C1_PROMPT,), generator=g).tolist()
        model.generate_graphed(prompt, 8)                      # warm-up (capture + replays)
        graph = model.capture()
        model.prefill(prompt)
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(C1_GEN):
            graph.replay()
        b.record()
        torch.cuda.synchronize(device)
        model.moe.sync_status()
        ms = a.elapsed_time(b)
        toks = model.seq[C1_PROMPT:C1_PROMPT + C1_GEN].tolist()
        return {"metric": "C1 decode tok/s (OLMoE shape, whole model: 16 layers attention + MoE, lm-head)",
                "value": round(C1_GEN / ms * 1e3, 1), "unit": "tok/s", "ms_per_token": round(ms / C1_GEN, 4),
                "prompt": C1_PROMPT, "generated": C1_GEN, "distinct_tokens": len(set(toks)),
                "kv_cache": "f16", "timing": "CUDA events around 64 replays of the captured per-token graph"}
    finally:
        model.close()


C3_PROMPT, C3_GEN, C3_CTX = 512, 256, 4096
C5_PROMPT, C5_GEN, C5_CTX = 1024, 256, 2048


def measure_c3_decode(device):
    """C3: the Qwen3-30B-A3B-shape model (48 layers, GQA 32/4 x 128, per-head QK norm, theta 1e6,
    vocab 151936, 128 experts top-8 + renorm, I 768, Q4_K_M, 4096-slot bf16 KV cache), seeded weights,
    every expert resident; a 512-token prompt, then 256 greedy tokens."""
    from hoard_b200 import harness as hx
    return measure_whole_decode(device, hx.C3_QWEN3, C3_PROMPT, C3_GEN, C3_CTX, SEED + 303,
                                "C3 decode tok/s (Qwen3-30B-A3B shape, whole model: 48 layers attention + MoE, lm-head)")


def measure_c5_decode(device):
    """C5: the Qwen3-Next-80B-A3B-shape hybrid model (48 layers: 36 gated delta-net + 12 gated attention
    with 16 q / 2 KV heads of 256, RoPE on 64 dims; 512 experts top-10 + renorm, I 512, a gated shared
    expert of 512; vocab 151936; Q4_K_M), seeded weights, every expert resident, bf16 KV cache for the
    attention layers; a 1024-token prompt, then 256 greedy tokens."""
    from hoard_b200 import harness as hx
    return measure_whole_decode(device, hx.C5_QWEN3NEXT, C5_PROMPT, C5_GEN, C5_CTX, SEED + 505,
                                "C5 decode tok/s (Qwen3-Next-80B-A3B shape, whole model: 36 delta-net + 12 gated "
                                "attention layers, MoE with a shared expert, lm-head)")


def measure_whole_decode(device, cfg, n_prompt, n_gen, ctx, seed, metric):
    """Whole-model greedy decode of a seeded model: the prompt through the per-token step, then n_gen
    tokens, each one replay of the captured per-token graph (embedding, the layers' attention or
    delta-net blocks + MoE layers, lm-head, argmax), timed with CUDA events around the replays. The MoE
    share is n_layer single-layer MoE launches (the graph's own MoE calls) timed alone on the same
    context."""
    import torch
    from hoard_b200 import harness as hx
    tensors = hx.seeded_tensors(cfg, seed=seed, device=device)
    model = hx.DecodeModel(cfg, tensors, device=device.index, max_ctx=ctx, kv_dtype=torch.bfloat16)
    del tensors
    torch.cuda.empty_cache()
    try:
        g = torch.Generator().manual_seed(seed + 1)
        prompt = torch.randint(0, cfg.n_vocab, (n_prompt,), generator=g).tolist()
        graph = model.capture()
        model.prefill(prompt)
        for _ in range(4):                                    # warm-up replays
            graph.replay()
        model.prefill(prompt)
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n_gen):
            graph.replay()
        b.record()
        torch.cuda.synchronize(device)
        model.moe.sync_status()
        ms = a.elapsed_time(b)
        toks = model.seq[n_prompt:n_prompt + n_gen].tolist()
        xb = torch.zeros(1, cfg.n_embd, device=device)
        xb.normal_()
        for il in range(cfg.n_layer):
            model.moe.layers(il, 1, xb)
        torch.cuda.synchronize(device)
        a.record()
        for _ in range(10):
            for il in range(cfg.n_layer):
                model.moe.layers(il, 1, xb)
        b.record()
        torch.cuda.synchronize(device)
        moe_ms = a.elapsed_time(b) / 10
        return {"metric": metric, "value": round(n_gen / ms * 1e3, 1), "unit": "tok/s",
                "ms_per_token": round(ms / n_gen, 4), "prompt": n_prompt, "generated": n_gen,
                "distinct_tokens": len(set(toks)), "kv_cache": f"bf16, {ctx} slots", "moe_ms_per_token": round(moe_ms, 4),
                "moe_share": round(moe_ms / (ms / n_gen), 3),
                "timing": f"CUDA events around {n_gen} replays of the captured per-token graph; the MoE share from "
                          f"{cfg.n_layer} single-layer MoE launches timed alone"}
    finally:
        model.close()


LRU_SLOTS = 32       # C3 run (ii): K = 32 slots per layer
LRU_TOKENS = 8
LRU_SKEW_TOKENS = 16   # tokens of the skewed-routing variant
ZIPF_S = 1.0           # expert popularity exponent of the skewed variant


def measure_lru(device, stream, n_layer: int):
    """C3 run (ii): batch-1 decode through a K = 32 per-layer LRU slot pool backed by a pinned-host RAM
    tier, hoard's own schedule: per layer route (T = 1) -> host readback of the 8 expert ids ->
    hoard_moe_ensure (misses uploaded on the library's upload stream) -> experts on the slots. The RAM
    tier holds layer 0's 128 experts (392 MB pinned) and serves every layer (same bytes, same traffic
    as distinct layers); routers are the benchmark model's. Timed with CUDA events around whole
    tokens (host round trips included)."""
    import numpy as np
    import torch
    from hoard_b200 import moe, quant
    ctx = moe.MoEContext(n_embd=H, n_expert=E, n_expert_used=K_USED, n_ff=I, n_layer=n_layer, n_slots=LRU_SLOTS,
                         norm_topk=True, eps=1e-6, resid_dtype=torch.float32, gate_types=[Q4_K] * n_layer,
                         up_types=[Q4_K] * n_layer, down_types=[down_type(layer) for layer in range(n_layer)],
                         max_tokens=1, device=device.index)
    ctx.set_decode_impl(0)
    ctx.set_gemm_min_tokens(0)
    g = torch.Generator(device=device)
    host = {}
    for dt in sorted(set(down_type(layer) for layer in range(n_layer))):
        g.manual_seed(SEED + 31 * dt)
        gate = quant.quantize_q4k(torch.randn(E, I, H, generator=g, device=device) * 0.02).cpu().pin_memory()
        up = quant.quantize_q4k(torch.randn(E, I, H, generator=g, device=device) * 0.02).cpu().pin_memory()
        down = quant.quantize(torch.randn(E, H, I, generator=g, device=device) * 0.02, dt).cpu().pin_memory()
        host[dt] = (gate, up, down)
    for layer in range(n_layer):
        g.manual_seed(SEED + 7919 * layer)
        ctx.set_router(layer, torch.randn(E, H, generator=g, device=device) * 0.02,
                       1.0 + 0.1 * torch.randn(H, generator=g, device=device))
        gate, up, down = host[down_type(layer)]
        for e in range(E):
            ctx.ram_tier(layer, e, gate[e], up[e], down[e])
    xs = token_rows(LRU_TOKENS + 2, device)
    slot_dev = torch.empty(K_USED, dtype=torch.int32, device=device)

    def token(x):
        for layer in range(n_layer):
            sel, w = ctx.route(layer, x)
            slots = ctx.ensure(layer, sel.cpu().numpy())
            slot_dev.copy_(torch.from_numpy(slots), non_blocking=False)
            ctx.experts(layer, sel, w, x, slot_of_sel=slot_dev)

    for i in range(2):                                   # warm-up: fills the pool
        token(xs[LRU_TOKENS + i].clone())
    torch.cuda.synchronize(device)
    st0 = ctx.residency_stats()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(LRU_TOKENS):
        token(xs[i].clone())
    b.record(stream)
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b)
    ctx.sync_status()
    st = ctx.residency_stats()
    hits, misses = st["hits"] - st0["hits"], st["misses"] - st0["misses"]
    up_bytes = st["bytes_uploaded"] - st0["bytes_uploaded"]
    out = {"metric": f"decode tok/s b=1, {LRU_SLOTS}-slot LRU per layer + pinned-host RAM tier ({n_layer} layers)",
           "value": round(LRU_TOKENS / (ms * 1e-3), 3), "unit": "tok/s", "tokens": LRU_TOKENS,
           "hit_rate": round(hits / max(1, hits + misses), 4), "misses_per_token": round(misses / LRU_TOKENS, 1),
           "h2d_gbs": round(up_bytes / (ms * 1e-3) / 1e9, 2),
           "note": "uniform random routing on random weights: the hit rate is the pool's share of experts"}

    # Skewed variant: the same schedule (the router still runs and its ids are read back), but the
    # experts computed are drawn per layer from a Zipf(s = 1.0) law over a fixed random permutation of
    # the experts -- the skew fitted to hoard's real routing traces -- with weights 1/k. Ids are drawn
    # before the timed region.
    rng = np.random.default_rng(SEED)
    prob = 1.0 / np.arange(1, E + 1) ** ZIPF_S
    prob /= prob.sum()
    perms = [rng.permutation(E) for _ in range(n_layer)]
    n_tok = LRU_SKEW_TOKENS + 4
    draws = [[perms[layer][rng.choice(E, K_USED, replace=False, p=prob)].astype(np.int32) for layer in range(n_layer)]
             for _ in range(n_tok)]
    w_flat = torch.full((1, K_USED), 1.0 / K_USED, device=device)
    sel_dev = torch.empty(1, K_USED, dtype=torch.int32, device=device)

    def token_skewed(x, ids):
        for layer in range(n_layer):
            sel, _ = ctx.route(layer, x)
            sel.cpu()
            slots = ctx.ensure(layer, ids[layer])
            sel_dev.copy_(torch.from_numpy(ids[layer]).view(1, K_USED))
            slot_dev.copy_(torch.from_numpy(slots), non_blocking=False)
            ctx.experts(layer, sel_dev, w_flat, x, slot_of_sel=slot_dev)

    for i in range(4):                                   # warm-up: the pool takes the skewed working set
        token_skewed(xs[i % LRU_TOKENS].clone(), draws[LRU_SKEW_TOKENS + i])
    torch.cuda.synchronize(device)
    st0 = ctx.residency_stats()
    a.record(stream)
    for i in range(LRU_SKEW_TOKENS):
        token_skewed(xs[i % LRU_TOKENS].clone(), draws[i])
    b.record(stream)
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b)
    ctx.sync_status()
    st = ctx.residency_stats()
    hits, misses = st["hits"] - st0["hits"], st["misses"] - st0["misses"]
    up_bytes = st["bytes_uploaded"] - st0["bytes_uploaded"]
    out["skewed"] = {"value": round(LRU_SKEW_TOKENS / (ms * 1e-3), 3), "unit": "tok/s", "tokens": LRU_SKEW_TOKENS,
                     "hit_rate": round(hits / max(1, hits + misses), 4),
                     "misses_per_token": round(misses / LRU_SKEW_TOKENS, 1),
                     "h2d_gbs": round(up_bytes / (ms * 1e-3) / 1e9, 2),
                     "routing": f"expert ids per layer ~ Zipf(s = {ZIPF_S}) over a fixed permutation, weights 1/k"}
    ctx.close()
    return out


def run_gpu(args, rank, world, local_rank):
    import torch
    from hoard_b200 import moe

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    ctx = moe.MoEContext(n_embd=H, n_expert=E, n_expert_used=K_USED, n_ff=I, n_layer=N_LAYER, norm_topk=True,
                         eps=1e-6, resid_dtype=torch.float32, gate_types=[Q4_K] * N_LAYER, up_types=[Q4_K] * N_LAYER,
                         down_types=[down_type(layer) for layer in range(N_LAYER)],
                         max_tokens=PREFILL_T if not args.no_prefill else 16, device=local_rank)
    if args.decode_impl is not None:
        ctx.set_decode_impl(args.decode_impl)
    build_model(ctx, device, N_LAYER)
    steps, warm = args.steps, args.warmup
    xs = token_rows(steps + warm, device)
    sel = torch.empty(steps + warm, N_LAYER, 1, K_USED, dtype=torch.int32, device=device)
    wts = torch.empty(steps + warm, N_LAYER, 1, K_USED, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)

    # ---- device-resident timing ----
    for i in range(warm):
        ctx.layers(0, N_LAYER, xs[steps + i], sel[steps + i], wts[steps + i])
    ctx.sync_status()
    if dist:
        dist.barrier()
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        # the timed region is tens of ms, shorter than nvidia-smi's sampling period: keep the GPU in the
        # same decode loop for ~0.5 s first, so the clock samples see the load the timed steps run under
        t_pre = time.time()
        while time.time() - t_pre < 0.5:
            for i in range(warm):
                ctx.layers(0, N_LAYER, xs[steps + i], sel[steps + i], wts[steps + i])
            torch.cuda.synchronize(device)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(device)
        launches0 = ctx.launch_count
        ev0.record(stream)
        for i in range(steps):
            ctx.layers(0, N_LAYER, xs[i], sel[i], wts[i])
        ev1.record(stream)
        torch.cuda.synchronize(device)
    launches = ctx.launch_count - launches0
    ms = ev0.elapsed_time(ev1)
    ctx.sync_status()
    if dist:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_step = ms / steps

    sel_h = sel[:steps].cpu().numpy()
    bytes_step = float(np.mean([algorithmic_bytes_per_token(sel_h[i]) for i in range(steps)]))

    # ---- end to end through the public API with host buffers ----
    x_host = token_rows(steps + warm, device).cpu().pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    xbuf = torch.empty(1, H, device=device)
    for i in range(warm):
        xbuf.copy_(x_host[i], non_blocking=True)
        ctx.layers(0, N_LAYER, xbuf)
        out_host[i].copy_(xbuf, non_blocking=True)
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        xbuf.copy_(x_host[i], non_blocking=True)
        ctx.layers(0, N_LAYER, xbuf)
        out_host[i].copy_(xbuf, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(device)
    ms_e2e = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms_e2e], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())

    phases = None
    if args.trace:
        phases = trace_breakdown(ctx, xs[0], device)

    prefill = None
    if not args.no_prefill:
        prefill = measure_prefill(ctx, device, stream, dist, rank, world, args.ep_chunks, args.ep_gemm_ctas,
                                  args.ep_transport)

    lru = None
    if not args.no_lru and rank == 0 and world == 1:
        lru = measure_lru(device, stream, N_LAYER)

    c1 = None
    if not args.no_c1 and rank == 0 and world == 1:
        c1 = measure_c1_decode(device)

    c3 = None
    if not args.no_c3 and rank == 0 and world == 1:
        c3 = measure_c3_decode(device)
        torch.cuda.empty_cache()

    c5 = None
    if not args.no_c5 and rank == 0 and world == 1:
        c5 = measure_c5_decode(device)
        torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as orc
        threads = orc.max_threads()
        tok_s_cpu, sample = cpu_sample(args.cpu_seconds, threads)
        cpu = {"value": round(tok_s_cpu, 4), "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        peak, peak_src = float(peaks["hbm_gbs"]), "measured"
    except Exception:
        peak, peak_src = 6650.0, "fallback"
    achieved = bytes_step / (ms_step * 1e-3) / 1e9
    traffic = None
    try:
        # DRAM bytes of one 48-layer step from an ncu capture (profiles/), scaled to the layers run
        traffic = json.load(open(os.path.join(ROOT, "profiles", "traffic.json"))).get("decode_step_bytes")
        traffic = int(traffic * N_LAYER / 48) if traffic else None
    except Exception:
        pass
    if rank == 0:
        tok_s = world * 1000.0 / ms_step
        line = {
            "metric": METRIC, "value": round(tok_s, 3), "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 dot (Q8_K x Q4_K/Q6_K) + f32",
            "data": "synthetic (seeded N(0,0.02) weights quantized Q4_K/Q6_K on device; seeded N(0,1) "
                    "RMS-normalised token rows)",
            "config": {"workload": WORKLOAD, "T": 1, "layers": N_LAYER, "H": H, "E": E, "k": K_USED, "I": I,
                       "down_types": "Q6_K even / Q4_K odd", "resid": "f32",
                       "parallelism": f"replicas x{world} (decode does not shard)",
                       "l2": "1.2 GB of distinct weights per step > 126 MB L2; no flush"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "peak_source": peak_src, "bytes_per_step": int(bytes_step),
                         "kernel": f"k_decode: one launch = the whole decode step ({N_LAYER} layers)"},
            "e2e": {"value": round(world * 1000.0 * steps / ms_e2e, 3), "unit": "tok/s",
                    "h2d_bytes_per_step": H * 4, "d2h_bytes_per_step": H * 4},
            "gpu_launches": int(launches),
            "clocks": dict(clk.summary(), window="0.5 s of the same decode steps, then the timed steps"),
        }
        if prefill:
            prefill["value"] = round(prefill["value"], 1)           # whole job: C4's tokens over all ranks
        if lru:
            line["lru_decode"] = lru
        if prefill:
            line["prefill"] = prefill
        if c1:
            line["c1_decode"] = c1
        if c3:
            line["c3_decode"] = c3
        if c5:
            line["c5_decode"] = c5
        if cpu:
            line["cpu_baseline"] = cpu
        if phases:
            line["phase_us"] = phases
        print(json.dumps(line), flush=True)
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    global N_LAYER
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="hoard_b200", choices=["hoard_b200", "reference"])
    ap.add_argument("--decode-impl", type=int, default=None, help="0 grouped kernels, 1 persistent kernel")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--trace", action="store_true", help="add the persistent kernel's per-phase breakdown")
    ap.add_argument("--no-prefill", action="store_true", help="skip the batched-token (prefill) measurements")
    ap.add_argument("--no-lru", action="store_true", help="skip the LRU slot pool + RAM tier decode measurement")
    ap.add_argument("--no-c1", action="store_true", help="skip the C1 whole-model decode (device driver) measurement")
    ap.add_argument("--no-c3", action="store_true", help="skip the C3 whole-model decode (device driver) measurement")
    ap.add_argument("--no-c5", action="store_true", help="skip the C5 whole-model (hybrid) decode measurement")
    ap.add_argument("--c2-only", default=None, help="comma-separated token counts: time only the isolated C2 layer")
    ap.add_argument("--gemm-min-tokens", type=int, default=None,
                    help="with --c2-only: T at or above which the tensor-core path runs (0: never)")
    ap.add_argument("--ep-transport", default="p2p", choices=["p2p", "nccl"],
                    help="expert-parallel prefill exchange: the library's peer-memory kernels or NCCL all-to-all")
    ap.add_argument("--ep-chunks", type=int, default=2, help="expert-parallel prefill: micro-batches per layer "
                    "whose all-to-alls overlap the other micro-batches' GEMMs")
    ap.add_argument("--ep-gemm-ctas", type=int, default=132, help="expert-parallel prefill with micro-batches: "
                    "CTAs of the tensor-core GEMMs (the remaining SMs run NCCL's kernels)")
    ap.add_argument("--layers", type=int, default=N_LAYER, help="MoE layers per step (48 = the full stack; "
                    "fewer only for small profiling captures)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    N_LAYER = args.layers
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.c2_only:
        run_c2_only(args, local_rank)
    else:
        run_gpu(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
