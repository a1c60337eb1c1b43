#!/usr/bin/env python
"""Benchmark of the per-action-chunk denoising path on B200.

Workload (the configuration the metric is quoted on):
the baseline action expert — ActionDiT hidden 1024, 16 heads x 64, 28 blocks,
FFN 4096, text_dim 4096 — denoising one 32 x 7 action chunk in 10 Euler
flow-matching steps (shift 1) with joint attention over a cached 1760-token
video K/V per block (N(0,1), all-True joint mask) and cross attention to a
64-token text context, batch 1.  Weights are seeded random-init of the
reference architecture (default nn.Linear init, modulation randn/sqrt(D)); all
inputs are seeded synthetic tensors (no dataset or checkpoint exists here).

One bench step = one whole action chunk (10 model evaluations + Euler updates)
replayed from a CUDA graph.  `value` = chunks/s over all ranks with inputs
resident in HBM (device time, CUDA events, max over ranks); `e2e` = the same
through the public engine call with the chunk's inputs copied from pinned host
memory every step and the final chunk read back.  The working set of one
chunk (0.82 GB of weights per model evaluation + 0.20 GB of K/V cache) is far
larger than the 126 MB L2, so no L2 flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl fam|reference]

(`--euler-steps N` shortens the chunk for ncu captures of the fused kernel; the
reported workload name then no longer matches the metric's configuration.)

`--impl reference` times the reference algorithm's CPU implementation (the
CPU oracle restating FastWAM's PyTorch code, bf16 like the reference model)
on this host's cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import csv
import importlib
import io
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "action-chunk latency p50 ms (bs=1); chunks/sec at 1/2/4/8 B200 vs roofline"
CFG = dict(hidden_dim=1024, action_dim=7, ffn_dim=4096, text_dim=4096, freq_dim=256, eps=1e-6,
           num_heads=16, attn_head_dim=64, num_layers=28)
SA, SV, CTX, NSTEPS, SHIFT = 32, 1760, 64, 10, 1.0
# DRAM read + write of fused_chunk_kernel per Euler step: one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum) of this workload at 2 Euler
# steps, 2,079,377,664 B / 2.  Every step streams the same weights and K/V, so a
# launch's traffic scales with the step count.
FUSED_DRAM_BYTES_PER_STEP = 1_039_688_832


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = [r for r in csv.reader(io.StringIO(self.out or "")) if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        load = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(load) if load else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def build_workload(dev, seed=0):
    M = importlib.import_module("faster-action-models_b200.models")
    torch.manual_seed(seed)
    dit = M.ActionDiT(**CFG).to(torch.bfloat16).to(dev)
    g = torch.Generator(device="cpu").manual_seed(1000 + seed)
    D = CFG["hidden_dim"]
    HD = CFG["num_heads"] * CFG["attn_head_dim"]
    L = CFG["num_layers"]
    cache_k = torch.randn(L, 1, SV, HD, generator=g).bfloat16().to(dev)
    cache_v = torch.randn(L, 1, SV, HD, generator=g).bfloat16().to(dev)
    ctx = torch.randn(1, CTX, CFG["text_dim"], generator=g).bfloat16()
    cm = torch.ones(1, CTX, dtype=torch.uint8)  # bool masks passed as uint8 (True = attend)
    noise = torch.randn(1, SA, CFG["action_dim"], generator=g).bfloat16()
    mask = torch.ones(SA, SV + SA, dtype=torch.uint8)
    return M, dit, cache_k, cache_v, ctx, cm, noise, mask


def algorithmic_bytes_per_chunk(dit) -> dict:
    """Bytes a chunk must move at least once: per model evaluation the weights of
    every block except the hoisted cross K/V projections, plus the head/encoder,
    plus the K/V cache; per chunk the hoisted context projections and time MLP."""
    D = CFG["hidden_dim"]
    HD = CFG["num_heads"] * CFG["attn_head_dim"]
    F = CFG["ffn_dim"]
    L = CFG["num_layers"]
    per_block = (3 * HD * D + HD * D + HD * D + HD * D + F * D + D * F) * 2 + (6 * D) * 2
    per_eval = L * per_block + (2 * SA * CFG["action_dim"] + D * CFG["action_dim"] * 2) * 2
    kv = L * 2 * SV * HD * 2
    prologue = (CFG["text_dim"] * D + D * D + CFG["freq_dim"] * D + D * D + 6 * D * D) * 2 \
        + L * 2 * HD * D * 2 + CTX * CFG["text_dim"] * 2
    total = prologue + NSTEPS * (per_eval + kv)
    flops = NSTEPS * (2 * SA * L * (3 * HD * D + 2 * HD * D + 2 * HD * D + 2 * F * D)
                      + 4 * SA * (SV + SA) * HD * L + 4 * SA * CTX * HD * L)
    return {"bytes": total, "per_eval_weights": per_eval, "kv": kv, "prologue": prologue,
            "flops": flops}


def time_dominant_kernel(M, dit, dev, reps=5):
    """The weight-streaming GEMM of the FFN down projection (ffn.2: [1024, 4096] bf16,
    split-K, weights-as-A) over all 28 blocks' weights, timed with CUDA events on the
    launching stream.  Returns (avg ms per launch, algorithmic bytes per launch)."""
    ops = importlib.import_module("faster-action-models_b200.ops")
    F, D = CFG["ffn_dim"], CFG["hidden_dim"]
    x = torch.randn(SA, F, device=dev).bfloat16()
    ws = [b.ffn[2].weight.detach().contiguous() for b in dit.blocks]
    outs = torch.empty(16, SA, D, device=dev)
    for w in ws:  # warm-up (tensor maps, attributes)
        ops.gemm(w, x, weights_as_a=True, splits=16, out=outs)
    torch.cuda.synchronize()
    # Back-to-back launches replayed from a CUDA graph (programmatic launch, as in
    # the chunk chain) so that host launch overhead is not timed.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            for w in ws:
                ops.gemm(w, x, weights_as_a=True, splits=16, out=outs, pdl=True)
    graph.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    graph.replay()
    e.record()
    torch.cuda.synchronize()
    per = s.elapsed_time(e) / (reps * len(ws))
    alg = F * D * 2 + SA * F * 2 + SA * D * 2
    return per, alg


def time_fused_kernel(eng, chunk, reps=5):
    """The fused persistent chunk kernel alone: CUDA events recorded by the library
    on the launching stream immediately around its launch (fam_action_set_kernel_events)
    in plain (not graph-replayed) chunk calls, averaged over `reps` chunks.  Returns
    ms per launch."""
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    e.record()
    torch.cuda.synchronize()  # torch creates the CUDA events on first record
    eng.set_kernel_events(s, e)
    times = []
    try:
        for _ in range(reps + 1):
            chunk()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
    finally:
        eng.set_kernel_events(None, None)
    return statistics.mean(times[1:])


def cpu_reference_chunks_per_s(n_steps_timed: int, warmup: int = 1):
    """The reference algorithm on this host's CPU cores (bf16, like the reference model):
    one sample = one model evaluation of the chunk; chunks/s = 1 / (10 x eval time)."""
    from oracle import fam_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    M, dit, ck, cv, ctx, cm, noise, mask = build_workload("cpu")
    sd = {k: v.bfloat16() for k, v in dit.state_dict().items()}
    cfg = O.DiTConfig(hidden_dim=CFG["hidden_dim"], ffn_dim=CFG["ffn_dim"],
                      num_heads=CFG["num_heads"], attn_head_dim=CFG["attn_head_dim"],
                      num_layers=CFG["num_layers"], text_dim=CFG["text_dim"],
                      action_dim=CFG["action_dim"])
    ts, ds = O.build_inference_schedule(NSTEPS, SHIFT, dtype=torch.bfloat16)
    ckl, cvl = list(ck[:, :]), list(cv[:, :])
    times = []
    with torch.no_grad():
        for i in range(warmup + n_steps_timed):
            t0 = time.perf_counter()
            O.denoise_action_with_video_cache(sd, cfg, noise, ts[i % NSTEPS].reshape(1), ctx,
                                              cm.bool(), ckl, cvl, mask.bool())
            dt = time.perf_counter() - t0
            if i >= warmup:
                times.append(dt)
    per_eval = statistics.mean(times)
    return 1.0 / (NSTEPS * per_eval), torch.get_num_threads(), len(times), per_eval


def run_reference(args):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    cps, cores, n, per_eval = cpu_reference_chunks_per_s(args.steps, args.warmup)
    sample = (f"{n} single model evaluations of the 10-step chunk after {args.warmup} warm-up; "
              f"chunk time = 10 x {per_eval * 1e3:.1f} ms")
    line = {"metric": METRIC, "impl": "reference", "value": cps, "unit": "chunks/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 / cps, "latency_p50_ms": 1e3 / cps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded), random-init weights",
            "config": {"workload": "BASELINE configs[1]: action expert 1024h/16x64/28 blocks, "
                                   "1760-token K/V cache, 64-token context, 10 Euler steps, bs=1",
                       "device": "cpu"},
            "cpu_baseline": {"value": cps, "unit": "chunks/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": cps, "unit": "chunks/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_fam(args):
    ws, rank, local = _dist()
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    M, dit, ck, cv, ctx, cm, noise, mask = build_workload(dev, seed=rank)
    eng = dit.engine()
    ts, ds = M.build_inference_schedule(NSTEPS, SHIFT)
    ctx_d, cm_d, noise_d, mask_d = ctx.to(dev), cm.to(dev), noise.to(dev), mask.to(dev)
    lat = noise_d.clone()
    cks, cvs = list(ck), list(cv)

    def chunk():
        lat.copy_(noise_d)
        eng.chunk(lat, ts, ds, ctx_d, cm_d, cks, cvs, mask_d, out=lat)

    for _ in range(max(3, args.warmup)):
        chunk()
    torch.cuda.synchronize()
    launches = eng.launch_count()
    K = args.steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0.record()
        for i in range(K):
            starts[i].record()
            chunk()
            ends[i].record()
        t1.record()
        torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    elapsed_ms = t0.elapsed_time(t1)
    lat_ms = sorted(s.elapsed_time(e) for s, e in zip(starts, ends))
    p50 = lat_ms[len(lat_ms) // 2]
    tmax = torch.tensor([elapsed_ms, p50], device=dev)
    if ws > 1:
        torch.distributed.all_reduce(tmax, op=torch.distributed.ReduceOp.MAX)
    elapsed_ms, p50_max = tmax.tolist()

    # ---- end to end: pinned host inputs -> device, chunk, result -> host, every step
    noise_h = noise.pin_memory()
    ctx_h = ctx.pin_memory()
    cm_h = cm.to(torch.uint8).pin_memory()
    out_h = torch.empty(SA, CFG["action_dim"], dtype=torch.float32).pin_memory()
    cm_u8 = torch.empty(1, CTX, dtype=torch.uint8, device=dev)

    def chunk_e2e():
        lat.copy_(noise_h, non_blocking=True)
        ctx_d.copy_(ctx_h, non_blocking=True)
        cm_u8.copy_(cm_h, non_blocking=True)
        eng.chunk(lat, ts, ds, ctx_d, cm_u8, cks, cvs, mask_d, out=lat)
        out_h.copy_(lat[0].float(), non_blocking=True)

    for _ in range(3):
        chunk_e2e()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(K):
        chunk_e2e()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if ws > 1:
        torch.distributed.all_reduce(e2e_ms, op=torch.distributed.ReduceOp.MAX)
    e2e_ms = e2e_ms.item()
    h2d = noise_h.numel() * 2 + ctx_h.numel() * 2 + cm_h.numel()
    d2h = out_h.numel() * 4

    path = eng.last_path()
    alg = algorithmic_bytes_per_chunk(dit)
    if path == "fused":
        def chunk_eager():
            lat.copy_(noise_d)
            eng.chunk(lat, ts, ds, ctx_d, cm_d, cks, cvs, mask_d, out=lat, use_graph=False)
        k_ms = time_fused_kernel(eng, chunk_eager)
        k_bytes = NSTEPS * (alg["per_eval_weights"] + alg["kv"])
        k_name = "fused_chunk_kernel (persistent: every step and block of the chunk, 1 launch)"
        k_traffic = FUSED_DRAM_BYTES_PER_STEP * NSTEPS
    else:
        k_ms, k_bytes = time_dominant_kernel(M, dit, dev)
        k_name = "gemm_bf16_tc_kernel<32> (ffn.2 weight stream, split-K 16)"
        k_traffic = None
    if rank == 0:
        hbm, tc, src = _peaks()
        chunk_ms = elapsed_ms / K
        value = ws * K / (elapsed_ms / 1e3)
        line = {
            "metric": METRIC, "value": value, "unit": "chunks/s", "n_gpus": ws, "steps": K,
            "warmup": max(3, args.warmup), "ms_per_step": chunk_ms, "latency_p50_ms": p50_max,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) inputs and K/V cache), random-init weights",
            "config": {"workload": "BASELINE configs[1]: action expert 1024h/16x64/28 blocks, "
                                   f"1760-token K/V cache, 64-token context, {NSTEPS} Euler steps",
                       "batch_per_gpu": 1, "action_tokens": SA, "video_tokens": SV,
                       "context_tokens": CTX, "euler_steps": NSTEPS, "parallelism": f"replicas x{ws}",
                       "l2": "working set per chunk (8.2 GB weights + 2 GB K/V streamed) >> 126 MB L2; no flush"},
            "path": path,
            "roofline": {"bound": "hbm", "kernel": k_name,
                         "achieved": k_bytes / (k_ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": k_bytes / (k_ms * 1e-3) / 1e9 / hbm, "traffic": k_traffic,
                         "peak_source": src, "avg_launch_us": k_ms * 1e3,
                         "bytes_per_launch": k_bytes},
            "chunk_roofline": {"bound": "hbm", "bytes_per_chunk": alg["bytes"],
                               "floor_ms": alg["bytes"] / (hbm * 1e9) * 1e3,
                               "achieved_gbs": alg["bytes"] / (chunk_ms * 1e-3) / 1e9,
                               "frac": alg["bytes"] / (hbm * 1e9) * 1e3 / chunk_ms,
                               "flops_per_chunk": alg["flops"]},
            "e2e": {"value": ws * K / (e2e_ms / 1e3), "unit": "chunks/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "K/V cache and weights resident (model state); per step the noise, "
                            "context and mask go H2D and the chunk D2H"},
            "gpu_launches": launches * K,
            "clocks": clk.summary(),
        }
        if ws == 1 and not args.no_cpu_baseline:
            cps, cores, n, per_eval = cpu_reference_chunks_per_s(max(3, min(10, args.cpu_samples)))
            line["cpu_baseline"] = {"value": cps, "unit": "chunks/s", "cores": cores, "kind": "port",
                                    "sample": f"{n} model evaluations (10 per chunk) of the same "
                                              f"workload by the CPU oracle in bf16; "
                                              f"{per_eval * 1e3:.1f} ms each"}
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["fam", "reference"], default="fam")
    ap.add_argument("--cpu-samples", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--euler-steps", type=int, default=NSTEPS,
                    help="Euler steps per chunk (profiling captures only; the metric is quoted at 10)")
    args = ap.parse_args()
    if args.euler_steps != NSTEPS:
        globals()["NSTEPS"] = args.euler_steps
    if args.impl == "reference":
        run_reference(args)
    else:
        run_fam(args)


if __name__ == "__main__":
    main()
