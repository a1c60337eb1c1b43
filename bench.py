#!/usr/bin/env python
"""Benchmark of the per-action-chunk denoising path on B200.

Headline workload (the one the metric's "chunks/sec at
1/2/4/8 B200" half is defined on): the batched CAE pipeline.  Per observation:
the Wan2.2-5B-shaped video backbone forward (hidden 3072, 30 blocks, 24 x 128
heads, FFN 14336, 2 views x 5 latent frames x 16 x 11 patches = 1760 tokens, 64
context tokens, t = 500), then the config-0 compact action expert (hidden 32,
4 x 8 heads, 8 blocks, FFN 128) cross-attending the backbone's final token
states over 4 Euler steps (t = 1000, 750, 500, 250), then the Action-VAE decoder
(latent 8 x 16 -> 32 x 7, hidden 256).  Each GPU runs `batch_per_gpu`
independent seeded observations per step (per-rollout noise generators, as
fastwam_batched_infer.py draws them); under torchrun the batch is sharded by
rank with no collective on the data path (weak scaling).  Weights are seeded
random-init of the reference architectures; all inputs are seeded synthetic
tensors (no dataset or checkpoint exists here).

One bench step = one batch of `batch_per_gpu` chunks on every GPU.  `value` =
chunks/s over all ranks with inputs resident in HBM (CUDA events, max over
ranks); `e2e` = the same through CAEPipeline with every step's inputs copied
from pinned host memory and the decoded chunks read back.  The working set
(10 GB of backbone weights streamed per micro-batch, 10 GB of K/V cache
written) is far larger than the 126 MB L2, so no L2 flush is needed.

At N = 1, rank 0 also measures sub-records in the same run, each with its own
roofline and CPU baseline:
  c0  BASELINE configs[0]: the CAE expert chunk + Action-VAE decode at batch 1
      (p50 latency; the north-star "well under 1 ms" target);
  c1  BASELINE configs[1]: the hidden-1024 action expert, 28 blocks, over a
      1760-token K/V cache, 10 Euler steps, batch 1 (fused kernel) and batch 8;
  c2  BASELINE configs[2]: the 30-block backbone forward (prefill) at batch 1.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl fam|reference]
  python bench.py --case NAME [--reps R]     (fixed single-GPU kernel workloads for profilers)

`--impl reference` times the reference algorithm's CPU implementation (the CPU
oracle restating FastWAM's PyTorch code) on this host's cores for the same
config, rank 0 only (see run_reference).
"""
from __future__ import annotations

import argparse
import csv
import importlib
import io
import json
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

# ---------------------------------------------------------------- workloads
VIDEO_CFG = dict(hidden_dim=3072, in_dim=48, ffn_dim=14336, out_dim=48, text_dim=4096, freq_dim=256, eps=1e-6,
                 patch_size=(1, 2, 2), num_heads=24, attn_head_dim=128, num_layers=30, has_image_input=False,
                 seperated_timestep=True, video_attention_mask_mode="first_frame_causal")
LATENT = (48, 5, 32, 44)          # 2 views side by side: 5 x 16 x 22 patches = 1760 tokens, 352 per frame
VIDEO_CTX, VIDEO_T = 64, 500.0
EXPERT_CFG = dict(hidden_dim=32, action_dim=16, ffn_dim=128, text_dim=3072, freq_dim=256, eps=1e-6,
                  num_heads=4, attn_head_dim=8, num_layers=8)
DECODER_CFG = dict(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16, decoder_hidden=256,
                   video_cond_dim=0, variational=True)
CAE_STEPS, CAE_SHIFT = 4, 1.0
BATCH_PER_GPU = 16
MICRO_BATCH = 16
C0_CTX = 512

# DRAM traffic of the headline roofline's launch (ffn.0 at the config-4 micro-batch), from one ncu
# capture of `bench.py --case gemm_ffn0_c4` (read 1,842,168,064 B + write 755,133,184 B), and its
# algorithmic bytes (A 28,160 x 3,072, weights 14,336 x 3,072, output 28,160 x 14,336 bf16, bias)
FFN0_C4_DRAM_BYTES = 1842168064 + 755133184
FFN0_C4_ALG_BYTES = 2 * (MICRO_BATCH * 1760 * 3072 + 14336 * 3072 + MICRO_BATCH * 1760 * 14336 + 14336)

C1_CFG = dict(hidden_dim=1024, action_dim=7, ffn_dim=4096, text_dim=4096, freq_dim=256, eps=1e-6,
              num_heads=16, attn_head_dim=64, num_layers=28)
C1_SA, C1_SV, C1_CTX, C1_STEPS, C1_SHIFT = 32, 1760, 64, 10, 1.0

HEADLINE_CONFIG = {
    "workload": "BASELINE configs[4]: CAE pipeline per observation = config-2 backbone forward (Wan2.2-5B "
                "shape, 30 blocks, 1760 tokens) + config-0 compact expert (hidden 32, 8 blocks, 4 Euler steps) "
                "over the backbone's final token states + Action-VAE decode (32 x 7 chunk)",
    "batch_per_gpu": BATCH_PER_GPU, "micro_batch": MICRO_BATCH, "video_tokens": 1760,
    "context_tokens": VIDEO_CTX, "euler_steps": CAE_STEPS,
    "l2": "working set per step (10 GB weights streamed per micro-batch, 10 GB K/V written) >> 126 MB L2; no flush",
}


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm": float(d["hbm_gbs"]), "tc": float(d["bf16_tflops"]),
                "tc_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm": 6650.0, "tc": 1590.0, "tc_sustained": 1400.0, "source": "fallback"}


def _dist():
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), \
        int(os.environ.get("LOCAL_RANK", "0"))


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = ""

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


# ------------------------------------------------------------ work counts
def backbone_flops(S: int, tpf: int, C: int, cfg=VIDEO_CFG) -> float:
    """Algorithmic FLOPs of one backbone forward (WanVideoDiT.prepare + every block, the
    last block's post-block included as the reference computes it) for one sample of S
    tokens (tpf per latent frame, first-frame-causal self attention) and C context tokens."""
    D, F, L, T = cfg["hidden_dim"], cfg["ffn_dim"], cfg["num_layers"], cfg["text_dim"]
    HD = cfg["num_heads"] * cfg["attn_head_dim"]
    patch = 2.0 * S * cfg["in_dim"] * 4 * D
    text = 2.0 * C * (T * D + D * D)
    time_mlp = 2.0 * 2 * (cfg["freq_dim"] * D + D * D + 6 * D * D)   # two unique timestep rows
    linear = 2.0 * S * (3 * HD * D + HD * D + HD * D + HD * D + 2 * F * D)
    ctx_kv = 2.0 * C * 2 * HD * D
    pairs = tpf * tpf + (S - tpf) * S                                   # first-frame-causal mask
    attn = 4.0 * HD * pairs + 4.0 * HD * S * C
    return patch + text + time_mlp + L * (linear + ctx_kv + attn)


def c1_work():
    """Bytes (and FLOPs) a config-1 chunk must move at least once: per model evaluation
    the weights of every block except the hoisted cross K/V projections, plus the
    head / encoder, plus the K/V cache; per chunk the hoisted context projections."""
    c = C1_CFG
    D, HD, F, L = c["hidden_dim"], c["num_heads"] * c["attn_head_dim"], c["ffn_dim"], c["num_layers"]
    per_block = (3 * HD * D + HD * D + HD * D + HD * D + F * D + D * F) * 2 + (6 * D) * 2
    per_eval = L * per_block + (2 * C1_SA * c["action_dim"] + D * c["action_dim"] * 2) * 2
    kv = L * 2 * C1_SV * HD * 2
    prologue = (c["text_dim"] * D + D * D + c["freq_dim"] * D + D * D + 6 * D * D) * 2 \
        + L * 2 * HD * D * 2 + C1_CTX * c["text_dim"] * 2
    flops = C1_STEPS * (2 * C1_SA * L * (3 * HD * D + 2 * HD * D + 2 * HD * D + 2 * F * D)
                        + 4 * C1_SA * (C1_SV + C1_SA) * HD * L + 4 * C1_SA * C1_CTX * HD * L)
    return {"bytes": prologue + C1_STEPS * (per_eval + kv), "kernel_bytes": C1_STEPS * (per_eval + kv),
            "flops": flops}


def c0_bytes() -> int:
    """Bytes a config-0 chunk must move at least once: the fp32 context (512 x 3072), the
    expert and decoder weights (fp32)."""
    M = importlib.import_module("faster-action-models_b200.models")
    exp = M.ActionDiT(**{**EXPERT_CFG})
    ae = M.ActionAE(M.ActionAEConfig(**DECODER_CFG))
    n = sum(p.numel() for p in exp.parameters()) + sum(p.numel() for p in ae.decoder.parameters())
    return C0_CTX * EXPERT_CFG["text_dim"] * 4 + n * 4


# ------------------------------------------------------------ builders
def build_c4(dev, seed: int):
    M = importlib.import_module("faster-action-models_b200.models")
    P = importlib.import_module("faster-action-models_b200.pipeline")
    torch.manual_seed(seed)
    with torch.device(dev):
        vid = M.WanVideoDiT(**VIDEO_CFG)
        exp = M.ActionDiT(**EXPERT_CFG)
        ae = M.ActionAE(M.ActionAEConfig(**DECODER_CFG))
    vid, exp = vid.to(torch.bfloat16), exp.to(torch.bfloat16)
    pipe = P.CAEPipeline(vid, exp, ae, num_steps=CAE_STEPS, shift=CAE_SHIFT, micro_batch=MICRO_BATCH)
    return vid, exp, ae, pipe


def c4_inputs(first_rollout: int, B: int):
    """Host inputs of rollouts first_rollout .. first_rollout + B - 1: seeded latents and
    context, per-rollout noise generators (fastwam_batched_infer.py:59-66)."""
    R = importlib.import_module("faster-action-models_b200.replicas")
    g = torch.Generator().manual_seed(10_000 + first_rollout)
    lat = torch.randn(B, *LATENT, generator=g).bfloat16()
    ctx = torch.randn(B, VIDEO_CTX, VIDEO_CFG["text_dim"], generator=g).bfloat16()
    cm = torch.ones(B, VIDEO_CTX, dtype=torch.bool)
    noise = R.seeded_noise(range(first_rollout, first_rollout + B), (DECODER_CFG["num_tokens"],
                                                                    DECODER_CFG["latent_dim"]))
    return lat, ctx, cm, noise


def build_c1(dev, seed: int = 0):
    M = importlib.import_module("faster-action-models_b200.models")
    torch.manual_seed(seed)
    dit = M.ActionDiT(**C1_CFG).to(torch.bfloat16).to(dev)
    g = torch.Generator(device="cpu").manual_seed(1000 + seed)
    HD = C1_CFG["num_heads"] * C1_CFG["attn_head_dim"]
    L = C1_CFG["num_layers"]
    ck = torch.randn(L, 1, C1_SV, HD, generator=g).bfloat16().to(dev)
    cv = torch.randn(L, 1, C1_SV, HD, generator=g).bfloat16().to(dev)
    ctx = torch.randn(1, C1_CTX, C1_CFG["text_dim"], generator=g).bfloat16()
    cm = torch.ones(1, C1_CTX, dtype=torch.uint8)  # bool masks passed as uint8 (True = attend)
    noise = torch.randn(1, C1_SA, C1_CFG["action_dim"], generator=g).bfloat16()
    mask = torch.ones(C1_SA, C1_SV + C1_SA, dtype=torch.uint8)
    return M, dit, ck, cv, ctx, cm, noise, mask


# ------------------------------------------------------------ timing helpers
def time_calls(fn, reps: int, warmup: int = 2):
    """Per-call device times (ms) of fn() bracketed by CUDA events on the current stream."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for s, e in ev:
        s.record()
        fn()
        e.record()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in ev]


def p50(xs):
    xs = sorted(xs)
    return xs[len(xs) // 2]


def time_fused_kernel(eng, chunk, reps=5):
    """The fused persistent chunk kernel alone: CUDA events the library records on the
    launching stream immediately around its launch (fam_action_set_kernel_events), in
    plain (not graph-replayed) chunk calls.  Returns ms per launch."""
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


def time_dominant_gemm(vid, dev, reps=10):
    """The largest backbone GEMM as the prefill launches it (ffn.0 of one block, GELU
    epilogue, CTA pairs, automatic split round) at the micro-batch's token count, timed
    alone with CUDA events on the launching stream.  Returns (ms per launch, FLOPs)."""
    ops = importlib.import_module("faster-action-models_b200.ops")
    M_ = MICRO_BATCH * 1760
    blk = vid.blocks[0]
    w = blk.ffn[0].weight.detach().contiguous()
    b = blk.ffn[0].bias.detach().contiguous()
    h = torch.randn(M_, VIDEO_CFG["hidden_dim"], device=dev).bfloat16()
    out = torch.empty(M_, w.shape[0], device=dev, dtype=torch.bfloat16)
    ms = time_calls(lambda: ops.gemm(h, w, bias=b, act="gelu_tanh", out=out, pair=True, tile_n=256,
                                     split_round="auto"), reps, warmup=3)
    return statistics.mean(ms), 2.0 * M_ * w.shape[0] * w.shape[1]


# ------------------------------------------------------------ CPU reference
def _cpu_threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_c4_sample(reps: int = 1):
    """The reference algorithm on this host's cores, on a bounded sample of one config-4
    chunk: WanVideoDiT.prepare + ONE backbone block at config-2 widths (bf16, the
    reference model dtype), and the compact expert's 4-step chunk + decode (fp32) over a
    1760 x 3072 context.  A chunk = prepare + 30 x block + expert chunk.  Returns a dict
    of seconds (medians over reps)."""
    from oracle import fam_oracle as O
    M = importlib.import_module("faster-action-models_b200.models")
    cores = _cpu_threads()
    torch.manual_seed(0)
    vid = M.WanVideoDiT(**{**VIDEO_CFG, "num_layers": 1}).to(torch.bfloat16)
    exp = M.ActionDiT(**EXPERT_CFG)
    ae = M.ActionAE(M.ActionAEConfig(**DECODER_CFG))
    sd = {k: v.detach() for k, v in vid.state_dict().items()}
    cfg = O.DiTConfig(hidden_dim=3072, ffn_dim=14336, num_heads=24, attn_head_dim=128, num_layers=1,
                      text_dim=4096, in_dim=48, out_dim=48)
    esd = {k: v.detach().float() for k, v in exp.state_dict().items()}
    dsd = {k: v.detach().float() for k, v in ae.state_dict().items()}
    ecfg = O.DiTConfig(hidden_dim=32, ffn_dim=128, num_heads=4, attn_head_dim=8, num_layers=8, text_dim=3072,
                       action_dim=16)
    dcfg = O.DecoderConfig(7, 32, 8, 16, 256)
    lat, ctx, cm, noise = c4_inputs(0, 1)
    t = torch.full((1,), VIDEO_T).bfloat16()
    prep, block, expert = [], [], []
    with torch.no_grad():
        for _ in range(reps):
            t0 = time.perf_counter()
            tok, _, tmod, cemb, cmask, freqs, _, tpf = O.video_prepare(sd, cfg, lat, t, ctx, cm)
            t1 = time.perf_counter()
            _, _, hid = O.prefill_video_cache(sd, cfg, tok, freqs, tmod, cemb, cmask,
                                              O.build_video_to_video_mask(tok.shape[1], tpf), return_hidden=True)
            t2 = time.perf_counter()
            O.cae_chunk(esd, ecfg, dsd, dcfg, noise, hid.float(), num_steps=CAE_STEPS, shift=CAE_SHIFT)
            t3 = time.perf_counter()
            prep.append(t1 - t0)
            block.append(t2 - t1)
            expert.append(t3 - t2)
    r = {"prepare": statistics.median(prep), "block": statistics.median(block),
         "expert": statistics.median(expert), "cores": cores}
    r["backbone"] = r["prepare"] + VIDEO_CFG["num_layers"] * r["block"]
    r["chunk"] = r["backbone"] + r["expert"]
    return r


def cpu_c0_ms(reps: int = 7):
    """BASELINE config 0 on the CPU as the reference runs it (fp32): 4 Euler steps of the
    standalone expert over a 512 x 3072 context + decode; p50 ms."""
    from oracle import fam_oracle as O
    M = importlib.import_module("faster-action-models_b200.models")
    cores = _cpu_threads()
    torch.manual_seed(0)
    exp = M.ActionDiT(**EXPERT_CFG)
    ae = M.ActionAE(M.ActionAEConfig(**DECODER_CFG))
    esd = {k: v.detach().float() for k, v in exp.state_dict().items()}
    dsd = {k: v.detach().float() for k, v in ae.state_dict().items()}
    ecfg = O.DiTConfig(hidden_dim=32, ffn_dim=128, num_heads=4, attn_head_dim=8, num_layers=8, text_dim=3072,
                       action_dim=16)
    g = torch.Generator().manual_seed(0)
    ctx = torch.randn(1, C0_CTX, 3072, generator=g)
    noise = torch.randn(1, 8, 16, generator=g)
    ms = []
    with torch.no_grad():
        for i in range(reps + 1):
            t0 = time.perf_counter()
            O.cae_chunk(esd, ecfg, dsd, O.DecoderConfig(7, 32, 8, 16, 256), noise, ctx, num_steps=4, shift=1.0)
            if i:
                ms.append((time.perf_counter() - t0) * 1e3)
    return p50(ms), cores, len(ms)


def cpu_c1_chunks_per_s(n: int = 5):
    """Config 1 on the CPU (bf16, like the reference model): one sample = one model
    evaluation of the chunk; chunks/s = 1 / (10 x evaluation time)."""
    from oracle import fam_oracle as O
    cores = _cpu_threads()
    M, dit, ck, cv, ctx, cm, noise, mask = build_c1("cpu")
    sd = {k: v.bfloat16() for k, v in dit.state_dict().items()}
    c = C1_CFG
    cfg = O.DiTConfig(hidden_dim=c["hidden_dim"], ffn_dim=c["ffn_dim"], num_heads=c["num_heads"],
                      attn_head_dim=c["attn_head_dim"], num_layers=c["num_layers"], text_dim=c["text_dim"],
                      action_dim=c["action_dim"])
    ts, _ = O.build_inference_schedule(C1_STEPS, C1_SHIFT, dtype=torch.bfloat16)
    times = []
    with torch.no_grad():
        for i in range(n + 1):
            t0 = time.perf_counter()
            O.denoise_action_with_video_cache(sd, cfg, noise, ts[i % C1_STEPS].reshape(1), ctx, cm.bool(),
                                              list(ck), list(cv), mask.bool())
            if i:
                times.append(time.perf_counter() - t0)
    per_eval = statistics.mean(times)
    return 1.0 / (C1_STEPS * per_eval), cores, len(times), per_eval


# ------------------------------------------------------------ sub-records (N = 1)
def sub_c0(dev, peaks):
    M = importlib.import_module("faster-action-models_b200.models")
    torch.manual_seed(0)
    with torch.device(dev):
        exp = M.ActionDiT(**EXPERT_CFG)
        ae = M.ActionAE(M.ActionAEConfig(**DECODER_CFG))
    g = torch.Generator().manual_seed(0)
    ctx = torch.randn(1, C0_CTX, 3072, generator=g).to(dev)
    noise = torch.randn(1, 8, 16, generator=g).to(dev)
    ts, ds = M.build_inference_schedule(CAE_STEPS, CAE_SHIFT, dtype=torch.float32)
    eng = exp.engine()
    with ClockSampler(dev.index or 0) as clk:
        ms = time_calls(lambda: eng.chunk_decode(noise, ts, ds, ctx, ae), 50, warmup=5)
        fused = eng.decode_fused
        ms_fused = time_calls(lambda: eng.chunk_decode(noise, ts, ds, ctx, ae, decode="fused"), 50, warmup=5)
    cpu_ms, cores, n = cpu_c0_ms()
    by = c0_bytes()
    return {"workload": "BASELINE configs[0]: CAE expert (hidden 32, 4 x 8 heads, 8 blocks) over a 512 x 3072 "
                        "context, 4 Euler steps + Action-VAE decode (hidden 256) -> 32 x 7, batch 1, fp32",
            "decode": "step-kernel epilogue" if fused else "separate launches (decode=auto)",
            "latency_p50_ms": p50(ms), "chunks_per_s": 1e3 / p50(ms), "reps": len(ms),
            "epilogue_decode_p50_ms": p50(ms_fused), "clocks": clk.summary(),
            "roofline": {"bound": "latency (HBM floor shown)", "bytes_per_chunk": by,
                         "floor_ms": by / (peaks["hbm"] * 1e9) * 1e3,
                         "achieved_gbs": by / (p50(ms) * 1e-3) / 1e9,
                         "frac": by / (p50(ms) * 1e-3) / 1e9 / peaks["hbm"], "peak": peaks["hbm"],
                         "unit": "GB/s", "peak_source": peaks["source"]},
            "cpu_baseline": {"value": cpu_ms, "unit": "ms (p50)", "cores": cores, "kind": "port",
                             "sample": f"{n} whole config-0 chunks + decode by the CPU oracle in fp32"}}


def sub_c1(dev, peaks):
    M, dit, ck, cv, ctx, cm, noise, mask = build_c1(dev)
    eng = dit.engine()
    ts, ds = M.build_inference_schedule(C1_STEPS, C1_SHIFT)
    ctx_d, cm_d, noise_d, mask_d = ctx.to(dev), cm.to(dev), noise.to(dev), mask.to(dev)
    lat = noise_d.clone()
    cks, cvs = list(ck), list(cv)

    def chunk(use_graph=True):
        lat.copy_(noise_d)
        eng.chunk(lat, ts, ds, ctx_d, cm_d, cks, cvs, mask_d, out=lat, use_graph=use_graph)

    with ClockSampler(dev.index or 0) as clk:
        ms = time_calls(chunk, 20, warmup=3)
        path = eng.last_path()
        k_ms = time_fused_kernel(eng, lambda: chunk(False)) if path == "fused" else None
    work = c1_work()
    rec = {"workload": "BASELINE configs[1]: action expert 1024h/16x64/28 blocks, 1760-token K/V cache, "
                       "64-token context, 10 Euler steps, batch 1",
           "path": path, "latency_p50_ms": p50(ms), "chunks_per_s": 1e3 / p50(ms), "clocks": clk.summary(),
           "chunk_roofline": {"bound": "hbm", "bytes_per_chunk": work["bytes"],
                              "floor_ms": work["bytes"] / (peaks["hbm"] * 1e9) * 1e3,
                              "frac": work["bytes"] / (peaks["hbm"] * 1e9) * 1e3 / p50(ms)}}
    if k_ms is not None:
        ach = work["kernel_bytes"] / (k_ms * 1e-3) / 1e9
        rec["roofline"] = {"bound": "hbm", "kernel": "fused_chunk_kernel (every step and block of the chunk, "
                                                     "1 launch)",
                           "achieved": ach, "peak": peaks["hbm"], "unit": "GB/s", "frac": ach / peaks["hbm"],
                           "traffic": None, "avg_launch_us": k_ms * 1e3, "bytes_per_launch": work["kernel_bytes"],
                           "peak_source": peaks["source"],
                           "traffic_note": "ncu replay of the cooperative 2-CTA-cluster launch fails on this "
                                           "pool; DRAM bytes not captured"}
    # batch 8 (launch chain: per-step weights shared by 8 samples)
    B = 8
    g = torch.Generator().manual_seed(8)
    HD = C1_CFG["num_heads"] * C1_CFG["attn_head_dim"]
    ck8 = [torch.randn(B, C1_SV, HD, generator=g).bfloat16().to(dev) for _ in range(C1_CFG["num_layers"])]
    cv8 = [torch.randn(B, C1_SV, HD, generator=g).bfloat16().to(dev) for _ in range(C1_CFG["num_layers"])]
    ctx8 = torch.randn(B, C1_CTX, C1_CFG["text_dim"], generator=g).bfloat16().to(dev)
    cm8 = torch.ones(B, C1_CTX, dtype=torch.uint8, device=dev)
    n8 = torch.randn(B, C1_SA, C1_CFG["action_dim"], generator=g).bfloat16().to(dev)
    lat8 = n8.clone()

    def chunk8():
        lat8.copy_(n8)
        eng.chunk(lat8, ts, ds, ctx8, cm8, ck8, cv8, mask_d, out=lat8)

    with ClockSampler(dev.index or 0) as clk8:
        ms8 = time_calls(chunk8, 10, warmup=3)
    rec["batch8"] = {"path": eng.last_path(), "latency_p50_ms": p50(ms8), "chunks_per_s": B * 1e3 / p50(ms8),
                     "clocks": clk8.summary()}
    del ck8, cv8
    # batch 64 (BASELINE config 1's largest batch): inputs made on the device (12.9 GB of K/V)
    B = 64
    gd = torch.Generator(device=dev).manual_seed(64)
    ck64 = [torch.randn(B, C1_SV, HD, device=dev, generator=gd).bfloat16() for _ in range(C1_CFG["num_layers"])]
    cv64 = [torch.randn(B, C1_SV, HD, device=dev, generator=gd).bfloat16() for _ in range(C1_CFG["num_layers"])]
    ctx64 = torch.randn(B, C1_CTX, C1_CFG["text_dim"], device=dev, generator=gd).bfloat16()
    cm64 = torch.ones(B, C1_CTX, dtype=torch.uint8, device=dev)
    n64 = torch.randn(B, C1_SA, C1_CFG["action_dim"], device=dev, generator=gd).bfloat16()
    lat64 = n64.clone()

    def chunk64():
        lat64.copy_(n64)
        eng.chunk(lat64, ts, ds, ctx64, cm64, ck64, cv64, mask_d, out=lat64)

    with ClockSampler(dev.index or 0) as clk64:
        ms64 = time_calls(chunk64, 5, warmup=3)
    rec["batch64"] = {"path": eng.last_path(), "latency_p50_ms": p50(ms64), "chunks_per_s": B * 1e3 / p50(ms64),
                      "clocks": clk64.summary()}
    del ck64, cv64
    cps, cores, n, per_eval = cpu_c1_chunks_per_s()
    rec["cpu_baseline"] = {"value": cps, "unit": "chunks/s", "cores": cores, "kind": "port",
                           "sample": f"{n} model evaluations (10 per chunk) by the CPU oracle in bf16; "
                                     f"{per_eval * 1e3:.1f} ms each"}
    return rec


def sub_c2(vid, dev, peaks, cpu):
    lat, ctx, cm, _ = c4_inputs(0, 1)
    lat, ctx, cm = lat.to(dev), ctx.to(dev), cm.to(dev)
    t = torch.full((1,), VIDEO_T).bfloat16()
    eng = vid.engine()
    with ClockSampler(dev.index or 0) as clk:
        ms = time_calls(lambda: eng.prefill(lat, t, ctx, cm), 10, warmup=3)
    fl = backbone_flops(1760, 352, VIDEO_CTX)
    ach = fl / (p50(ms) * 1e-3) / 1e12
    return {"workload": "BASELINE configs[2]: Wan2.2-5B-shaped backbone forward (30 blocks, 1760 tokens, 64 "
                        "context tokens), per-layer K/V cache out, batch 1",
            "latency_p50_ms": p50(ms), "clocks": clk.summary(),
            "roofline": {"bound": "tensor", "flops": fl, "achieved": ach, "peak": peaks["tc_sustained"],
                         "unit": "TFLOP/s", "frac": ach / peaks["tc_sustained"],
                         "frac_of_burst": ach / peaks["tc"], "peak_source": peaks["source"]},
            "cpu_baseline": {"value": cpu["backbone"] * 1e3, "unit": "ms", "cores": cpu["cores"], "kind": "port",
                             "sample": "WanVideoDiT.prepare + one block by the CPU oracle in bf16, extrapolated "
                                       f"to 30 blocks ({cpu['prepare'] * 1e3:.0f} ms + 30 x "
                                       f"{cpu['block'] * 1e3:.0f} ms)"}}


# ------------------------------------------------------------ arms
def run_reference(args):
    """The reference algorithm on this host's CPU cores for the headline config: each
    step is a bounded sample of one chunk (prepare + one of the 30 backbone blocks + the
    expert chunk and decode) extrapolated to the whole chunk.  Rank 0 only."""
    ws, rank, _ = _dist()
    if rank != 0:
        return
    cpu_c4_sample(1)  # warm-up (allocator, threads)
    samples = []
    for i in range(max(1, args.warmup) + args.steps):
        r = cpu_c4_sample(1)
        if i >= max(1, args.warmup):
            samples.append(r)
    chunk_s = statistics.median(s["chunk"] for s in samples)
    cps = 1.0 / chunk_s
    med = {k: statistics.median(s[k] for s in samples) for k in ("prepare", "block", "expert")}
    sample = (f"{len(samples)} steps, each WanVideoDiT.prepare + one backbone block (bf16) + the compact "
              f"expert's 4-step chunk and decode (fp32) of one observation by the CPU oracle; chunk = prepare "
              f"{med['prepare'] * 1e3:.0f} ms + 30 x block {med['block'] * 1e3:.0f} ms + expert "
              f"{med['expert'] * 1e3:.0f} ms")
    line = {"metric": METRIC, "impl": "reference", "value": cps, "unit": "chunks/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": chunk_s * 1e3,
            "latency_p50_ms": chunk_s * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded), random-init weights",
            "config": dict(HEADLINE_CONFIG, parallelism=f"batch-sharded replicas x{args.gpus}"),
            "cpu_baseline": {"value": cps, "unit": "chunks/s", "cores": samples[0]["cores"], "kind": "port",
                             "sample": sample},
            "e2e": {"value": cps, "unit": "chunks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_fam(args):
    ws, rank, local = _dist()
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks = _peaks()
    B = BATCH_PER_GPU
    vid, exp, ae, pipe = build_c4(dev, seed=0)
    lat_h, ctx_h, cm_h, noise_h = c4_inputs(rank * B, B)
    lat, ctx, cm, noise = lat_h.to(dev), ctx_h.to(dev), cm_h.to(dev), noise_h.to(dev)

    def step():
        return pipe(lat, VIDEO_T, ctx, cm, noise)

    for _ in range(max(3, args.warmup)):
        out = step()
    torch.cuda.synchronize()
    assert out.shape == (B, 32, 7) and bool(torch.isfinite(out).all())
    # per micro-batch: the backbone's launches, the CAE context (2) and step (1) launches, and
    # the decoder's input, 3 per upsampling stage and output launches unless it ran fused
    dec_launches = 0 if exp.engine().decode_fused else 2 + 3 * len(ae.decoder.strides)
    launches = (vid.engine().launch_count() + 3 + dec_launches) * ((B + MICRO_BATCH - 1) // MICRO_BATCH)
    K = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("timed_steps")
        t0.record()
        for s, e in ev:
            s.record()
            step()
            e.record()
        t1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    tm = torch.tensor([t0.elapsed_time(t1), p50([s.elapsed_time(e) for s, e in ev])], device=dev)
    if ws > 1:
        torch.distributed.all_reduce(tm, op=torch.distributed.ReduceOp.MAX)
    elapsed_ms, step_p50 = tm.tolist()

    # ---- end to end: pinned host inputs -> device, pipeline, decoded chunks -> host, every step
    lat_p, ctx_p, cm_p, noise_p = (x.pin_memory() for x in (lat_h, ctx_h, cm_h.to(torch.uint8), noise_h))
    cm_u8 = torch.empty(B, VIDEO_CTX, dtype=torch.uint8, device=dev)
    out_h = torch.empty(B, 32, 7, dtype=torch.float32).pin_memory()

    def step_e2e():
        lat.copy_(lat_p, non_blocking=True)
        ctx.copy_(ctx_p, non_blocking=True)
        cm_u8.copy_(cm_p, non_blocking=True)
        noise.copy_(noise_p, non_blocking=True)
        o = pipe(lat, VIDEO_T, ctx, cm_u8, noise)
        out_h.copy_(o, non_blocking=True)

    for _ in range(2):
        step_e2e()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(K):
        step_e2e()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if ws > 1:
        torch.distributed.all_reduce(e2e_ms, op=torch.distributed.ReduceOp.MAX)
    e2e_ms = e2e_ms.item()
    h2d = sum(x.numel() * x.element_size() for x in (lat_p, ctx_p, cm_p, noise_p))
    d2h = out_h.numel() * 4

    g_ms, g_flops = time_dominant_gemm(vid, dev)
    if rank == 0:
        step_ms = elapsed_ms / K
        flops_chunk = backbone_flops(1760, 352, VIDEO_CTX)
        pipe_tf = flops_chunk * B / (step_ms * 1e-3) / 1e12
        g_tf = g_flops / (g_ms * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": ws * B * K / (elapsed_ms / 1e3), "unit": "chunks/s", "n_gpus": ws,
            "steps": K, "warmup": max(3, args.warmup), "ms_per_step": step_ms, "latency_p50_ms": step_p50,
            "latency_note": "p50 of one step = batch_per_gpu chunks; batch-1 chunk latencies are in sub_records",
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) latents, context and per-rollout noise), random-init weights",
            "config": dict(HEADLINE_CONFIG, parallelism=f"batch-sharded replicas x{ws}"),
            "roofline": {"bound": "tensor",
                         "kernel": f"backbone ffn.0 GEMM ({MICRO_BATCH * 1760} x 14336 x 3072, GELU epilogue, "
                                   "tcgen05 CTA pairs) as the prefill launches it, timed alone",
                         "achieved": g_tf, "peak": peaks["tc"], "unit": "TFLOP/s", "frac": g_tf / peaks["tc"],
                         "traffic": FFN0_C4_DRAM_BYTES, "algorithmic_bytes": FFN0_C4_ALG_BYTES,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of this launch "
                                           "(bench.py --case gemm_ffn0_c4, one capture)",
                         "avg_launch_us": g_ms * 1e3, "flops_per_launch": g_flops, "peak_source": peaks["source"]},
            "pipeline_roofline": {"bound": "tensor", "flops_per_chunk": flops_chunk, "achieved": pipe_tf,
                                  "peak": peaks["tc_sustained"], "unit": "TFLOP/s",
                                  "frac": pipe_tf / peaks["tc_sustained"],
                                  "floor_chunks_per_s_per_gpu": peaks["tc_sustained"] * 1e12 / flops_chunk},
            "e2e": {"value": ws * B * K / (e2e_ms / 1e3), "unit": "chunks/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "note": "per step the latents, context, mask and noise go H2D and the decoded chunks D2H"},
            "gpu_launches": launches * K,
            "clocks": clk.summary(),
        }
        if ws == 1 and not args.no_sub_records:
            cpu = cpu_c4_sample(2)
            line["cpu_baseline"] = {
                "value": 1.0 / cpu["chunk"], "unit": "chunks/s", "cores": cpu["cores"], "kind": "port",
                "sample": f"one observation: WanVideoDiT.prepare + one backbone block (bf16) + the compact "
                          f"expert chunk and decode (fp32) by the CPU oracle, extrapolated to 30 blocks "
                          f"({cpu['chunk']:.1f} s per chunk)"}
            line["sub_records"] = {"c0": sub_c0(dev, peaks), "c1": sub_c1(dev, peaks),
                                   "c2": sub_c2(vid, dev, peaks, cpu)}
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------ profiler cases
def run_case(case: str, reps: int) -> None:
    """Fixed single-GPU workloads of the library's kernels, for profilers: each runs its
    library call `reps` times on cuda:0 and synchronizes (under ncu, skip the warm-up
    launches with -s).
      gemm_ffn0_c4      the headline roofline's kernel: backbone ffn.0 at the config-4 micro-batch
                        ([28160, 3072] x [14336, 3072]^T, GELU, CTA pairs, automatic split round)
      gemm_qkv_c2       ops.gemm [1760, 3072] x [9216, 3072]^T + bias (backbone qkv)
      gemm_qkv_pair_c2  the same on CTA pairs, as the prefill runs it
      attn_c2           ops.attention: 1760 tokens, 24 x 128 heads, first-frame-causal (352)
      xattn_c2          the backbone's cross attention: 1760 queries over 64 context keys
      cae_c0            config 0: compact expert chunk with the Action-VAE decode in its epilogue
      fused_c1          config 1: the fused chunk kernel (plain launches), `--euler-steps`
      chain_c1_b8       config 1 at batch 8: the launch chain (plain launches), the last
                        repetition inside the NVTX range "chain_c1_b8"
      prefill_c2        config 2: the 30-block backbone prefill, batch 1
      vae_c1            VideoVAE38 encode of one 512 x 704 observation frame (p50 printed)
    """
    ops = importlib.import_module("faster-action-models_b200.ops")
    M = importlib.import_module("faster-action-models_b200.models")
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    if case == "gemm_ffn0_c4":
        M_ = MICRO_BATCH * 1760
        h = torch.randn(M_, 3072, device=dev).bfloat16()
        w = (torch.randn(14336, 3072, device=dev) * 0.02).bfloat16()
        b = torch.randn(14336, device=dev).bfloat16()
        out = torch.empty(M_, 14336, device=dev, dtype=torch.bfloat16)
        for _ in range(reps):
            ops.gemm(h, w, bias=b, act="gelu_tanh", out=out, pair=True, tile_n=256, split_round="auto")
    elif case in ("gemm_qkv_c2", "gemm_qkv_pair_c2"):
        a = torch.randn(1760, 3072, device=dev).bfloat16()
        w = (torch.randn(9216, 3072, device=dev) * 0.02).bfloat16()
        b = torch.randn(9216, device=dev).bfloat16()
        for _ in range(reps):
            if case == "gemm_qkv_c2":
                ops.gemm(a, w, bias=b)
            else:
                ops.gemm(a, w, bias=b, pair=True, tile_n=256)
    elif case == "attn_c2":
        q, k, v = (torch.randn(1, 1760, 24 * 128, device=dev).bfloat16() for _ in range(3))
        for _ in range(reps):
            ops.attention(q, k, v, 24, first_frame_tokens=352)
    elif case == "xattn_c2":
        q = torch.randn(1, 1760, 3072, device=dev).bfloat16()
        kv = torch.randn(1, 64, 6144, device=dev).bfloat16()
        km = torch.ones(1, 64, dtype=torch.uint8, device=dev)
        out = torch.empty_like(q)
        for _ in range(reps):
            ops.attention(q, kv[:, :, :3072], kv[:, :, 3072:], 24, key_mask=km, kv_splits=1, out=out)
    elif case == "cae_c0":
        with torch.device(dev):
            exp = M.ActionDiT(**EXPERT_CFG)
            ae = M.ActionAE(M.ActionAEConfig(**DECODER_CFG))
        ctx = torch.randn(1, C0_CTX, 3072, device=dev)
        noise = torch.randn(1, 8, 16, device=dev)
        ts, ds = M.build_inference_schedule(CAE_STEPS, CAE_SHIFT, dtype=torch.float32)
        eng = exp.engine()
        for _ in range(reps):
            eng.chunk_decode(noise, ts, ds, ctx, ae, decode="fused")
    elif case == "fused_c1":
        M_, dit, ck, cv, ctx, cm, noise, mask = build_c1(dev)
        eng = dit.engine()
        ts, ds = M.build_inference_schedule(C1_STEPS, C1_SHIFT)
        lat = noise.to(dev).clone()
        for _ in range(reps):
            eng.chunk(lat, ts, ds, ctx.to(dev), cm.to(dev), list(ck), list(cv), mask.to(dev), use_graph=False)
    elif case == "chain_c1_b8":
        M_, dit, ck, cv, ctx, cm, noise, mask = build_c1(dev)
        eng = dit.engine()
        ts, ds = M.build_inference_schedule(C1_STEPS, C1_SHIFT)
        B = 8
        g = torch.Generator().manual_seed(8)
        HD = C1_CFG["num_heads"] * C1_CFG["attn_head_dim"]
        ck8 = [torch.randn(B, C1_SV, HD, generator=g).bfloat16().to(dev) for _ in range(C1_CFG["num_layers"])]
        cv8 = [torch.randn(B, C1_SV, HD, generator=g).bfloat16().to(dev) for _ in range(C1_CFG["num_layers"])]
        ctx8 = torch.randn(B, C1_CTX, C1_CFG["text_dim"], generator=g).bfloat16().to(dev)
        cm8 = torch.ones(B, C1_CTX, dtype=torch.uint8, device=dev)
        n8 = torch.randn(B, C1_SA, C1_CFG["action_dim"], generator=g).bfloat16().to(dev)
        lat8 = n8.clone()
        for r in range(reps):
            if r == reps - 1:
                torch.cuda.synchronize()
                torch.cuda.nvtx.range_push("chain_c1_b8")
            lat8.copy_(n8)
            eng.chunk(lat8, ts, ds, ctx8, cm8, ck8, cv8, mask.to(dev), out=lat8, use_graph=False)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    elif case == "prefill_c2":
        with torch.device(dev):
            vid = M.WanVideoDiT(**VIDEO_CFG)
        vid = vid.to(torch.bfloat16)
        lat, ctx, cm, _ = c4_inputs(0, 1)
        t = torch.full((1,), VIDEO_T).bfloat16()
        for _ in range(reps):
            vid.prefill(lat.to(dev), t, ctx.to(dev), cm.to(dev))
    elif case == "vae_c1":
        VAE = importlib.import_module("faster-action-models_b200.vae")
        g = torch.Generator().manual_seed(0)
        sd = {}
        for name, shape in VAE.encoder_param_shapes(160, 48).items():
            if name.endswith("gamma"):
                sd[name] = (1.0 + 0.1 * torch.randn(shape, generator=g)).bfloat16()
            elif name.endswith("bias"):
                sd[name] = (0.05 * torch.randn(shape, generator=g)).bfloat16()
            else:
                fan_in = 1
                for d in shape[1:]:
                    fan_in *= d
                sd[name] = (torch.randn(shape, generator=g) / fan_in ** 0.5).bfloat16()
        vae = VAE.WanVideoVAE38(sd, torch.zeros(48), torch.ones(48), z_dim=48, dim=160)
        img = (torch.rand(1, 3, 1, 512, 704, generator=g) * 2 - 1).bfloat16().to(dev)
        print("vae_c1 encode ms p50", round(p50(time_calls(lambda: vae.model.encode(img, vae.scale), reps)), 3))
    else:
        raise SystemExit(f"unknown case {case!r}")
    torch.cuda.synchronize()
    print("ok", case)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["fam", "reference"], default="fam")
    ap.add_argument("--no-sub-records", action="store_true",
                    help="headline only (skip the N = 1 sub-records and CPU baselines)")
    ap.add_argument("--case", default=None, help="run one profiler workload and exit")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--euler-steps", type=int, default=C1_STEPS,
                    help="Euler steps of the fused_c1 case (profiling captures only)")
    args = ap.parse_args()
    if args.case is not None:
        globals()["C1_STEPS"] = args.euler_steps
        run_case(args.case, args.reps)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_fam(args)


if __name__ == "__main__":
    main()
