"""Fixed single-GPU workloads of the library's kernels, for profilers.

    python faster-action-models_b200/kernel_cases.py {gemm_qkv_c2,gemm_qkv_pair_c2,attn_c2,cae_c0,prefill_c2,dit4dit_c3,joint_c2,vae_c1} [repeats]

Each case runs its library call `repeats` times (default 3) on cuda:0 and
synchronizes; under ncu, skip the warm-up launches with `-s`.
  gemm_qkv_c2  ops.gemm: [1760, 3072] x [9216, 3072]^T + bias (backbone qkv, config 2)
  gemm_qkv_pair_c2  the same on CTA pairs (ops.gemm(pair=True, tile_n=256)), as the prefill runs it
  attn_c2      ops.attention: 1760 tokens, 24 heads x 128, first-frame-causal (352)
  cae_c0       CAEEngine.chunk + ActionAE.decode of BASELINE config 0
  prefill_c2   WanVideoDiT.prefill of BASELINE config 2 (30 blocks, 1,760 tokens, batch 1)
  dit4dit_c3   DiT4DiTPipeline of BASELINE config 3 (backbone to block 18 of 28 at 3,520
               tokens + 16-block action head, 4 Euler steps, batch 1); prints the
               p50 chunk latency over the repeats
  joint_c2     FastWAMJointPolicy.joint_step at config-2 scale: the 30-layer backbone over
               1,760 noisy video tokens + its output head, and a 30-layer action expert
               (hidden 1024, 24 x 128 heads) over that step's K/V; prints the p50 latency
  vae_c1       WanVideoVAE38 encode of one 512 x 704 observation frame (dim 160, z 48,
               the configs-1/2 latent grid 32 x 44); prints the p50 latency
  xattn_c2     ops.attention as the backbone's cross attention: 1,760 query tokens, 24 heads
               x 128, over 64 context tokens with a key mask (K and V halves of one
               [64, 6144] row)
  cae_c4       CAEPipeline of BASELINE config 4 on one GPU: the config-2 backbone (final
               token states), the config-0 compact expert (4 Euler steps, text_dim 3072)
               and the Action-VAE decode, for B = 1, 16, 128 independent observations in
               micro-batches of 16; prints chunks/s per B (p50 over the repeats)
"""
import importlib
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
ops = importlib.import_module("faster-action-models_b200.ops")
M = importlib.import_module("faster-action-models_b200.models")
P = importlib.import_module("faster-action-models_b200.pipeline")
VAE = importlib.import_module("faster-action-models_b200.vae")


def main(case: str, reps: int) -> None:
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    if case == "gemm_qkv_c2":
        a = torch.randn(1760, 3072, device=dev).bfloat16()
        w = (torch.randn(9216, 3072, device=dev) * 0.02).bfloat16()
        b = torch.randn(9216, device=dev).bfloat16()
        for _ in range(reps):
            ops.gemm(a, w, bias=b)
    elif case == "gemm_qkv_pair_c2":
        a = torch.randn(1760, 3072, device=dev).bfloat16()
        w = (torch.randn(9216, 3072, device=dev) * 0.02).bfloat16()
        b = torch.randn(9216, device=dev).bfloat16()
        for _ in range(reps):
            ops.gemm(a, w, bias=b, pair=True, tile_n=256)
    elif case == "attn_c2":
        q, k, v = (torch.randn(1, 1760, 24 * 128, device=dev).bfloat16() for _ in range(3))
        for _ in range(reps):
            ops.attention(q, k, v, 24, first_frame_tokens=352)
    elif case == "cae_c0":
        dit = M.ActionDiT(hidden_dim=32, action_dim=16, ffn_dim=128, text_dim=3072, freq_dim=256, eps=1e-6,
                          num_heads=4, attn_head_dim=8, num_layers=8).to(dev)
        ae = M.ActionAE(M.ActionAEConfig(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16,
                                         decoder_hidden=256, video_cond_dim=0, variational=True)).to(dev)
        ctx = torch.randn(1, 512, 3072, device=dev)
        noise = torch.randn(1, 8, 16, device=dev)
        ts, ds = M.build_inference_schedule(4, 1.0, dtype=torch.float32)
        eng = dit.engine()
        for _ in range(reps):
            ae.decode(eng.chunk(noise, ts, ds, ctx))
    elif case == "prefill_c2":
        with torch.device(dev):
            vid = M.WanVideoDiT(hidden_dim=3072, in_dim=48, ffn_dim=14336, out_dim=48, text_dim=4096, freq_dim=256,
                                eps=1e-6, patch_size=(1, 2, 2), num_heads=24, attn_head_dim=128, num_layers=30,
                                has_image_input=False, seperated_timestep=True,
                                video_attention_mask_mode="first_frame_causal")
        vid = vid.to(torch.bfloat16)
        lat = torch.randn(1, 48, 5, 32, 44, device=dev).bfloat16()
        ctx = torch.randn(1, 64, 4096, device=dev).bfloat16()
        cm = torch.ones(1, 64, dtype=torch.bool, device=dev)
        t = torch.full((1,), 500.0).bfloat16()
        for _ in range(reps):
            vid.prefill(lat, t, ctx, cm)
    elif case == "dit4dit_c3":
        with torch.device(dev):
            vid = M.WanVideoDiT(hidden_dim=2048, in_dim=48, ffn_dim=8192, out_dim=48, text_dim=4096, freq_dim=256,
                                eps=1e-6, patch_size=(1, 2, 2), num_heads=16, attn_head_dim=128, num_layers=28,
                                has_image_input=False, seperated_timestep=True,
                                video_attention_mask_mode="first_frame_causal")
            head = M.ActionDiT(1024, 29, 4096, 2048, 256, 1e-6, 16, 64, 16)
        vid, head = vid.to(torch.bfloat16), head.to(torch.bfloat16)
        pipe = P.DiT4DiTPipeline(vid, head, extract_layer=17, num_steps=4, shift=1.0, micro_batch=1)
        g = torch.Generator().manual_seed(0)
        lat = torch.randn(1, 48, 4, 44, 80, generator=g).bfloat16().to(dev)
        ctx = torch.randn(1, 64, 4096, generator=g).bfloat16().to(dev)
        noise = torch.randn(1, 16, 29, generator=g).to(dev)
        t = torch.full((1,), 500.0).bfloat16()
        times = []
        for _ in range(reps + 2):
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            pipe(lat, t, ctx, None, noise)
            e0.record()
            torch.cuda.synchronize()
            times.append(s0.elapsed_time(e0))
        times = sorted(times[2:])
        print("dit4dit_c3 chunk ms p50", round(times[len(times) // 2], 3))
    elif case == "joint_c2":
        with torch.device(dev):
            vid = M.WanVideoDiT(hidden_dim=3072, in_dim=48, ffn_dim=14336, out_dim=48, text_dim=4096, freq_dim=256,
                                eps=1e-6, patch_size=(1, 2, 2), num_heads=24, attn_head_dim=128, num_layers=30,
                                has_image_input=False, seperated_timestep=True,
                                video_attention_mask_mode="first_frame_causal")
            act = M.ActionDiT(1024, 7, 4096, 4096, 256, 1e-6, 24, 128, 30)
        vid, act = vid.to(torch.bfloat16), act.to(torch.bfloat16)
        pol = P.FastWAMJointPolicy(vid, act)
        g = torch.Generator().manual_seed(0)
        lat_v = torch.randn(1, 48, 5, 32, 44, generator=g).bfloat16().to(dev)
        lat_a = torch.randn(1, 32, 7, generator=g).bfloat16().to(dev)
        ctx = torch.randn(1, 64, 4096, generator=g).bfloat16().to(dev)
        cm = torch.ones(1, 64, dtype=torch.bool, device=dev)
        times = []
        for _ in range(reps + 2):
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            pol.joint_step(lat_v, lat_a, torch.tensor([700.0]), torch.tensor([700.0]), ctx, cm)
            e0.record()
            torch.cuda.synchronize()
            times.append(s0.elapsed_time(e0))
        times = sorted(times[2:])
        print("joint_c2 step ms p50", round(times[len(times) // 2], 3))
    elif case == "vae_c1":
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
        times = []
        for _ in range(reps + 2):
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            vae.model.encode(img, vae.scale)
            e0.record()
            torch.cuda.synchronize()
            times.append(s0.elapsed_time(e0))
        times = sorted(times[2:])
        print("vae_c1 encode ms p50", round(times[len(times) // 2], 3))
    elif case == "xattn_c2":
        q = torch.randn(1, 1760, 3072, device=dev).bfloat16()
        kv = torch.randn(1, 64, 6144, device=dev).bfloat16()
        km = torch.ones(1, 64, dtype=torch.uint8, device=dev)
        out = torch.empty_like(q)
        for _ in range(reps):
            ops.attention(q, kv[:, :, :3072], kv[:, :, 3072:], 24, key_mask=km, kv_splits=1, out=out)
    elif case == "cae_c4":
        torch.manual_seed(0)
        with torch.device(dev):
            vid = M.WanVideoDiT(hidden_dim=3072, in_dim=48, ffn_dim=14336, out_dim=48, text_dim=4096, freq_dim=256,
                                eps=1e-6, patch_size=(1, 2, 2), num_heads=24, attn_head_dim=128, num_layers=30,
                                has_image_input=False, seperated_timestep=True,
                                video_attention_mask_mode="first_frame_causal")
            dit = M.ActionDiT(hidden_dim=32, action_dim=16, ffn_dim=128, text_dim=3072, freq_dim=256, eps=1e-6,
                              num_heads=4, attn_head_dim=8, num_layers=8)
            ae = M.ActionAE(M.ActionAEConfig(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16,
                                             decoder_hidden=256, video_cond_dim=0, variational=True))
        pipe = P.CAEPipeline(vid.to(torch.bfloat16), dit.to(torch.bfloat16), ae, num_steps=4, shift=1.0,
                             micro_batch=16)
        g = torch.Generator().manual_seed(0)
        for B in (1, 16, 128):
            lat = torch.randn(B, 48, 5, 32, 44, generator=g).bfloat16().to(dev)
            ctx = torch.randn(B, 64, 4096, generator=g).bfloat16().to(dev)
            cm = torch.ones(B, 64, dtype=torch.bool, device=dev)
            noise = torch.randn(B, 8, 16, generator=g).to(dev)
            pipe(lat, 500.0, ctx, cm, noise)
            torch.cuda.synchronize()
            ms = []
            for _ in range(reps):
                s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record()
                out = pipe(lat, 500.0, ctx, cm, noise)
                s1.record()
                torch.cuda.synchronize()
                ms.append(s0.elapsed_time(s1))
            assert out.shape == (B, 32, 7) and bool(torch.isfinite(out).all())
            p50 = sorted(ms)[len(ms) // 2]
            print(f"cae_c4 B={B} p50 {p50:.2f} ms  {B / (p50 * 1e-3):.1f} chunks/s")
            del lat, ctx, cm, noise
    else:
        raise SystemExit(f"unknown case {case!r}")
    torch.cuda.synchronize()
    print("ok", case)


if __name__ == "__main__":
    main(sys.argv[1], int(sys.argv[2]) if len(sys.argv) > 2 else 3)
