"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/faster-action-models

It imports the reference's own FastWAM modules (FastWAM/src/fastwam/...),
builds small seeded random-init models with the reference constructors, runs
the reference code paths of the hot path on the CPU and saves
{config, state dicts, inputs, outputs} as ``*.pt`` files beside this script.
The reference cannot travel to the GPU machines, so these fixtures are the
reference's voice in the test suite there.

Reference code paths exercised:
  c0  ActionDiT.forward Euler loop + ActionAE.decode          (fp32)
        FastWAM/src/fastwam/models/wan22/action_dit.py:333-362
        FastWAM/src/fastwam/models/action_ae.py:154-187
  c1  FastWAM._denoise_action_with_video_cache + scheduler     (bf16)
        FastWAM/src/fastwam/models/wan22/fastwam.py:771-804, 1241-1263
        FastWAM/src/fastwam/models/wan22/mot.py:528-578
  c2  WanVideoDiT.prepare + MoT.prefill_video_cache_tensor     (bf16)
        FastWAM/src/fastwam/models/wan22/wan_video_dit.py:640-720
        FastWAM/src/fastwam/models/wan22/mot.py:474-526
      plus the final hidden state through DiTBlock.forward (wan_video_dit.py:248-267)
  sched / masks / rope / sinusoid: scheduler_continuous.py:63-88, fastwam.py:429-451,
        wan_video_dit.py:30-60, 489-523
  joint FastWAM._joint_denoise_core: both experts, MoT joint attention   (bf16)
        FastWAM/src/fastwam/models/wan22/fastwam.py:492-554, mot.py:580-708
  idm   FastWAMIDM._denoise_video (one video-only step) and FastWAMJoint's mask (bf16)
        FastWAM/src/fastwam/models/wan22/fastwam_idm.py:283-313, fastwam_joint.py:29-49
  vae VideoVAE38_.encode of one observation frame (fp32 and bf16)
        FastWAM/src/fastwam/models/wan22/wan_video_vae.py:1285-1304, 619-733
  fastwam_infer_action  FastWAM.infer_action end to end (VAE encode, proprio token, prefill,
        action Euler loop, Action-VAE decode) and its checkpoint payload, small shapes, bf16
        FastWAM/src/fastwam/models/wan22/fastwam.py:257-306, 1080-1274, 1300-1345
  dit4dit_action_vae  DiT4DiT's ActionVAE.decode (task-conditioned, crop, two stages) and
        the latent un-normalisation of DiT4DiT._decode_action_predictions           (fp32)
        DiT4DiT/DiT4DiT/model/modules/action_model/action_vae.py:136-197, 276-283
        DiT4DiT/DiT4DiT/model/framework/DiT4DiT.py:393-410
"""
from __future__ import annotations

import argparse
import sys
import types
from pathlib import Path
from types import SimpleNamespace

import torch

OUT = Path(__file__).resolve().parent


def _import_reference(ref_root: Path):
    src = ref_root / "FastWAM" / "src"
    if not src.exists():
        raise SystemExit(f"reference sources not found under {src}")
    # fastwam.utils imports imageio for video I/O, which this path never uses.
    for name in ("imageio", "imageio.v3"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.path.insert(0, str(src))
    from fastwam.models.wan22.action_dit import ActionDiT
    from fastwam.models.wan22.wan_video_dit import (WanVideoDiT, sinusoidal_embedding_1d,
                                                    precompute_freqs_cis, precompute_freqs_cis_3d,
                                                    rope_apply)
    from fastwam.models.wan22.mot import MoT
    from fastwam.models.wan22.fastwam import FastWAM
    from fastwam.models.wan22.schedulers.scheduler_continuous import \
        WanContinuousFlowMatchScheduler
    from fastwam.models.action_ae import ActionAE, ActionAEConfig
    from fastwam.models.wan22.wan_video_vae import VideoVAE38_
    from fastwam.models.wan22.fastwam_idm import FastWAMIDM
    from fastwam.models.wan22.fastwam_joint import FastWAMJoint
    return SimpleNamespace(**locals())


def _round_params_bf16(module):
    """Round every parameter to bf16-representable values (keeps fixtures small
    and lets an fp32 model and a bf16 kernel see identical weights)."""
    with torch.no_grad():
        for p in module.parameters():
            p.copy_(p.to(torch.bfloat16).to(p.dtype))


def _sd(module, dtype):
    return {k: v.detach().to(dtype).clone() for k, v in module.state_dict().items()}


def make_c0(R):
    """Standalone CAE-style expert + Action-VAE decoder, fp32 (config 0 shape family)."""
    torch.manual_seed(0)
    cfg = dict(hidden_dim=32, action_dim=16, ffn_dim=128, text_dim=96, freq_dim=256, eps=1e-6,
               num_heads=4, attn_head_dim=8, num_layers=3)
    dit = R.ActionDiT(**cfg).eval()
    ae_cfg = R.ActionAEConfig(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16,
                              decoder_hidden=32, video_cond_dim=0, variational=True)
    ae = R.ActionAE(ae_cfg).eval()
    _round_params_bf16(dit)
    _round_params_bf16(ae)
    g = torch.Generator().manual_seed(0)
    ctx = torch.randn(1, 24, 96, generator=g).bfloat16().float()
    noise = torch.randn(1, 8, 16, generator=g)
    sched = R.WanContinuousFlowMatchScheduler(shift=5.0)
    ts, ds = sched.build_inference_schedule(4, device="cpu", dtype=torch.float32, shift_override=1.0)
    x = noise.clone()
    vs = []
    with torch.no_grad():
        for t, d in zip(ts, ds):
            v = dit(x, t.unsqueeze(0), ctx)
            vs.append(v.clone())
            x = sched.step(v, d, x)
        chunk = ae.decode(x)
    return {
        "kind": "c0", "dit_cfg": cfg, "dec_cfg": dict(action_dim=7, action_horizon=32, num_tokens=8,
                                                      latent_dim=16, decoder_hidden=32),
        "num_steps": 4, "shift": 1.0,
        "dit": _sd(dit, torch.bfloat16), "ae": _sd(ae, torch.bfloat16),
        "context": ctx.bfloat16(), "noise": noise,
        "timesteps": ts, "deltas": ds, "velocities": torch.stack(vs), "latent": x, "chunk": chunk,
    }


def make_c1(R):
    """Action expert over a video K/V cache, bf16 (config 1 shape family)."""
    torch.manual_seed(1)
    cfg = dict(hidden_dim=64, action_dim=7, ffn_dim=256, text_dim=96, freq_dim=256, eps=1e-6,
               num_heads=4, attn_head_dim=16, num_layers=2)
    dit = R.ActionDiT(**cfg).to(torch.bfloat16).eval()
    Sv, tpf, Sa, C = 40, 10, 8, 12
    g = torch.Generator().manual_seed(1)
    ctx = torch.randn(1, C, 96, generator=g).bfloat16()
    ctx_mask = torch.ones(1, C, dtype=torch.bool)
    ctx_mask[0, C - 3:] = False
    cache_k = [torch.randn(1, Sv, 64, generator=g).bfloat16() for _ in range(2)]
    cache_v = [torch.randn(1, Sv, 64, generator=g).bfloat16() for _ in range(2)]
    noise = torch.randn(1, Sa, 7, generator=g).bfloat16()
    # FastWAM._build_mot_attention_mask, called unbound with only what it reads.
    host = SimpleNamespace(video_expert=SimpleNamespace(
        build_video_to_video_mask=lambda video_seq_len, video_tokens_per_frame, device:
        R.WanVideoDiT.build_video_to_video_mask(
            SimpleNamespace(video_attention_mask_mode="first_frame_causal"), video_seq_len,
            video_tokens_per_frame, device)))
    mask = R.FastWAM._build_mot_attention_mask(host, Sv, Sa, tpf, torch.device("cpu"))
    action_mask = mask[Sv:, :]
    # MoT needs a video expert with the same layer count / heads / head dim.
    video = R.WanVideoDiT(hidden_dim=32, in_dim=16, ffn_dim=64, out_dim=16, text_dim=96,
                          freq_dim=256, eps=1e-6, patch_size=(1, 2, 2), num_heads=4,
                          attn_head_dim=16, num_layers=2, has_image_input=False,
                          seperated_timestep=True).to(torch.bfloat16)
    mot = R.MoT({"video": video, "action": dit}).eval()
    mot_host = SimpleNamespace(action_expert=dit, mot=mot)
    sched = R.WanContinuousFlowMatchScheduler(shift=5.0)
    ts, ds = sched.build_inference_schedule(3, device="cpu", dtype=torch.bfloat16)
    x = noise.clone()
    vs = []
    with torch.no_grad():
        for t, d in zip(ts, ds):
            v = R.FastWAM._denoise_action_with_video_cache(
                mot_host, latents_action=x, timestep_action=t.unsqueeze(0).to(torch.bfloat16),
                context=ctx, context_mask=ctx_mask, video_cache_k=cache_k, video_cache_v=cache_v,
                action_attention_mask=action_mask)
            vs.append(v.clone())
            x = sched.step(v, d, x)
    return {
        "kind": "c1", "dit_cfg": cfg, "num_steps": 3, "shift": 5.0, "tokens_per_frame": tpf,
        "dit": _sd(dit, torch.bfloat16), "context": ctx, "context_mask": ctx_mask,
        "cache_k": torch.stack(cache_k), "cache_v": torch.stack(cache_v), "noise": noise,
        "action_mask": action_mask, "timesteps": ts, "deltas": ds,
        "velocities": torch.stack(vs), "latent": x,
    }


def make_c2(R):
    """Video DiT prefill producing the per-layer K/V cache, bf16 (config 2 shape family)."""
    torch.manual_seed(2)
    # head_dim 24 splits into even (8, 8, 8) RoPE parts, as 128 -> (44, 42, 42) does.
    vcfg = dict(hidden_dim=96, in_dim=16, ffn_dim=128, out_dim=16, text_dim=96, freq_dim=256,
                eps=1e-6, patch_size=(1, 2, 2), num_heads=4, attn_head_dim=24, num_layers=2,
                has_image_input=False, seperated_timestep=True,
                video_attention_mask_mode="first_frame_causal")
    video = R.WanVideoDiT(**vcfg).to(torch.bfloat16).eval()
    action = R.ActionDiT(hidden_dim=32, action_dim=7, ffn_dim=64, text_dim=96, freq_dim=256,
                         eps=1e-6, num_heads=4, attn_head_dim=24, num_layers=2).to(torch.bfloat16)
    mot = R.MoT({"video": video, "action": action}).eval()
    g = torch.Generator().manual_seed(2)
    latents = torch.randn(1, 16, 3, 4, 6, generator=g).bfloat16()
    C = 12
    ctx = torch.randn(1, C, 96, generator=g).bfloat16()
    ctx_mask = torch.ones(1, C, dtype=torch.bool)
    ctx_mask[0, -2:] = False
    timestep = torch.tensor([500.0]).bfloat16()
    with torch.no_grad():
        (tokens, t, t_mod, vctx, vctx_mask, freqs, f, h, w, tpf) = video.prepare(
            x=latents, timestep=timestep, context=ctx, context_mask=ctx_mask, action=None,
            fuse_vae_embedding_in_latents=True)
        vmask = video.build_video_to_video_mask(tokens.shape[1], tpf, torch.device("cpu"))
        ks, vs = mot.prefill_video_cache_tensor(
            video_tokens=tokens, video_freqs=freqs, video_t_mod=t_mod, video_context=vctx,
            video_context_mask=vctx_mask, video_attention_mask=vmask)
        x = tokens
        for blk in video.blocks:
            x = blk(x, vctx, t_mod, freqs, context_mask=vctx_mask, self_attn_mask=vmask)
    cfg = {k: vcfg[k] for k in ("hidden_dim", "in_dim", "ffn_dim", "out_dim", "text_dim",
                                "freq_dim", "eps", "num_heads", "attn_head_dim", "num_layers")}
    cfg["patch_size"] = list(vcfg["patch_size"])
    return {
        "kind": "c2", "dit_cfg": cfg, "video": _sd(video, torch.bfloat16), "latents": latents,
        "context": ctx, "context_mask": ctx_mask, "timestep": timestep, "tokens": tokens,
        "t_mod": t_mod, "context_emb": vctx, "freqs": freqs, "grid": (f, h, w),
        "tokens_per_frame": tpf, "video_mask": vmask, "cache_k": torch.stack(ks),
        "cache_v": torch.stack(vs), "hidden": x,
    }


def make_primitives(R):
    """Known-answer vectors for the small numeric building blocks."""
    g = torch.Generator().manual_seed(3)
    pos = torch.tensor([0.0, 1.0, 250.0, 500.0, 936.0, 1000.0])
    x = torch.randn(2, 5, 4 * 16, generator=g).bfloat16()
    freqs1 = R.precompute_freqs_cis(16, end=1024)[:5].view(5, 1, -1)
    f3 = R.precompute_freqs_cis_3d(128)
    sched = R.WanContinuousFlowMatchScheduler(shift=5.0)
    out = {"kind": "primitives"}
    for n, s in ((10, 1.0), (10, 5.0), (4, 1.0), (4, 5.0)):
        for dt in (torch.float32, torch.bfloat16):
            t, d = sched.build_inference_schedule(n, device="cpu", dtype=dt, shift_override=s)
            out[f"sched_{n}_{s}_{str(dt).split('.')[-1]}"] = (t, d)
    out.update({
        "sin_pos": pos, "sin_f32": R.sinusoidal_embedding_1d(256, pos),
        "sin_bf16": R.sinusoidal_embedding_1d(256, pos.bfloat16()),
        "rope_x": x, "rope_out": R.rope_apply(x, freqs1, 4),
        "freqs3_shapes": [tuple(t.shape) for t in f3],
        "freqs3_row7": torch.cat([t[7] for t in f3]),
    })
    return out


def make_joint(R):
    """One joint video + action model evaluation (infer_joint's step), bf16."""
    torch.manual_seed(5)
    # head_dim 128: the 3-D RoPE splits it into (44, 42, 42) as at full size
    vcfg = dict(hidden_dim=128, in_dim=16, ffn_dim=256, out_dim=16, text_dim=96, freq_dim=256,
                eps=1e-6, patch_size=(1, 2, 2), num_heads=2, attn_head_dim=128, num_layers=2,
                has_image_input=False, seperated_timestep=True,
                video_attention_mask_mode="first_frame_causal")
    acfg = dict(hidden_dim=64, action_dim=7, ffn_dim=128, text_dim=96, freq_dim=256, eps=1e-6,
                num_heads=2, attn_head_dim=128, num_layers=2)
    video = R.WanVideoDiT(**vcfg).to(torch.bfloat16).eval()
    action = R.ActionDiT(**acfg).to(torch.bfloat16).eval()
    mot = R.MoT({"video": video, "action": action}).eval()
    g = torch.Generator().manual_seed(5)
    latents_video = torch.randn(1, 16, 3, 4, 6, generator=g).bfloat16()
    latents_action = torch.randn(1, 8, 7, generator=g).bfloat16()
    C = 12
    ctx = torch.randn(1, C, 96, generator=g).bfloat16()
    ctx_mask = torch.ones(1, C, dtype=torch.bool)
    ctx_mask[0, -3:] = False
    tv = torch.tensor([700.0]).bfloat16()
    ta = torch.tensor([700.0]).bfloat16()
    host = SimpleNamespace(video_expert=SimpleNamespace(
        build_video_to_video_mask=lambda video_seq_len, video_tokens_per_frame, device:
        R.WanVideoDiT.build_video_to_video_mask(
            SimpleNamespace(video_attention_mask_mode="first_frame_causal"), video_seq_len,
            video_tokens_per_frame, device)))
    tpf, Sv, Sa = 6, 18, 8
    mask = R.FastWAM._build_mot_attention_mask(host, Sv, Sa, tpf, torch.device("cpu"))
    core_host = SimpleNamespace(video_expert=video, action_expert=action, mot=mot)
    with torch.no_grad():
        pv, pa = R.FastWAM._joint_denoise_core(
            core_host, latents_video=latents_video, latents_action=latents_action, timestep_video=tv,
            timestep_action=ta, context=ctx, context_mask=ctx_mask, attention_mask=mask,
            fuse_vae_embedding_in_latents=True)
    return {"kind": "joint", "video_cfg": vcfg, "action_cfg": acfg, "video": _sd(video, torch.bfloat16),
            "action": _sd(action, torch.bfloat16), "latents_video": latents_video,
            "latents_action": latents_action, "timestep_video": tv, "timestep_action": ta,
            "context": ctx, "context_mask": ctx_mask, "mask": mask, "pred_video": pv, "pred_action": pa}


def make_idm(R):
    """One video-only denoising step of FastWAMIDM and the FastWAMJoint MoT mask
    (action rows see the whole video), bf16; weights of the joint fixture's shape."""
    torch.manual_seed(6)
    vcfg = dict(hidden_dim=128, in_dim=16, ffn_dim=256, out_dim=16, text_dim=96, freq_dim=256,
                eps=1e-6, patch_size=(1, 2, 2), num_heads=2, attn_head_dim=128, num_layers=2,
                has_image_input=False, seperated_timestep=True,
                video_attention_mask_mode="first_frame_causal")
    video = R.WanVideoDiT(**vcfg).to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(6)
    latents_video = torch.randn(1, 16, 3, 4, 6, generator=g).bfloat16()
    C = 12
    ctx = torch.randn(1, C, 96, generator=g).bfloat16()
    ctx_mask = torch.ones(1, C, dtype=torch.bool)
    ctx_mask[0, -2:] = False
    tv = torch.tensor([600.0]).bfloat16()
    tpf, Sv, Sa = 6, 18, 8
    vmask = video.build_video_to_video_mask(Sv, tpf, torch.device("cpu"))
    host = SimpleNamespace(video_expert=video)
    with torch.no_grad():
        pred = R.FastWAMIDM._denoise_video(host, latents_video=latents_video, timestep_video=tv, context=ctx,
                                           context_mask=ctx_mask, video_self_attn_mask=vmask,
                                           fuse_vae_embedding_in_latents=True)
        mask = R.FastWAMJoint._build_mot_attention_mask(host, Sv, Sa, tpf, torch.device("cpu"))
    return {"kind": "idm", "video_cfg": vcfg, "video": _sd(video, torch.bfloat16), "latents_video": latents_video,
            "timestep_video": tv, "context": ctx, "context_mask": ctx_mask, "pred_video": pred, "joint_mask": mask}


def make_vae(R):
    """Wan2.2 VAE (VideoVAE38_) encode of a first frame at a small width.

    Every parameter is re-drawn (the reference zero-initialises the attention
    projection, which would hide the attention path) and rounded to bf16."""
    torch.manual_seed(4)
    cfg = dict(dim=8, z_dim=8, dec_dim=8)
    m = R.VideoVAE38_(**cfg).eval()
    g = torch.Generator().manual_seed(4)
    with torch.no_grad():
        for name, prm in m.named_parameters():
            if name.endswith("gamma"):
                prm.copy_(1.0 + 0.1 * torch.randn(prm.shape, generator=g))
            elif name.endswith("bias"):
                prm.copy_(0.05 * torch.randn(prm.shape, generator=g))
            else:
                fan_in = prm[0].numel()
                prm.copy_(torch.randn(prm.shape, generator=g) / fan_in ** 0.5)
    _round_params_bf16(m)
    image = (torch.rand(1, 3, 1, 64, 96, generator=g) * 2 - 1).bfloat16()
    mean = (0.2 * torch.randn(8, generator=g)).bfloat16().float()
    inv_std = (1.0 + 0.5 * torch.rand(8, generator=g)).bfloat16().float()
    out = {"kind": "vae", "cfg": cfg, "image": image, "mean": mean, "inv_std": inv_std,
           # the temporal downsample convs never run on a first frame
           "params": {k: v.detach().to(torch.bfloat16).clone() for k, v in m.state_dict().items()
                      if (k.startswith("encoder.") or k.startswith("conv1.")) and ".time_conv." not in k}}
    with torch.no_grad():
        out["mu_f32"] = m.float().encode(image.float(), [mean, inv_std])
        out["mu_bf16"] = m.bfloat16().encode(image, [mean.bfloat16(), inv_std.bfloat16()])
    return out


class _VaeHolder:
    """The attributes FastWAM reads from its `vae`: .model.encode(x, scale), .scale, .to()."""

    def __init__(self, model, mean, inv_std):
        self.model, self.scale = model, [mean, inv_std]

    def to(self, *args, **kwargs):
        self.model.to(*args, **kwargs)
        return self


def make_fastwam(R):
    """FastWAM.infer_action end to end at small shapes (fastwam.py:1080-1274): VAE encode of
    the observation, proprio token appended to the context, video prefill at t = 0, the MoT
    action Euler loop over the K/V cache, Action-VAE decode.  bf16 experts, VAE and proprio
    encoder (the reference's torch_dtype), fp32 Action-VAE; the checkpoint payload is saved in
    the reference's own format ({"mot": mot.state_dict(), "proprio_encoder": ...})."""
    torch.manual_seed(9)
    vcfg = dict(hidden_dim=128, in_dim=8, ffn_dim=256, out_dim=8, text_dim=96, freq_dim=256, eps=1e-6,
                patch_size=(1, 2, 2), num_heads=2, attn_head_dim=128, num_layers=2, has_image_input=False,
                seperated_timestep=True, video_attention_mask_mode="first_frame_causal")
    acfg = dict(hidden_dim=64, action_dim=16, ffn_dim=128, text_dim=96, freq_dim=256, eps=1e-6,
                num_heads=2, attn_head_dim=128, num_layers=2)
    ae_cfg = dict(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16, decoder_hidden=64,
                  video_cond_dim=0, variational=True)
    vae_cfg = dict(dim=8, z_dim=8, dec_dim=8)
    video = R.WanVideoDiT(**vcfg).to(torch.bfloat16).eval()
    action = R.ActionDiT(**acfg).to(torch.bfloat16).eval()
    mot = R.MoT({"video": video, "action": action}).eval()
    vmodel = R.VideoVAE38_(**vae_cfg).eval()
    g = torch.Generator().manual_seed(9)
    with torch.no_grad():
        for name, prm in vmodel.named_parameters():
            if name.endswith("gamma"):
                prm.copy_(1.0 + 0.1 * torch.randn(prm.shape, generator=g))
            elif name.endswith("bias"):
                prm.copy_(0.05 * torch.randn(prm.shape, generator=g))
            else:
                prm.copy_(torch.randn(prm.shape, generator=g) / prm[0].numel() ** 0.5)
    vmodel = vmodel.bfloat16()
    mean = (0.2 * torch.randn(8, generator=g)).bfloat16()
    inv_std = (1.0 + 0.5 * torch.rand(8, generator=g)).bfloat16()
    ae = R.ActionAE(R.ActionAEConfig(**ae_cfg)).eval()
    model = R.FastWAM(video_expert=video, action_expert=action, mot=mot, vae=_VaeHolder(vmodel, mean, inv_std),
                      text_dim=96, proprio_dim=8, action_vae=ae, device="cpu", torch_dtype=torch.bfloat16,
                      action_infer_shift=5.0)
    image = (torch.rand(1, 3, 64, 96, generator=g) * 2 - 1).bfloat16()
    C = 12
    ctx = torch.randn(1, C, 96, generator=g).bfloat16()
    ctx_mask = torch.ones(1, C, dtype=torch.bool)
    ctx_mask[0, -3:] = False
    proprio = torch.randn(1, 8, generator=g).bfloat16()
    with torch.no_grad():
        out = model.infer_action(prompt=None, input_image=image, action_horizon=32, proprio=proprio,
                                 context=ctx, context_mask=ctx_mask, num_inference_steps=4, seed=42,
                                 rand_device="cpu", return_action_latents=True)
    payload = {"mot": {k: v.detach().clone() for k, v in mot.state_dict().items()}, "step": None,
               "torch_dtype": str(torch.bfloat16),
               "proprio_encoder": {k: v.detach().clone() for k, v in model.proprio_encoder.state_dict().items()}}
    return {"kind": "fastwam", "video_cfg": vcfg, "action_cfg": acfg, "ae_cfg": ae_cfg, "vae_cfg": vae_cfg,
            "checkpoint": payload,
            "vae_params": {k: v.detach().clone() for k, v in vmodel.state_dict().items()
                           if (k.startswith("encoder.") or k.startswith("conv1.")) and ".time_conv." not in k},
            "vae_mean": mean, "vae_inv_std": inv_std,
            "action_vae": {"config": ae_cfg, "model": {k: v.detach().clone() for k, v in ae.state_dict().items()}},
            "input_image": image, "context": ctx, "context_mask": ctx_mask, "proprio": proprio,
            "num_inference_steps": 4, "seed": 42, "action_horizon": 32, "action_infer_shift": 5.0,
            "action": out["action"], "action_latents": out["action_latents"]}


def _import_dit4dit_action_vae(ref_root: Path):
    """DiT4DiT's ActionVAE module, loaded from its file alone (its package __init__ files pull
    in the VLM stack, which the decode never touches)."""
    import importlib.util
    path = ref_root / "DiT4DiT" / "DiT4DiT" / "model" / "modules" / "action_model" / "action_vae.py"
    spec = importlib.util.spec_from_file_location("dit4dit_action_vae", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # dataclass resolution needs the module registered
    spec.loader.exec_module(mod)
    return mod


def make_dit4dit_vae(ref_root: Path):
    """DiT4DiT ActionVAE.decode (DiT4DiT/model/modules/action_model/action_vae.py:136-197), fp32,
    in the shapes that exercise every branch of the decoder: the config-3 compact chunk
    (8 x 48 latents -> 16 x 29) with the decoder's task embedding (conditioning_mode
    "encoder_decoder"), an "encoder_only" model whose decoder ignores task ids, a stride-3
    ConvTranspose1d whose 3L + 1 output is cropped, and two upsampling stages (3, 3) with a
    crop.  (The zero-pad branch of decode is unreachable through ActionVAE, whose encoder
    requires the horizon to be a multiple of num_tokens.)  Each case saves the reference's
    checkpoint layout ({"config": ActionVAEConfig.to_dict(), "model": state_dict}, as
    load_action_vae reads it, action_vae.py:276-283).  The config-3 case also records
    DiT4DiT._decode_action_predictions' latent un-normalisation followed by the decode
    (DiT4DiT/model/framework/DiT4DiT.py:403-407)."""
    V = _import_dit4dit_action_vae(ref_root)
    cases = {
        "c3_task_conditioned": dict(action_dim=29, action_horizon=16, num_tokens=8, latent_dim=48,
                                    encoder_hidden=32, decoder_hidden=64, num_tasks=3,
                                    conditioning_mode="encoder_decoder", batch=3),
        "encoder_only": dict(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16, encoder_hidden=32,
                             decoder_hidden=32, num_tasks=2, conditioning_mode="encoder_only", batch=2),
        "stride3_crop": dict(action_dim=5, action_horizon=12, num_tokens=4, latent_dim=8, encoder_hidden=32,
                             decoder_hidden=32, batch=2),
        "two_stage_crop": dict(action_dim=6, action_horizon=18, num_tokens=2, latent_dim=8, encoder_hidden=32,
                               decoder_hidden=32, batch=2),
    }
    out = {"kind": "dit4dit_action_vae", "cases": {}}
    for i, (name, kw) in enumerate(cases.items()):
        kw = dict(kw)
        B = kw.pop("batch")
        torch.manual_seed(100 + i)
        cfg = V.ActionVAEConfig(**kw)
        vae = V.ActionVAE(cfg).eval()
        g = torch.Generator().manual_seed(200 + i)
        with torch.no_grad():
            # GroupNorm affines and the (zero-initialised) task embeddings get values, so
            # every parameter changes the output
            for mod in vae.modules():
                if isinstance(mod, torch.nn.GroupNorm):
                    mod.weight.copy_(1.0 + 0.2 * torch.randn(mod.weight.shape, generator=g))
                    mod.bias.copy_(0.2 * torch.randn(mod.bias.shape, generator=g))
                elif isinstance(mod, torch.nn.Embedding):
                    mod.weight.copy_(0.5 * torch.randn(mod.weight.shape, generator=g))
        _round_params_bf16(vae)
        z = torch.randn(B, cfg.num_tokens, cfg.latent_dim, generator=g)
        task_ids = torch.randint(0, max(1, cfg.num_tasks), (B,), generator=g) if cfg.num_tasks > 0 else None
        with torch.no_grad():
            actions = vae.decode(z, task_ids=task_ids)
        rec = {"checkpoint": {"config": cfg.to_dict(),
                              "model": {k: v.detach().clone() for k, v in vae.state_dict().items()}},
               "latent": z, "task_ids": task_ids, "actions": actions}
        if name == "c3_task_conditioned":
            # per token and channel, as DiT4DiT registers them (DiT4DiT.py:256-266)
            mean = 0.3 * torch.randn(cfg.num_tokens, cfg.latent_dim, generator=g)
            std = 0.5 + torch.rand(cfg.num_tokens, cfg.latent_dim, generator=g)
            with torch.no_grad():
                rec["actions_denorm"] = vae.decode(z * std + mean, task_ids=task_ids)
            rec["checkpoint"].update(latent_mean=mean, latent_std=std, apply_latent_normalization=True)
        out["cases"][name] = rec
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of the reference project checkout (holds FastWAM/src)")
    ap.add_argument("--only", nargs="*", default=None, help="fixture names to (re)generate")
    args = ap.parse_args()
    ref_root = Path(args.reference)
    R = _import_reference(ref_root)
    torch.set_num_threads(4)
    for name, fn in (("c0_cae_expert", make_c0), ("c1_action_cache", make_c1),
                     ("c2_video_prefill", make_c2), ("primitives", make_primitives),
                     ("vae_encode", make_vae), ("joint_step", make_joint), ("idm_step", make_idm),
                     ("fastwam_infer_action", make_fastwam),
                     ("dit4dit_action_vae", lambda _: make_dit4dit_vae(ref_root))):
        if args.only is not None and name not in args.only:
            continue
        fx = fn(R)
        path = OUT / f"{name}.pt"
        torch.save(fx, path)
        print(f"{path.name}: {path.stat().st_size / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
