"""Joint video + action denoising (FastWAM.infer_joint's model evaluation,
_joint_denoise_core) on the GPU: the video expert's forward + output head and the
action expert over that step's K/V, against the reference's recorded output (golden
fixture) and a multi-step loop against the CPU oracle.  Bound: max|d| <= 2e-2 x
max(1, max|ref|) and cosine >= 0.999."""
import importlib
from pathlib import Path

import pytest
import torch

from oracle import fam_oracle as O

pytestmark = pytest.mark.gpu

M = importlib.import_module("faster-action-models_b200.models")
P = importlib.import_module("faster-action-models_b200.pipeline")
GOLDEN = Path(__file__).resolve().parent / "golden"


def _check(got, ref, name):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert got.shape == ref.shape, (name, got.shape, ref.shape)
    err = (got - ref).abs().max().item()
    scale = max(1.0, ref.abs().max().item())
    cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
    assert err <= 2e-2 * scale and cos >= 0.999, f"{name}: max|d| {err} (scale {scale}) cos {cos}"


def _policy(fx):
    vc, ac = dict(fx["video_cfg"]), dict(fx["action_cfg"])
    vid = M.WanVideoDiT(**vc)
    vid.load_state_dict({k: v.float() for k, v in fx["video"].items()})
    act = M.ActionDiT(**ac)
    act.load_state_dict({k: v.float() for k, v in fx["action"].items()})
    vid, act = vid.to("cuda", torch.bfloat16), act.to("cuda", torch.bfloat16)
    return P.FastWAMJointPolicy(vid, act), vc, ac


def _cfgs(vc, ac):
    vcfg = O.DiTConfig(hidden_dim=vc["hidden_dim"], ffn_dim=vc["ffn_dim"], num_heads=vc["num_heads"],
                       attn_head_dim=vc["attn_head_dim"], num_layers=vc["num_layers"], text_dim=vc["text_dim"],
                       freq_dim=vc["freq_dim"], eps=vc["eps"], in_dim=vc["in_dim"], out_dim=vc["out_dim"],
                       patch_size=tuple(vc["patch_size"]))
    acfg = O.DiTConfig(hidden_dim=ac["hidden_dim"], ffn_dim=ac["ffn_dim"], num_heads=ac["num_heads"],
                       attn_head_dim=ac["attn_head_dim"], num_layers=ac["num_layers"], text_dim=ac["text_dim"],
                       freq_dim=ac["freq_dim"], eps=ac["eps"], action_dim=ac["action_dim"])
    return vcfg, acfg


def test_joint_step_golden():
    fx = torch.load(GOLDEN / "joint_step.pt", weights_only=False)
    pol, _, _ = _policy(fx)
    pv, pa = pol.joint_step(fx["latents_video"].cuda(), fx["latents_action"].cuda(), fx["timestep_video"],
                            fx["timestep_action"], fx["context"].cuda(), fx["context_mask"].cuda())
    torch.cuda.synchronize()
    _check(pv, fx["pred_video"], "video prediction")
    _check(pa, fx["pred_action"], "action prediction")


def test_infer_joint_against_oracle_loop():
    """Three joint Euler steps from seeded noise with the first latent frame pinned."""
    fx = torch.load(GOLDEN / "joint_step.pt", weights_only=False)
    pol, vc, ac = _policy(fx)
    vcfg, acfg = _cfgs(vc, ac)
    first = fx["latents_video"][:, :, :1].clone()
    ctx, cm = fx["context"], fx["context_mask"]
    out = pol.infer_joint(first.cuda(), 3, ctx.cuda(), cm.cuda(), action_horizon=8, num_inference_steps=3,
                          seed=7)
    torch.cuda.synchronize()
    # oracle: the same loop in fp32 on the bf16 weights
    pv32 = {k: v.float() for k, v in fx["video"].items()}
    pa32 = {k: v.float() for k, v in fx["action"].items()}
    gv = torch.Generator().manual_seed(7)
    ga = torch.Generator().manual_seed(7)
    lat_v = torch.randn((1, 16, 3, 4, 6), generator=gv).bfloat16().float()
    lat_a = torch.randn((1, 8, 7), generator=ga).bfloat16().float()
    lat_v[:, :, 0:1] = first.float()
    ts, ds = O.build_inference_schedule(3, 5.0, dtype=torch.bfloat16)
    for t, d in zip(ts, ds):
        tt = t.reshape(1).float()
        pv, pa = O.joint_denoise_core(pv32, vcfg, pa32, acfg, lat_v, lat_a, tt, tt, ctx.float(), cm)
        lat_v = O.scheduler_step(pv, d.float(), lat_v)
        lat_a = O.scheduler_step(pa, d.float(), lat_a)
        lat_v[:, :, 0:1] = first.float()
    _check(out["video_latents"], lat_v, "video latents")
    _check(out["action"], lat_a[0], "action latents")


def test_joint_step_full_video_mask():
    """FastWAMJoint: the action rows attend to every video token."""
    fx = torch.load(GOLDEN / "joint_step.pt", weights_only=False)
    pol, vc, ac = _policy(fx)
    pol = P.FastWAMJointPolicy(pol.video_expert, pol.action_expert, action_sees_full_video=True)
    vcfg, acfg = _cfgs(vc, ac)
    pv, pa = pol.joint_step(fx["latents_video"].cuda(), fx["latents_action"].cuda(), fx["timestep_video"],
                            fx["timestep_action"], fx["context"].cuda(), fx["context_mask"].cuda())
    torch.cuda.synchronize()
    f32 = lambda sd: {k: v.float() for k, v in sd.items()}
    rv, ra = O.joint_denoise_core(f32(fx["video"]), vcfg, f32(fx["action"]), acfg, fx["latents_video"].float(),
                                  fx["latents_action"].float(), fx["timestep_video"].float(),
                                  fx["timestep_action"].float(), fx["context"].float(), fx["context_mask"],
                                  full_video=True)
    _check(pv, rv, "video prediction")
    _check(pa, ra, "action prediction (full video)")


def test_idm_video_step_golden():
    """FastWAMIDM._denoise_video against the reference's recorded output."""
    fx = torch.load(GOLDEN / "idm_step.pt", weights_only=False)
    vid = M.WanVideoDiT(**dict(fx["video_cfg"]))
    vid.load_state_dict({k: v.float() for k, v in fx["video"].items()})
    act = M.ActionDiT(64, 7, 128, 96, 256, 1e-6, 2, 128, 2)
    pol = P.FastWAMIDMPolicy(vid.to("cuda", torch.bfloat16), act.to("cuda", torch.bfloat16))
    pv = pol.video_step(fx["latents_video"].cuda(), fx["timestep_video"], fx["context"].cuda(),
                        fx["context_mask"].cuda())
    torch.cuda.synchronize()
    _check(pv, fx["pred_video"], "IDM video step")


def test_idm_infer_action_against_oracle_loop():
    """Two video-only steps (first frame pinned), the timestep-0 cache, then two action
    steps over it with every video token visible."""
    fx = torch.load(GOLDEN / "joint_step.pt", weights_only=False)
    pol, vc, ac = _policy(fx)
    pol = P.FastWAMIDMPolicy(pol.video_expert, pol.action_expert)
    vcfg, acfg = _cfgs(vc, ac)
    first = fx["latents_video"][:, :, :1].clone()
    ctx, cm = fx["context"], fx["context_mask"]
    out = pol.infer_action(first.cuda(), 3, ctx.cuda(), cm.cuda(), action_horizon=8, num_inference_steps=2, seed=3)
    torch.cuda.synchronize()
    pv32 = {k: v.float() for k, v in fx["video"].items()}
    pa32 = {k: v.float() for k, v in fx["action"].items()}
    gv = torch.Generator().manual_seed(3)
    ga = torch.Generator().manual_seed(3)
    lat_v = torch.randn((1, 16, 3, 4, 6), generator=gv).bfloat16().float()
    lat_a = torch.randn((1, 8, 7), generator=ga).bfloat16().float()
    lat_v[:, :, 0:1] = first.float()
    ts, ds = O.build_inference_schedule(2, 5.0, dtype=torch.bfloat16)
    for t, d in zip(ts, ds):
        pv = O.video_denoise_step(pv32, vcfg, lat_v, t.reshape(1).float(), ctx.float(), cm)
        lat_v = O.scheduler_step(pv, d.float(), lat_v)
        lat_v[:, :, 0:1] = first.float()
    tokens, _t, t_mod, cemb, cmask, freqs, grid, tpf = O.video_prepare(pv32, vcfg, lat_v, torch.zeros(1), ctx.float(), cm)
    vmask = O.build_video_to_video_mask(tokens.shape[1], tpf)
    ks, vs = O.prefill_video_cache(pv32, vcfg, tokens, freqs, t_mod, cemb, cmask, vmask)
    amask = O.build_joint_model_mask(tokens.shape[1], 8, tpf)[tokens.shape[1]:]
    for t, d in zip(ts, ds):
        pa = O.denoise_action_with_video_cache(pa32, acfg, lat_a, t.reshape(1).float(), ctx.float(), cm, ks, vs, amask)
        lat_a = O.scheduler_step(pa, d.float(), lat_a)
    _check(out["video_latents"], lat_v, "IDM video latents")
    _check(out["action"], lat_a[0], "IDM action")


def test_optional_idm_modes_match_their_policies():
    """FastWAMOptionalIDM.infer_action: "first_frame" is FastWAM's path, "idm" the IDM path."""
    fx = torch.load(GOLDEN / "joint_step.pt", weights_only=False)
    pol, _, _ = _policy(fx)
    opt = P.FastWAMOptionalIDMPolicy(pol.video_expert, pol.action_expert)
    first = fx["latents_video"][:, :, :1].clone().cuda()
    ctx, cm = fx["context"].cuda(), fx["context_mask"].cuda()
    a = opt.infer_action(first, ctx, cm, action_horizon=8, num_inference_steps=2, seed=5,
                         action_infer_mode="first_frame")
    b = P.FastWAMActionPolicy(pol.video_expert, pol.action_expert).infer_action(
        first, ctx, cm, action_horizon=8, num_inference_steps=2, seed=5)
    _check(a["action"], b["action"], "first_frame mode")
    c = opt.infer_action(first, ctx, cm, action_horizon=8, num_inference_steps=2, seed=5, num_latent_frames=3,
                         action_infer_mode="idm")
    d = P.FastWAMIDMPolicy(pol.video_expert, pol.action_expert).infer_action(
        first, 3, ctx, cm, action_horizon=8, num_inference_steps=2, seed=5)
    _check(c["action"], d["action"], "idm mode")
    _check(c["video_latents"], d["video_latents"], "idm mode video")
