"""Pins the CPU oracle to the reference: every committed golden fixture was
produced by running the reference's own modules (tests/golden/make_golden.py);
the oracle, given the same state dicts and inputs, must reproduce them."""
from pathlib import Path

import pytest
import torch

from oracle import fam_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load(name):
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


def _f32(sd):
    return {k: v.float() for k, v in sd.items()}


def _same(got, ref, atol=0.0):
    got, ref = got.float(), ref.float()
    assert got.shape == ref.shape, (got.shape, ref.shape)
    err = (got - ref).abs().max().item()
    assert err <= atol, f"max |d| = {err}"


def test_primitives_match_reference():
    fx = _load("primitives")
    _same(O.sinusoidal_embedding_1d(256, fx["sin_pos"]), fx["sin_f32"])
    _same(O.sinusoidal_embedding_1d(256, fx["sin_pos"].bfloat16()), fx["sin_bf16"])
    freqs = O.precompute_freqs_cis(16, end=1024)[:5].view(5, 1, -1)
    _same(O.rope_apply(fx["rope_x"], freqs, 4), fx["rope_out"])
    f3 = O.precompute_freqs_cis_3d(128)
    assert [tuple(t.shape) for t in f3] == fx["freqs3_shapes"]
    assert torch.equal(torch.cat([t[7] for t in f3]), fx["freqs3_row7"])
    for key, (t_ref, d_ref) in ((k, v) for k, v in fx.items() if k.startswith("sched_")):
        _, n, s, dt = key.split("_")
        t, d = O.build_inference_schedule(int(n), float(s), dtype=getattr(torch, {"float32": "float32", "bfloat16": "bfloat16"}[dt]))
        assert torch.equal(t, t_ref) and torch.equal(d, d_ref), key


def test_schedule_known_answers():
    # shift 1, 4 steps: t = 1000, 750, 500, 250 and delta = -0.25
    t, d = O.build_inference_schedule(4, 1.0)
    assert t.tolist() == [1000.0, 750.0, 500.0, 250.0]
    assert torch.allclose(d, torch.full((4,), -0.25))
    # bf16 rounding of the shifted schedule: 937.5 -> 936
    t5, _ = O.build_inference_schedule(4, 5.0, dtype=torch.bfloat16)
    assert t5[1].item() == 936.0


def test_c0_cae_chunk_matches_reference():
    fx = _load("c0_cae_expert")
    cfg = O.DiTConfig(**{k: fx["dit_cfg"][k] for k in ("hidden_dim", "ffn_dim", "num_heads",
                                                       "attn_head_dim", "num_layers", "text_dim",
                                                       "freq_dim", "eps", "action_dim")})
    dcfg = O.DecoderConfig(**fx["dec_cfg"])
    chunk, latent, vs = O.cae_chunk(_f32(fx["dit"]), cfg, _f32(fx["ae"]), dcfg, fx["noise"],
                                    fx["context"].float(), num_steps=4, shift=1.0,
                                    return_trace=True)
    _same(torch.stack(vs), fx["velocities"], 1e-5)
    _same(latent, fx["latent"], 1e-5)
    _same(chunk, fx["chunk"], 1e-5)


def test_c1_action_cache_matches_reference():
    fx = _load("c1_action_cache")
    c = fx["dit_cfg"]
    cfg = O.DiTConfig(**{k: c[k] for k in ("hidden_dim", "ffn_dim", "num_heads", "attn_head_dim",
                                           "num_layers", "text_dim", "freq_dim", "eps",
                                           "action_dim")})
    x, vs = O.action_chunk_with_cache(fx["dit"], cfg, fx["noise"], fx["context"],
                                      fx["context_mask"], list(fx["cache_k"]), list(fx["cache_v"]),
                                      fx["action_mask"], fx["num_steps"], fx["shift"],
                                      return_trace=True)
    _same(torch.stack(vs), fx["velocities"])
    _same(x, fx["latent"])


def test_c1_mask_matches_reference():
    fx = _load("c1_action_cache")
    Sv = fx["cache_k"].shape[2]
    Sa = fx["noise"].shape[1]
    m = O.build_mot_attention_mask(Sv, Sa, fx["tokens_per_frame"])
    assert torch.equal(m[Sv:, :], fx["action_mask"])


def test_c2_video_prefill_matches_reference():
    fx = _load("c2_video_prefill")
    c = fx["dit_cfg"]
    cfg = O.DiTConfig(hidden_dim=c["hidden_dim"], ffn_dim=c["ffn_dim"], num_heads=c["num_heads"],
                      attn_head_dim=c["attn_head_dim"], num_layers=c["num_layers"],
                      text_dim=c["text_dim"], freq_dim=c["freq_dim"], eps=c["eps"],
                      in_dim=c["in_dim"], out_dim=c["out_dim"], patch_size=tuple(c["patch_size"]))
    p = fx["video"]
    tokens, t, t_mod, ctx, ctx_mask, freqs, grid, tpf = O.video_prepare(
        p, cfg, fx["latents"], fx["timestep"], fx["context"], fx["context_mask"])
    _same(tokens, fx["tokens"])
    _same(t_mod, fx["t_mod"])
    _same(ctx, fx["context_emb"])
    assert torch.equal(freqs, fx["freqs"])
    assert grid == tuple(fx["grid"]) and tpf == fx["tokens_per_frame"]
    vmask = O.build_video_to_video_mask(tokens.shape[1], tpf)
    assert torch.equal(vmask, fx["video_mask"])
    ks, vs, hidden = O.prefill_video_cache(p, cfg, tokens, freqs, t_mod, ctx, ctx_mask, vmask,
                                           return_hidden=True)
    _same(torch.stack(ks), fx["cache_k"])
    _same(torch.stack(vs), fx["cache_v"])
    _same(hidden, fx["hidden"])


def test_vae_encode_matches_reference():
    """VideoVAE38_.encode of one frame: bit-exact at bf16, fp32 to rounding."""
    fx = _load("vae_encode")
    c = fx["cfg"]
    cfg = O.VaeConfig(dim=c["dim"], z_dim=c["z_dim"])
    mu = O.vae_encode_first_frame(fx["params"], cfg, fx["image"], fx["mean"].bfloat16(),
                                  fx["inv_std"].bfloat16())
    assert torch.equal(mu, fx["mu_bf16"])
    p32 = {k: v.float() for k, v in fx["params"].items()}
    mu32 = O.vae_encode_first_frame(p32, cfg, fx["image"].float(), fx["mean"], fx["inv_std"])
    assert (mu32 - fx["mu_f32"]).abs().max().item() < 1e-5


def test_joint_step_matches_reference():
    """FastWAM._joint_denoise_core (both experts under the MoT mask): bit-exact at bf16."""
    fx = _load("joint_step")
    vc, ac = fx["video_cfg"], fx["action_cfg"]
    vcfg = O.DiTConfig(hidden_dim=vc["hidden_dim"], ffn_dim=vc["ffn_dim"], num_heads=vc["num_heads"],
                       attn_head_dim=vc["attn_head_dim"], num_layers=vc["num_layers"], text_dim=vc["text_dim"],
                       freq_dim=vc["freq_dim"], eps=vc["eps"], in_dim=vc["in_dim"], out_dim=vc["out_dim"],
                       patch_size=tuple(vc["patch_size"]))
    acfg = O.DiTConfig(hidden_dim=ac["hidden_dim"], ffn_dim=ac["ffn_dim"], num_heads=ac["num_heads"],
                       attn_head_dim=ac["attn_head_dim"], num_layers=ac["num_layers"], text_dim=ac["text_dim"],
                       freq_dim=ac["freq_dim"], eps=ac["eps"], action_dim=ac["action_dim"])
    pv, pa = O.joint_denoise_core(fx["video"], vcfg, fx["action"], acfg, fx["latents_video"],
                                  fx["latents_action"], fx["timestep_video"], fx["timestep_action"],
                                  fx["context"], fx["context_mask"])
    _same(pv, fx["pred_video"])
    _same(pa, fx["pred_action"])
    assert torch.equal(O.build_mot_attention_mask(pv.shape[2] * 6, pa.shape[1], 6), fx["mask"])


def test_idm_video_step_and_joint_mask_match_reference():
    """FastWAMIDM._denoise_video (video expert alone + head) and FastWAMJoint's MoT
    mask (action rows see the whole video): bit-exact at bf16."""
    fx = _load("idm_step")
    vc = fx["video_cfg"]
    vcfg = O.DiTConfig(hidden_dim=vc["hidden_dim"], ffn_dim=vc["ffn_dim"], num_heads=vc["num_heads"],
                       attn_head_dim=vc["attn_head_dim"], num_layers=vc["num_layers"], text_dim=vc["text_dim"],
                       freq_dim=vc["freq_dim"], eps=vc["eps"], in_dim=vc["in_dim"], out_dim=vc["out_dim"],
                       patch_size=tuple(vc["patch_size"]))
    pv = O.video_denoise_step(fx["video"], vcfg, fx["latents_video"], fx["timestep_video"], fx["context"],
                              fx["context_mask"])
    _same(pv, fx["pred_video"])
    assert torch.equal(O.build_joint_model_mask(18, 8, 6), fx["joint_mask"])


def test_oracle_infer_action_matches_reference_fastwam():
    """The oracle's restatement of FastWAM.infer_action (VAE encode, proprio token, video
    prefill at t = 0, MoT action Euler loop, Action-VAE decode) reproduces the reference run
    recorded in fastwam_infer_action.pt (bf16 experts)."""
    fx = torch.load(GOLDEN / "fastwam_infer_action.pt")
    vc, ac = fx["video_cfg"], fx["action_cfg"]
    vcfg = O.DiTConfig(hidden_dim=vc["hidden_dim"], ffn_dim=vc["ffn_dim"], num_heads=vc["num_heads"],
                       attn_head_dim=vc["attn_head_dim"], num_layers=vc["num_layers"], text_dim=vc["text_dim"],
                       in_dim=vc["in_dim"], out_dim=vc["out_dim"])
    acfg = O.DiTConfig(hidden_dim=ac["hidden_dim"], ffn_dim=ac["ffn_dim"], num_heads=ac["num_heads"],
                       attn_head_dim=ac["attn_head_dim"], num_layers=ac["num_layers"], text_dim=ac["text_dim"],
                       action_dim=ac["action_dim"])
    e = fx["ae_cfg"]
    dcfg = O.DecoderConfig(e["action_dim"], e["action_horizon"], e["num_tokens"], e["latent_dim"],
                           e["decoder_hidden"])
    vae_cfg = O.VaeConfig(dim=fx["vae_cfg"]["dim"], z_dim=fx["vae_cfg"]["z_dim"])
    act, lat = O.infer_action(fx["checkpoint"]["mot"], vcfg, acfg, fx["vae_params"], vae_cfg, fx["vae_mean"],
                              fx["vae_inv_std"], fx["action_vae"]["model"], dcfg,
                              fx["checkpoint"]["proprio_encoder"], fx["input_image"], fx["context"],
                              fx["context_mask"], fx["proprio"], fx["action_horizon"], fx["num_inference_steps"],
                              fx["action_infer_shift"], fx["seed"])
    assert torch.equal(lat, fx["action_latents"])
    assert torch.equal(act, fx["action"])


def dit4dit_decoder_params(ckpt):
    """DiT4DiT ActionVAE checkpoint -> (oracle decoder params, DecoderConfig, whether the decoder
    takes task ids): the decoder's task_embedding is the oracle's suite embedding."""
    c = ckpt["config"]
    cond = c["conditioning_mode"] == "encoder_decoder"
    p = {}
    for k, v in ckpt["model"].items():
        if k.startswith("decoder."):
            p[k.replace("decoder.task_embedding.", "decoder.suite_embed.")] = v.float()
    cfg = O.DecoderConfig(c["action_dim"], c["action_horizon"], c["num_tokens"], c["latent_dim"],
                          c["decoder_hidden"], c["num_tasks"] if cond else 0)
    return p, cfg, cond


@pytest.mark.parametrize("case", ["c3_task_conditioned", "encoder_only", "stride3_crop", "two_stage_crop"])
def test_dit4dit_action_vae_decode_matches_reference(case):
    """The oracle's decoder reproduces DiT4DiT's ActionVAE.decode (action_vae.py:136-197) on
    the fixture made from the reference module: task-conditioned, task ids ignored by an
    "encoder_only" decoder, a stride-3 crop and two upsampling stages; and the latent
    un-normalisation of DiT4DiT._decode_action_predictions (DiT4DiT.py:403-406)."""
    fx = _load("dit4dit_action_vae")["cases"][case]
    p, cfg, cond = dit4dit_decoder_params(fx["checkpoint"])
    ids = fx["task_ids"] if cond else None
    _same(O.action_decode(p, cfg, fx["latent"], suite_ids=ids), fx["actions"], atol=1e-6)
    if "actions_denorm" in fx:
        ck = fx["checkpoint"]
        z = fx["latent"] * ck["latent_std"].clamp_min(1e-4) + ck["latent_mean"]
        _same(O.action_decode(p, cfg, z, suite_ids=ids), fx["actions_denorm"], atol=1e-6)
