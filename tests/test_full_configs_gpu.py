"""BASELINE configs 2, 3 and 4 at their full widths through the libfam path, against the
oracle in fp32 on the same bf16 weights (the backbone's oracle runs on the GPU in fp32
with TF32 off, the action heads' on the CPU).  Gate: max|d| <= 2e-2 * max(1, max|ref|)
and cosine >= 0.999 on every compared tensor; the measured values are printed (PARITY
lines).

  config 2: the Wan2.2-5B-shaped backbone at full depth (30 blocks, 3072 hidden, 24 x 128
            heads, FFN 14336, 1760 tokens): K / V of blocks 0, 14 and 29 and the final
            token states.
  config 4: the CAE pipeline at config widths (backbone at config-2 widths, 2 blocks;
            the config-0 compact expert, 8 blocks, cross-attending the backbone's final
            1760 x 3072 token states; the Action-VAE decoder, hidden 256), batch 2.
  config 3: the DiT4DiT-shaped path at config widths (backbone hidden 2048, 16 x 128
            heads, FFN 8192, 1 x 4 x 22 x 40 = 3520 tokens, features after the first of
            2 blocks, the second elided as DiT4DiT's feature hook does;
            wide head hidden 1024 / 16 x 64 heads / FFN 4096 over a 16 x 29 chunk, and
            the compact head + Action-VAE over 8 x 48 latents), 4 Euler steps, 2 head
            blocks.
"""
import importlib

import pytest
import torch

from oracle import fam_oracle as O

pytestmark = pytest.mark.gpu

M = importlib.import_module("faster-action-models_b200.models")
P = importlib.import_module("faster-action-models_b200.pipeline")
R = importlib.import_module("faster-action-models_b200.replicas")


@pytest.fixture(autouse=True)
def _no_tf32():
    m, c = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = m, c
    torch.cuda.empty_cache()


def _check(name, got, ref):
    got, ref = got.float().cpu(), ref.float().cpu()
    err = (got - ref).abs().max().item()
    scale = max(1.0, ref.abs().max().item())
    cos = torch.nn.functional.cosine_similarity(got.double().flatten(), ref.double().flatten(), dim=0).item()
    print(f"PARITY {name}: max|d| {err:.4g} (gate {2e-2 * scale:.4g}) cos {cos:.6f}")
    assert err <= 2e-2 * scale and cos >= 0.999, f"{name}: max|d| {err} (scale {scale}) cos {cos}"


def _backbone(D, H, hd, F, T, L, Cin, seed):
    """A WanVideoDiT built on the GPU, with random norm weights so every parameter matters."""
    torch.manual_seed(seed)
    with torch.device("cuda"):
        vid = M.WanVideoDiT(hidden_dim=D, in_dim=Cin, ffn_dim=F, out_dim=Cin, text_dim=T, freq_dim=256,
                            eps=1e-6, patch_size=(1, 2, 2), num_heads=H, attn_head_dim=hd, num_layers=L,
                            has_image_input=False, seperated_timestep=True,
                            video_attention_mask_mode="first_frame_causal")
        with torch.no_grad():
            for n, p in vid.named_parameters():
                if "norm" in n:
                    p.copy_(1.0 + 0.2 * torch.randn_like(p))
    vid = vid.to(torch.bfloat16)
    cfg = O.DiTConfig(hidden_dim=D, ffn_dim=F, num_heads=H, attn_head_dim=hd, num_layers=L, text_dim=T,
                      in_dim=Cin, out_dim=Cin)
    return vid, cfg


def _backbone_oracle(vid, cfg, lat, t, ctx, cm, return_hidden=True):
    sd = {k: v.float() for k, v in vid.state_dict().items()}
    with torch.no_grad():
        tok, _, tmod, cemb, cmask, freqs, _, tpf = O.video_prepare(sd, cfg, lat.float(), t.float().cuda(),
                                                                   ctx.float(), cm)
        vmask = O.build_video_to_video_mask(tok.shape[1], tpf).cuda()
        out = O.prefill_video_cache(sd, cfg, tok, freqs.cuda(), tmod, cemb, cmask, vmask,
                                    return_hidden=return_hidden)
    del sd
    return out


def _inputs(B, Cin, Fr, Hh, Ww, C, T, seed):
    g = torch.Generator().manual_seed(seed)
    lat = torch.randn(B, Cin, Fr, Hh, Ww, generator=g).bfloat16().cuda()
    ctx = torch.randn(B, C, T, generator=g).bfloat16().cuda()
    cm = torch.ones(B, C, dtype=torch.bool, device="cuda")
    cm[-1, C - 3:] = False
    t = torch.full((B,), 500.0).bfloat16()
    return lat, ctx, cm, t


def test_config2_full_depth():
    """Config 2: the 30-block backbone prefill, batch 1, 2 views x 5 frames x 16 x 11
    patches (1760 tokens), 64 context tokens."""
    vid, cfg = _backbone(3072, 24, 128, 14336, 4096, 30, 48, seed=21)
    lat, ctx, cm, t = _inputs(1, 48, 5, 32, 44, 64, 4096, seed=22)
    ks, vs, hid = vid.prefill(lat, t, ctx, cm, return_hidden=True)
    ks = {l: ks[l].clone() for l in (0, 14, 29)}
    vs = {l: vs[l].clone() for l in (0, 14, 29)}
    hid = hid.clone()
    torch.cuda.synchronize()
    rk, rv, rh = _backbone_oracle(vid, cfg, lat, t, ctx, cm)
    for l in (0, 14, 29):
        _check(f"config2 K[{l}]", ks[l], rk[l])
        _check(f"config2 V[{l}]", vs[l], rv[l])
    _check("config2 final hidden", hid, rh)


def test_config4_full_width():
    """Config 4: backbone (config-2 widths, 2 blocks) -> config-0 compact expert over its
    final token states -> Action-VAE decode, batch 2 in micro-batches of 1."""
    vid, vcfg = _backbone(3072, 24, 128, 14336, 4096, 2, 48, seed=31)
    torch.manual_seed(32)
    exp = M.ActionDiT(hidden_dim=32, action_dim=16, ffn_dim=128, text_dim=3072, freq_dim=256, eps=1e-6,
                      num_heads=4, attn_head_dim=8, num_layers=8)
    ae = M.ActionAE(M.ActionAEConfig(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16,
                                     decoder_hidden=256, video_cond_dim=0))
    B = 2
    lat, ctx, cm, t = _inputs(B, 48, 5, 32, 44, 64, 4096, seed=33)
    noise = R.seeded_noise(range(B), (8, 16))
    pipe = P.CAEPipeline(vid, exp.cuda(), ae.cuda(), num_steps=4, shift=1.0, micro_batch=1)
    got = pipe(lat, t, ctx, cm, noise.cuda()).cpu()
    _, _, hidden = _backbone_oracle(vid, vcfg, lat, t, ctx, cm)
    ecfg = O.DiTConfig(hidden_dim=32, ffn_dim=128, num_heads=4, attn_head_dim=8, num_layers=8, text_dim=3072,
                       action_dim=16)
    esd = {k: v.float().cpu() for k, v in exp.state_dict().items()}
    dsd = {k: v.float().cpu() for k, v in ae.state_dict().items()}
    ref = O.cae_chunk(esd, ecfg, dsd, O.DecoderConfig(7, 32, 8, 16, 256), noise, hidden.cpu(),
                      num_steps=4, shift=1.0)
    assert got.shape == ref.shape == (B, 32, 7)
    _check("config4 decoded chunks (B=2)", got, ref)


@pytest.mark.parametrize("compact", [False, True])
def test_config3_full_width(compact):
    """Config 3: backbone features after the first of 2 blocks at DiT4DiT widths (3520 tokens), then
    the wide bf16 head (16 x 29 chunk) or the compact fp32 head + Action-VAE (8 x 48 latents
    -> 16 x 29), 4 Euler steps, batch 1."""
    D, H, hd, F, T, L, Cin = 2048, 16, 128, 8192, 4096, 2, 48
    vid, _ = _backbone(D, H, hd, F, T, L, Cin, seed=41)
    torch.manual_seed(42)
    if compact:
        head = M.ActionDiT(hidden_dim=32, action_dim=48, ffn_dim=128, text_dim=D, freq_dim=256, eps=1e-6,
                           num_heads=4, attn_head_dim=8, num_layers=2)
        ae = M.ActionAE(M.ActionAEConfig(action_dim=29, action_horizon=16, num_tokens=8, latent_dim=48,
                                         decoder_hidden=256, video_cond_dim=0))
        Sa, A = 8, 48
    else:
        head = M.ActionDiT(hidden_dim=1024, action_dim=29, ffn_dim=4096, text_dim=D, freq_dim=256, eps=1e-6,
                           num_heads=16, attn_head_dim=64, num_layers=2).to(torch.bfloat16)
        ae, Sa, A = None, 16, 29
    lat, ctx, cm, t = _inputs(1, Cin, 4, 44, 80, 64, T, seed=43)
    noise = torch.randn(1, Sa, A, generator=torch.Generator().manual_seed(44))
    k = 0  # features after block 0 (the elided tail: block 1)
    pipe = P.DiT4DiTPipeline(vid, head.cuda(), extract_layer=k, ae=ae.cuda() if ae is not None else None,
                             num_steps=4, shift=1.0, micro_batch=1)
    got = pipe(lat, t, ctx, cm, noise.cuda()).cpu()
    vcfg = O.DiTConfig(hidden_dim=D, ffn_dim=F, num_heads=H, attn_head_dim=hd, num_layers=k + 1, text_dim=T,
                       in_dim=Cin, out_dim=Cin)
    _, _, feats = _backbone_oracle(pipe.backbone, vcfg, lat, t, ctx, cm)
    hcfg = O.DiTConfig(hidden_dim=head.hidden_dim, ffn_dim=head.ffn_dim, num_heads=head.num_heads,
                       attn_head_dim=head.attn_head_dim, num_layers=head.num_layers, text_dim=D, action_dim=A)
    hsd = {kk: v.float().cpu() for kk, v in head.state_dict().items()}
    ts, ds = O.build_inference_schedule(4, 1.0, dtype=torch.float32)
    x = noise.clone()
    feats = feats.cpu()
    with torch.no_grad():
        for tt, dd in zip(ts, ds):
            x = O.scheduler_step(O.action_forward(hsd, hcfg, x, tt.reshape(1), feats), dd, x)
    ref = x
    if ae is not None:
        ref = O.action_decode({kk: v.float().cpu() for kk, v in ae.state_dict().items()},
                              O.DecoderConfig(29, 16, 8, 48, 256), x)
    assert got.shape == ref.shape
    _check(f"config3 {'compact head + decode' if compact else 'wide head'}", got, ref)
