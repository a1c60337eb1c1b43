"""Video DiT prefill (BASELINE config 2 family) through fam_video_prefill vs the oracle
(WanVideoDiT.prepare + MoT.prefill_video_cache_tensor restated) in fp32 on the same bf16
weights.  Per-block K/V and the final token states: max|d| <= 2e-2 x max(1, max|ref|),
cosine >= 0.999."""
import importlib

import pytest
import torch

from oracle import fam_oracle as O

pytestmark = pytest.mark.gpu

M = importlib.import_module("faster-action-models_b200.models")


def _check(got, ref, name):
    got, ref = got.float().cpu(), ref.float().cpu()
    err = (got - ref).abs().max().item()
    scale = max(1.0, ref.abs().max().item())
    cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
    assert err <= 2e-2 * scale and cos >= 0.999, f"{name}: max|d| {err} (scale {scale}) cos {cos}"


def _run(D, H, hd, F, T, L, Cin, B, Fr, Hh, Ww, C, ref_device, seed=0):
    torch.manual_seed(seed)
    dit = M.WanVideoDiT(hidden_dim=D, in_dim=Cin, ffn_dim=F, out_dim=Cin, text_dim=T, freq_dim=256,
                        eps=1e-6, patch_size=(1, 2, 2), num_heads=H, attn_head_dim=hd,
                        num_layers=L, has_image_input=False, seperated_timestep=True,
                        video_attention_mask_mode="first_frame_causal")
    with torch.no_grad():
        for n, p in dit.named_parameters():
            if "norm" in n:
                p.copy_(1.0 + 0.2 * torch.randn_like(p))
    dit = dit.to(torch.bfloat16)
    cfg = O.DiTConfig(hidden_dim=D, ffn_dim=F, num_heads=H, attn_head_dim=hd, num_layers=L,
                      text_dim=T, in_dim=Cin, out_dim=Cin)
    g = torch.Generator().manual_seed(seed + 1)
    lat = torch.randn(B, Cin, Fr, Hh, Ww, generator=g).bfloat16()
    ctx = torch.randn(B, C, T, generator=g).bfloat16()
    cm = torch.ones(B, C, dtype=torch.bool)
    cm[-1, C - 2:] = False
    t = torch.full((B,), 500.0).bfloat16()
    sd = {k: v.float().to(ref_device) for k, v in dit.state_dict().items()}
    with torch.no_grad():
        tok, _, tmod, cemb, cmask, freqs, (f, h, w), tpf = O.video_prepare(
            sd, cfg, lat.float().to(ref_device), t.float().to(ref_device), ctx.float().to(ref_device),
            cm.to(ref_device))
        vmask = O.build_video_to_video_mask(tok.shape[1], tpf).to(ref_device)
        rk, rv, rh = O.prefill_video_cache(sd, cfg, tok, freqs.to(ref_device), tmod, cemb, cmask,
                                           vmask, return_hidden=True)
    dit = dit.cuda()
    ks, vs, hid = dit.prefill(lat.cuda(), t, ctx.cuda(), cm.cuda(), return_hidden=True)
    ks2, vs2 = dit.prefill(lat.cuda(), t, ctx.cuda(), cm.cuda())  # cache only (last block short)
    torch.cuda.synchronize()
    for l in range(L):
        _check(ks[l], rk[l], f"K[{l}]")
        _check(vs[l], rv[l], f"V[{l}]")
        assert torch.equal(ks[l], ks2[l]) and torch.equal(vs[l], vs2[l])
    _check(hid, rh, "hidden")
    return dit


def test_small_prefill_cpu_oracle():
    _run(D=256, H=2, hd=128, F=512, T=64, L=2, Cin=16, B=2, Fr=3, Hh=8, Ww=12, C=10, ref_device="cpu")


def test_config2_width_two_blocks():
    """Full config-2 widths (3072 hidden, 24x128 heads, FFN 14336, 48 latent channels,
    2 views x 5 frames x 16x11 patches = 1760 tokens, 64 context tokens), two blocks; the
    oracle runs in fp32 on the GPU (torch) with TF32 off."""
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    _run(D=3072, H=24, hd=128, F=14336, T=4096, L=2, Cin=48, B=1, Fr=5, Hh=32, Ww=44, C=64,
         ref_device="cuda")


def test_per_block_cross_kv_layout_matches_stacked():
    """Blocks whose cross K/V projections are separate allocations take the per-block
    context GEMMs; the caches equal those of the stacked (one GEMM) layout."""
    dit = _run(D=256, H=2, hd=128, F=512, T=64, L=3, Cin=16, B=2, Fr=3, Hh=8, Ww=12, C=10, ref_device="cpu",
               seed=5)
    g = torch.Generator().manual_seed(9)
    lat = torch.randn(2, 16, 3, 8, 12, generator=g).bfloat16().cuda()
    ctx = torch.randn(2, 10, 64, generator=g).bfloat16().cuda()
    cm = torch.ones(2, 10, dtype=torch.bool, device="cuda")
    t = torch.full((2,), 300.0).bfloat16()
    ks, vs = dit.prefill(lat, t, ctx, cm)
    ks = [k.clone() for k in ks]
    vs = [v.clone() for v in vs]
    eng = M.VideoPrefillEngine(dit, stack_cross_kv=False)
    ks2, vs2 = eng.prefill(lat, t, ctx, cm)
    torch.cuda.synchronize()
    for l in range(3):
        _check(ks2[l], ks[l], f"K[{l}] per-block")
        _check(vs2[l], vs[l], f"V[{l}] per-block")
