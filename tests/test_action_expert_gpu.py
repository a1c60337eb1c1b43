"""Action expert (ActionDiT over a video K/V cache) through the C ABI vs the CPU oracle.

Tolerances: per model evaluation, max|d| <= 2e-2 * max(1, max|ref|) and cosine >= 0.999
against the fp32 oracle on the same bf16 weights.  For a whole multi-step chunk the
reference's own bf16 arithmetic drifts from fp32 (measured 5.7e-2 max|d| at full BASELINE
config 1 size), so the chunk gate is cosine >= 0.999 and max|d| within 2 x the oracle's
bf16-vs-fp32 disagreement on the same inputs (the calibration rule of the reference's
numerics oracle, geak/task/scripts/episode_oracle.py:145-199), and never above 0.1.
"""
import importlib

import pytest
import torch

from oracle import fam_oracle as O

pytestmark = pytest.mark.gpu

M = importlib.import_module("faster-action-models_b200.models")


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.float().flatten(), b.float().flatten(), dim=0).item()


def _build(D=256, H=4, hd=64, F=512, T=128, L=2, A=7, seed=0):
    torch.manual_seed(seed)
    dit = M.ActionDiT(hidden_dim=D, action_dim=A, ffn_dim=F, text_dim=T, freq_dim=256, eps=1e-6,
                      num_heads=H, attn_head_dim=hd, num_layers=L)
    with torch.no_grad():  # random affine norms / RMS weights so every parameter matters
        for n, p in dit.named_parameters():
            if "norm" in n:
                p.copy_(1.0 + 0.2 * torch.randn_like(p))
    dit = dit.to(torch.bfloat16)
    sd = {k: v.float() for k, v in dit.state_dict().items()}
    cfg = O.DiTConfig(hidden_dim=D, ffn_dim=F, num_heads=H, attn_head_dim=hd, num_layers=L,
                      text_dim=T, action_dim=A)
    return dit.cuda(), sd, cfg


def _inputs(B, Sa, Sv, C, T, D_attn, L, tpf, A=7, seed=1):
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randn(B, C, T, generator=g).bfloat16()
    cm = torch.ones(B, C, dtype=torch.bool)
    if C > 4:
        cm[-1, C - 3:] = False
    ck = [torch.randn(B, Sv, D_attn, generator=g).bfloat16() for _ in range(L)]
    cv = [torch.randn(B, Sv, D_attn, generator=g).bfloat16() for _ in range(L)]
    noise = torch.randn(B, Sa, A, generator=g).bfloat16()
    mask = O.build_mot_attention_mask(Sv, Sa, tpf)[Sv:, :]
    return ctx, cm, ck, cv, noise, mask


@pytest.mark.parametrize("B,Sa,Sv,C,tpf", [(1, 32, 200, 16, 50), (2, 8, 130, 9, 130), (3, 32, 0, 12, 1)])
def test_denoise_step_matches_oracle(B, Sa, Sv, C, tpf):
    dit, sd, cfg = _build()
    ctx, cm, ck, cv, noise, mask = _inputs(B, Sa, Sv, C, cfg.text_dim, 256, cfg.num_layers, tpf)
    t = torch.tensor([936.0]).bfloat16()
    if Sv == 0:
        mask = torch.ones(Sa, Sa, dtype=torch.bool)
    ref = O.denoise_action_with_video_cache(sd, cfg, noise.float(), t.float(), ctx.float(), cm,
                                            [k.float() for k in ck], [v.float() for v in cv], mask)
    eng = dit.engine()
    got = eng.denoise_step(noise.cuda(), t, ctx.cuda(), cm.cuda(), [k.cuda() for k in ck],
                           [v.cuda() for v in cv], mask.cuda()).cpu()
    err = (got.float() - ref).abs().max().item()
    scale = max(1.0, ref.abs().max().item())
    assert err <= 2e-2 * scale, f"max|d| {err} (scale {scale})"
    assert _cos(got, ref) >= 0.999


def test_chunk_matches_oracle_and_is_deterministic():
    dit, sd, cfg = _build(seed=3)
    B, Sa, Sv, C, tpf = 2, 32, 192, 16, 48
    ctx, cm, ck, cv, noise, mask = _inputs(B, Sa, Sv, C, cfg.text_dim, 256, cfg.num_layers, tpf)
    ts, ds = M.build_inference_schedule(4, 5.0)
    ref32 = O.action_chunk_with_cache(sd, cfg, noise.float(), ctx.float(), cm, [k.float() for k in ck],
                                      [v.float() for v in cv], mask, 4, 5.0)
    eng = dit.engine()
    args = (noise.cuda(), ts, ds, ctx.cuda(), cm.cuda(), [k.cuda() for k in ck], [v.cuda() for v in cv],
            mask.cuda())
    got, trace = eng.chunk(*args, return_trace=True, use_graph=False)
    got_g = eng.chunk(*args, use_graph=True)
    got_g2 = eng.chunk(*args, use_graph=True)  # graph replay
    torch.cuda.synchronize()
    assert torch.equal(got, got_g) and torch.equal(got_g, got_g2), "graph / eager / replay differ"
    err = (got.cpu().float() - ref32).abs().max().item()
    assert err <= 2e-2 * max(1.0, ref32.abs().max().item()), err
    assert _cos(got.cpu(), ref32) >= 0.999
    assert trace.shape == (4, B, Sa, 7)


@pytest.mark.parametrize("Sa,Sv,C,tpf", [(32, 200, 16, 50), (8, 97, 5, 97), (20, 300, 64, 60)])
def test_fused_kernel_matches_chain_and_oracle(Sa, Sv, C, tpf):
    """The fused persistent chunk kernel (batch 1) against the launch chain and the oracle
    (hidden 512 = two 256-wide halves per CTA pair, 8 heads)."""
    dit, sd, cfg = _build(D=512, H=8, F=1024, seed=11)
    ctx, cm, ck, cv, noise, mask = _inputs(1, Sa, Sv, max(C, 1), cfg.text_dim, 512, cfg.num_layers, tpf)
    ctx = ctx[:, :C] if C else ctx[:, :0]
    cm = cm[:, :C] if C else cm[:, :0]
    ts, ds = M.build_inference_schedule(3, 5.0)
    ref = O.action_chunk_with_cache(sd, cfg, noise.float(), ctx.float(), cm, [k.float() for k in ck],
                                    [v.float() for v in cv], mask, 3, 5.0)
    eng = dit.engine()
    args = (noise.cuda(), ts, ds, ctx.cuda(), cm.cuda(), [k.cuda() for k in ck], [v.cuda() for v in cv],
            mask.cuda())
    eng.set_mode("chain")
    got_c = eng.chunk(*args).cpu().float()
    assert eng.last_path() == "chain"
    eng.set_mode("fused")
    got_f, trace = eng.chunk(*args, return_trace=True)
    got_f = got_f.cpu().float()
    assert eng.last_path() == "fused" and eng.launch_count() < 100
    got_f2 = eng.chunk(*args).cpu().float()  # graph replay of the fused chunk
    eng.set_mode("auto")
    for got in (got_c, got_f, got_f2):
        err = (got - ref).abs().max().item()
        assert err <= 2e-2 * max(1.0, ref.abs().max().item()) and _cos(got, ref) >= 0.999, err
    assert (got_f - got_c).abs().max().item() <= 2e-2
    assert trace.shape == (3, 1, Sa, 7)


def test_full_config1_chunk():
    """BASELINE config 1 at full size: 1024 hidden, 16x64 heads, 28 blocks, 1760-token cache,
    10 steps, batch 1."""
    D, H, hd, F, T, L = 1024, 16, 64, 4096, 4096, 28
    dit, sd, cfg = _build(D=D, H=H, hd=hd, F=F, T=T, L=L, seed=7)
    B, Sa, Sv, C = 1, 32, 1760, 64
    ctx, cm, ck, cv, noise, _ = _inputs(B, Sa, Sv, C, T, D, L, 1760)
    cm[:] = True
    mask = torch.ones(Sa, Sv + Sa, dtype=torch.bool)  # all-True joint mask
    ts, ds = M.build_inference_schedule(10, 1.0)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ck32, cv32 = [k.float() for k in ck], [v.float() for v in cv]
    ref32 = O.action_chunk_with_cache(sd, cfg, noise.float(), ctx.float(), cm, ck32, cv32, mask, 10, 1.0)
    sd16 = {k: v.bfloat16() for k, v in sd.items()}
    ref16 = O.action_chunk_with_cache(sd16, cfg, noise, ctx, cm, ck, cv, mask, 10, 1.0).float()
    floor = (ref16 - ref32).abs().max().item()
    got = dit.engine().chunk(noise.cuda(), ts, ds, ctx.cuda(), cm.cuda(), [k.cuda() for k in ck],
                             [v.cuda() for v in cv], mask.cuda()).cpu().float()
    err32 = (got - ref32).abs().max().item()
    err16 = (got - ref16).abs().max().item()
    print(f"config1 chunk: max|gpu-fp32|={err32:.4f} max|gpu-bf16ref|={err16:.4f} "
          f"bf16-vs-fp32 floor={floor:.4f} cos={_cos(got, ref32):.6f}")
    assert _cos(got, ref32) >= 0.999 and _cos(got, ref16) >= 0.999
    assert err32 <= min(0.1, max(2e-2, 2 * floor))
    assert err16 <= min(0.1, max(2e-2, 2 * floor))
