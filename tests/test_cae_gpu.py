"""Compact action expert + Action-VAE decoder (BASELINE config 0 family) on the GPU,
checked against the reference's own recorded outputs (golden fixture) and the CPU
oracle at full config-0 size.  fp32 path: tolerance 2e-3 max|d| relative to scale,
cosine >= 0.999 (BASELINE bar 2e-2 / 0.999)."""
import importlib
from pathlib import Path

import pytest
import torch

from oracle import fam_oracle as O

pytestmark = pytest.mark.gpu

M = importlib.import_module("faster-action-models_b200.models")
GOLDEN = Path(__file__).resolve().parent / "golden"


def _close(got, ref, rel=2e-3):
    got, ref = got.float().cpu(), ref.float().cpu()
    err = (got - ref).abs().max().item()
    scale = max(1.0, ref.abs().max().item())
    cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
    assert err <= rel * scale and cos >= 0.999, f"max|d| {err} cos {cos}"


def test_c0_golden_chunk_and_decode():
    fx = torch.load(GOLDEN / "c0_cae_expert.pt", weights_only=False)
    dit = M.ActionDiT(**fx["dit_cfg"])
    dit.load_state_dict({k: v.float() for k, v in fx["dit"].items()})
    dit = dit.cuda()
    assert dit.is_compact()
    eng = dit.engine()
    ts, ds = fx["timesteps"].tolist(), fx["deltas"].tolist()
    lat, trace = eng.chunk(fx["noise"].cuda(), ts, ds, fx["context"].float().cuda(), return_trace=True)
    torch.cuda.synchronize()
    _close(trace, fx["velocities"])
    _close(lat, fx["latent"])
    c = fx["dec_cfg"]
    ae = M.ActionAE(M.ActionAEConfig(action_dim=c["action_dim"], action_horizon=c["action_horizon"],
                                     num_tokens=c["num_tokens"], latent_dim=c["latent_dim"],
                                     decoder_hidden=c["decoder_hidden"], video_cond_dim=0,
                                     variational=True))
    ae.load_state_dict({k: v.float() for k, v in fx["ae"].items()})
    ae = ae.cuda()
    chunk = ae.decode(fx["latent"].cuda())
    torch.cuda.synchronize()
    _close(chunk, fx["chunk"])


def test_full_config0_chunk():
    """hidden 32, 4x8 heads, 8 blocks, ctx 512 x 3072, 4 steps (shift 1), decoder hidden 256."""
    torch.manual_seed(0)
    dit = M.ActionDiT(hidden_dim=32, action_dim=16, ffn_dim=128, text_dim=3072, freq_dim=256,
                      eps=1e-6, num_heads=4, attn_head_dim=8, num_layers=8)
    cfg = O.DiTConfig(hidden_dim=32, ffn_dim=128, num_heads=4, attn_head_dim=8, num_layers=8,
                      text_dim=3072, action_dim=16)
    ae = M.ActionAE(M.ActionAEConfig(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16,
                                     decoder_hidden=256, video_cond_dim=0, variational=True))
    g = torch.Generator().manual_seed(0)
    ctx = torch.randn(1, 512, 3072, generator=g)
    noise = torch.randn(1, 8, 16, generator=g)
    sd = {k: v.float() for k, v in dit.state_dict().items()}
    dsd = {k: v.float() for k, v in ae.state_dict().items()}
    ref_chunk, ref_lat, _ = O.cae_chunk(sd, cfg, dsd, O.DecoderConfig(7, 32, 8, 16, 256), noise, ctx,
                                        num_steps=4, shift=1.0, return_trace=True)
    dit, ae = dit.cuda(), ae.cuda()
    ts, ds = M.build_inference_schedule(4, 1.0, dtype=torch.float32)
    lat = dit.engine().chunk(noise.cuda(), ts, ds, ctx.cuda())
    chunk = ae.decode(lat)
    torch.cuda.synchronize()
    _close(lat, ref_lat)
    _close(chunk, ref_chunk)


@pytest.mark.parametrize("horizon,tokens,hidden,suites", [(32, 8, 128, 0), (16, 8, 48, 3), (24, 8, 64, 0)])
def test_decoder_strides_and_suites(horizon, tokens, hidden, suites):
    torch.manual_seed(horizon + hidden)
    cfg = M.ActionAEConfig(action_dim=7, action_horizon=horizon, num_tokens=tokens, latent_dim=16,
                           decoder_hidden=hidden, video_cond_dim=0, num_suites=suites)
    ae = M.ActionAE(cfg)
    with torch.no_grad():
        for p in ae.parameters():
            p.add_(0.05 * torch.randn_like(p))  # non-trivial norms / suite embeddings
    z = torch.randn(3, tokens, 16)
    sid = torch.tensor([0, 2, 1]) if suites else None
    dsd = {k: v.float() for k, v in ae.state_dict().items()}
    ref = O.action_decode(dsd, O.DecoderConfig(7, horizon, tokens, 16, hidden, suites), z, sid)
    got = ae.cuda().decode(z.cuda(), sid.cuda() if sid is not None else None)
    torch.cuda.synchronize()
    _close(got, ref)


# (hidden, heads, head_dim, ffn, layers, tokens S, context C, batch, steps, masked)
# covers: several key chunks with a ragged last chunk (C=600, C=77), query rows
# that do not fill the 16-row tensor-core tile (S=6), head_dim 4/8/16, odd depth,
# a single block, more Euler steps than one t_mod batch (10), per-sample context
# masks, and shapes that take the unstaged kernel (hidden 64 with ffn 256, and
# 32 action tokens).
CAE_SHAPES = [
    (32, 4, 8, 128, 3, 6, 600, 2, 10, True),
    (16, 4, 4, 64, 1, 8, 16, 3, 5, True),
    (32, 2, 16, 64, 2, 16, 77, 1, 3, False),
    (64, 4, 16, 256, 2, 8, 40, 2, 2, True),
    (32, 4, 8, 128, 2, 32, 64, 1, 2, False),
]


@pytest.mark.parametrize("D,H,hd,F,L,S,C,B,N,masked", CAE_SHAPES)
def test_cae_shapes_vs_oracle(D, H, hd, F, L, S, C, B, N, masked):
    torch.manual_seed(D * 7 + L)
    T, A = 64, 16
    dit = M.ActionDiT(hidden_dim=D, action_dim=A, ffn_dim=F, text_dim=T, freq_dim=256, eps=1e-6,
                      num_heads=H, attn_head_dim=hd, num_layers=L)
    with torch.no_grad():
        for p in dit.parameters():
            p.add_(0.05 * torch.randn_like(p))  # non-zero AdaLN modulation / gates
    assert dit.is_compact()
    cfg = O.DiTConfig(hidden_dim=D, ffn_dim=F, num_heads=H, attn_head_dim=hd, num_layers=L,
                      text_dim=T, action_dim=A)
    g = torch.Generator().manual_seed(C + S)
    ctx = torch.randn(B, C, T, generator=g)
    noise = torch.randn(B, S, A, generator=g)
    mask = None
    if masked:
        mask = torch.rand(B, C, generator=g) > 0.3
        mask[:, 0] = True  # no fully masked sample (the reference softmax is undefined there)
    sd = {k: v.float() for k, v in dit.state_dict().items()}
    ts, ds = O.build_inference_schedule(N, 3.0, dtype=torch.float32)
    x, vel = noise.clone(), []
    for t, d in zip(ts, ds):
        v = O.action_forward(sd, cfg, x, t.reshape(1), ctx, mask)
        vel.append(v)
        x = O.scheduler_step(v, d, x)
    eng = dit.cuda().engine()
    lat, trace = eng.chunk(noise.cuda(), ts.tolist(), ds.tolist(), ctx.cuda(),
                           mask.cuda() if mask is not None else None, return_trace=True)
    torch.cuda.synchronize()
    assert eng.status() == 0
    _close(trace, torch.stack(vel))
    _close(lat, x)


def test_chunk_decode_in_step_kernel_epilogue():
    """fam_cae_chunk_decode: the Action-VAE decode in the staged step kernel's epilogue.
    The config-0 golden (one-CTA cluster) and full config 0 (512-key context: a 4-CTA
    cluster splitting the 256 decoder channels, decode="fused") give the reference's / the
    oracle's chunk and the same chunk as the separate decoder launches; decode="auto"
    leaves batch 2 to the separate launches; a decoder with two upsampling stages
    takes the separate launches (decode_fused False) with the same result."""
    fx = torch.load(GOLDEN / "c0_cae_expert.pt", weights_only=False)
    dit = M.ActionDiT(**fx["dit_cfg"])
    dit.load_state_dict({k: v.float() for k, v in fx["dit"].items()})
    dit = dit.cuda()
    c = fx["dec_cfg"]
    ae = M.ActionAE(M.ActionAEConfig(action_dim=c["action_dim"], action_horizon=c["action_horizon"],
                                     num_tokens=c["num_tokens"], latent_dim=c["latent_dim"],
                                     decoder_hidden=c["decoder_hidden"], video_cond_dim=0, variational=True))
    ae.load_state_dict({k: v.float() for k, v in fx["ae"].items()})
    ae = ae.cuda()
    eng = dit.engine()
    ts, ds = fx["timesteps"].tolist(), fx["deltas"].tolist()
    lat, chunk = eng.chunk_decode(fx["noise"].cuda(), ts, ds, fx["context"].float().cuda(), ae, decode="fused")
    torch.cuda.synchronize()
    assert eng.decode_fused
    _close(lat, fx["latent"])
    _close(chunk, fx["chunk"])

    torch.manual_seed(0)
    dit = M.ActionDiT(hidden_dim=32, action_dim=16, ffn_dim=128, text_dim=3072, freq_dim=256,
                      eps=1e-6, num_heads=4, attn_head_dim=8, num_layers=8)
    cfg = O.DiTConfig(hidden_dim=32, ffn_dim=128, num_heads=4, attn_head_dim=8, num_layers=8,
                      text_dim=3072, action_dim=16)
    ae = M.ActionAE(M.ActionAEConfig(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16,
                                     decoder_hidden=256, video_cond_dim=0, variational=True))
    g = torch.Generator().manual_seed(0)
    ctx = torch.randn(2, 512, 3072, generator=g)
    noise = torch.randn(2, 8, 16, generator=g)
    sd = {k: v.float() for k, v in dit.state_dict().items()}
    dsd = {k: v.float() for k, v in ae.state_dict().items()}
    ref_chunk = O.cae_chunk(sd, cfg, dsd, O.DecoderConfig(7, 32, 8, 16, 256), noise, ctx, num_steps=4, shift=1.0)
    dit, ae = dit.cuda(), ae.cuda()
    ts, ds = M.build_inference_schedule(4, 1.0, dtype=torch.float32)
    eng = dit.engine()
    for _ in range(2):  # a second call finds the first one's leftovers in the staging buffers
        lat, chunk = eng.chunk_decode(noise.cuda(), ts, ds, ctx.cuda(), ae, decode="fused")
        torch.cuda.synchronize()
        assert eng.decode_fused
        _close(chunk, ref_chunk)
        _close(chunk, ae.decode(lat))
    # batch 2: decode="auto" leaves the decode to the separate launches
    lat_a, chunk_a = eng.chunk_decode(noise.cuda(), ts, ds, ctx.cuda(), ae)
    torch.cuda.synchronize()
    assert not eng.decode_fused
    _close(chunk_a, ref_chunk)
    # batch 4: decode="auto" decodes in the epilogue, same chunks as the separate launches
    g4 = torch.Generator().manual_seed(4)
    ctx4, noise4 = torch.randn(4, 512, 3072, generator=g4).cuda(), torch.randn(4, 8, 16, generator=g4).cuda()
    lat4, chunk4 = eng.chunk_decode(noise4, ts, ds, ctx4, ae)
    torch.cuda.synchronize()
    assert eng.decode_fused
    _, chunk4s = eng.chunk_decode(noise4, ts, ds, ctx4, ae, decode="separate")
    torch.cuda.synchronize()
    assert not eng.decode_fused
    _close(chunk4, chunk4s)
    _close(chunk4, ae.decode(lat4))

    ae2 = M.ActionAE(M.ActionAEConfig(action_dim=7, action_horizon=64, num_tokens=8, latent_dim=16,
                                      decoder_hidden=64, video_cond_dim=0, variational=True)).cuda()
    lat2, chunk2 = eng.chunk_decode(noise.cuda(), ts, ds, ctx.cuda(), ae2)
    torch.cuda.synchronize()
    assert not eng.decode_fused  # 64 / 8 = strides 4 and 2, two upsampling stages: separate launches
    _close(chunk2, ae2.decode(lat2))
