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
