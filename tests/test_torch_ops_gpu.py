"""fam::* operators on the GPU: each returns what the engine call it wraps returns
(the same kernels; compared at the parity tolerance), the fake implementations agree with the real
outputs' shapes and dtypes, and the action step traces into a torch.compile
fullgraph region (aot_eager backend) with the same result."""
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu

M = importlib.import_module("faster-action-models_b200.models")
T = importlib.import_module("faster-action-models_b200.torch_ops")


def _close(got, ref):
    err = (got.float() - ref.float()).abs().max().item()
    assert err <= 2e-2 * max(1.0, ref.float().abs().max().item()), err


def _models():
    torch.manual_seed(3)
    act = M.ActionDiT(64, 7, 128, 96, 256, 1e-6, 2, 128, 2).to("cuda", torch.bfloat16)
    vid = M.WanVideoDiT(hidden_dim=256, in_dim=16, ffn_dim=512, out_dim=16, text_dim=96, freq_dim=256, eps=1e-6,
                        patch_size=(1, 2, 2), num_heads=2, attn_head_dim=128, num_layers=2, has_image_input=False,
                        seperated_timestep=True, video_attention_mask_mode="first_frame_causal")
    vid = vid.to("cuda", torch.bfloat16)
    ae = M.ActionAE(M.ActionAEConfig(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=7,
                                     decoder_hidden=64, video_cond_dim=0, variational=True)).cuda()
    return act, vid, ae


def test_operators_match_engine_calls():
    act, vid, ae = _models()
    ha, hv, he = T.register(act), T.register(vid), T.register(ae)
    try:
        g = torch.Generator().manual_seed(4)
        lat_v = torch.randn(1, 16, 3, 8, 12, generator=g).bfloat16().cuda()
        ctx = torch.randn(1, 10, 96, generator=g).bfloat16().cuda()
        cm = torch.ones(1, 10, dtype=torch.bool, device="cuda")
        t0 = torch.zeros(1)
        kv = torch.ops.fam.prefill_video_cache(hv, lat_v, [0.0], ctx, cm)
        k_ref, v_ref = vid.prefill(lat_v, t0, ctx, cm)
        assert all(torch.equal(a, b) for a, b in zip(kv, list(k_ref) + list(v_ref)))
        ck, cv = [k.clone() for k in kv[:2]], [v.clone() for v in kv[2:]]
        Sv = ck[0].shape[1]
        lat_a = torch.randn(1, 8, 7, generator=g).bfloat16().cuda()
        mask = torch.ones(8, Sv + 8, dtype=torch.bool, device="cuda")
        t = 750.0  # a host scalar: the operators never read the device back
        vel = torch.ops.fam.denoise_action_with_video_cache(ha, lat_a, t, ctx, cm, ck, cv, mask)
        ref = act.engine().denoise_step(lat_a, t, ctx, cm, ck, cv, mask)
        assert vel.shape == (1, 8, 7) and vel.dtype == torch.bfloat16
        _close(vel, ref)

        def step(x):
            return torch.ops.fam.denoise_action_with_video_cache(ha, x, t, ctx, cm, ck, cv, mask)

        compiled = torch.compile(step, fullgraph=True, backend="aot_eager")
        _close(compiled(lat_a), ref)
        ts, ds = M.build_inference_schedule(3, 5.0, dtype=torch.bfloat16)
        tsf, dsf = [float(x) for x in ts], [float(x) for x in ds]
        out = torch.ops.fam.action_chunk(ha, lat_a, tsf, dsf, ctx, cm, ck, cv, mask)
        _close(out, act.engine().chunk(lat_a, tsf, dsf, ctx, cm, ck, cv, mask))
        chunk = torch.ops.fam.action_decode(he, out.float(), None)
        assert chunk.shape == (1, 32, 7) and chunk.dtype == torch.float32
        _close(chunk, ae.decode(out.float()))
    finally:
        for h in (ha, hv, he):
            T.unregister(h)
