"""torch.library operators (fam::*) mirror the reference's custom-op boundary
(torch.library.custom_op + register_fake): they are registered, their fake
implementations give the output shapes / dtypes without running a kernel, and an
unknown handle fails loudly.  CPU only: FakeTensorMode, no libfam call."""
import importlib

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

M = importlib.import_module("faster-action-models_b200.models")
T = importlib.import_module("faster-action-models_b200.torch_ops")


def test_operators_registered():
    for name in ("prefill_video_cache", "denoise_action_with_video_cache", "action_chunk", "action_decode"):
        assert hasattr(torch.ops.fam, name), name


def test_fake_shapes():
    act = M.ActionDiT(64, 7, 128, 96, 256, 1e-6, 2, 32, 2)
    vid = M.WanVideoDiT(hidden_dim=64, in_dim=16, ffn_dim=128, out_dim=16, text_dim=96, freq_dim=256, eps=1e-6,
                        patch_size=(1, 2, 2), num_heads=2, attn_head_dim=32, num_layers=2, has_image_input=False,
                        seperated_timestep=True, video_attention_mask_mode="first_frame_causal")
    ae = M.ActionAE(M.ActionAEConfig(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16,
                                     decoder_hidden=64, video_cond_dim=0, variational=True))
    ha, hv, he = T.register(act), T.register(vid), T.register(ae)
    try:
        with FakeTensorMode():
            lat_v = torch.empty(1, 16, 3, 8, 12, dtype=torch.bfloat16)
            ctx = torch.empty(1, 10, 96, dtype=torch.bfloat16)
            kv = torch.ops.fam.prefill_video_cache(hv, lat_v, [0.0], ctx, None)
            assert len(kv) == 4 and all(t.shape == (1, 72, 64) and t.dtype == torch.bfloat16 for t in kv)
            lat_a = torch.empty(1, 8, 7, dtype=torch.bfloat16)
            mask = torch.ones(8, 80, dtype=torch.bool)
            vel = torch.ops.fam.denoise_action_with_video_cache(ha, lat_a, 500.0, ctx, None,
                                                                kv[:2], kv[2:], mask)
            assert vel.shape == (1, 8, 7) and vel.dtype == torch.bfloat16
            out = torch.ops.fam.action_chunk(ha, lat_a, [1000.0, 500.0], [-0.5, -0.5], ctx, None, [], [], None)
            assert out.shape == (1, 8, 7) and out.dtype == torch.bfloat16
            chunk = torch.ops.fam.action_decode(he, torch.empty(2, 8, 16), None)
            assert chunk.shape == (2, 32, 7) and chunk.dtype == torch.float32
            with pytest.raises(ValueError):  # a handle of another module kind
                torch.ops.fam.action_decode(ha, torch.empty(2, 8, 16), None)
    finally:
        for h in (ha, hv, he):
            T.unregister(h)


def test_unknown_handle_and_bad_module():
    with pytest.raises(ValueError):
        torch.ops.fam.action_decode(12345, torch.zeros(1, 8, 16), None)
    with pytest.raises(TypeError):
        T.register(torch.nn.Linear(2, 2))
