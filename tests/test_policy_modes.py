"""FastWAMOptionalIDM.infer_action's mode checks (fastwam_optional_idm.py): an unknown
action_infer_mode and the IDM mode without num_latent_frames raise ValueError before
any device work.  CPU only."""
import importlib

import pytest
import torch

M = importlib.import_module("faster-action-models_b200.models")
P = importlib.import_module("faster-action-models_b200.pipeline")


def _policy():
    kw = dict(freq_dim=256, eps=1e-6, num_heads=2, attn_head_dim=32, num_layers=2)
    vid = M.WanVideoDiT(hidden_dim=64, in_dim=16, ffn_dim=128, out_dim=16, text_dim=96, patch_size=(1, 2, 2),
                        has_image_input=False, seperated_timestep=True,
                        video_attention_mask_mode="first_frame_causal", **kw)
    act = M.ActionDiT(hidden_dim=64, action_dim=7, ffn_dim=128, text_dim=96, **kw)
    return P.FastWAMOptionalIDMPolicy(vid, act)


def test_unknown_mode_raises():
    pol = _policy()
    with pytest.raises(ValueError, match="action_infer_mode"):
        pol.infer_action(torch.zeros(1, 16, 1, 8, 12), torch.zeros(1, 4, 96), torch.ones(1, 4, dtype=torch.bool),
                         action_horizon=8, action_infer_mode="joint")


def test_idm_mode_needs_frame_count():
    pol = _policy()
    with pytest.raises(ValueError, match="num_latent_frames"):
        pol.infer_action(torch.zeros(1, 16, 1, 8, 12), torch.zeros(1, 4, 96), torch.ones(1, 4, dtype=torch.bool),
                         action_horizon=8, action_infer_mode="idm")
