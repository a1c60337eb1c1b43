"""FastWAM policy object on the GPU against the reference's own run.

tests/golden/fastwam_infer_action.pt holds FastWAM.infer_action of the reference at small
shapes (VAE encode of the observation, proprio token, video prefill at t = 0, the MoT
action Euler loop, Action-VAE decode; bf16) and the reference checkpoint payload.  The
repository's FastWAM loads that payload through load_checkpoint and reproduces the
decoded chunk: max|d| <= 2e-2 * max(1, max|ref|), cosine >= 0.999.
"""
import importlib
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

M = importlib.import_module("faster-action-models_b200.models")
FW = importlib.import_module("faster-action-models_b200.fastwam")
VAE = importlib.import_module("faster-action-models_b200.vae")
GOLDEN = Path(__file__).resolve().parent / "golden"


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0).item()


def _close(name, got, ref):
    err = (got.float() - ref.float()).abs().max().item()
    c = _cos(got, ref)
    print(f"PARITY {name}: max|d| {err:.4g} cos {c:.6f}")
    assert err <= 2e-2 * max(1.0, ref.abs().max().item()) and c >= 0.999, (name, err, c)


def _model(fx, with_action_vae=True):
    torch.manual_seed(0)
    video = M.WanVideoDiT(**fx["video_cfg"]).to(torch.bfloat16)
    action = M.ActionDiT(**fx["action_cfg"]).to(torch.bfloat16)
    mot = FW.MoT({"video": video, "action": action})
    vc = fx["vae_cfg"]
    vae = VAE.WanVideoVAE38(fx["vae_params"], fx["vae_mean"].float(), 1.0 / fx["vae_inv_std"].float(),
                            z_dim=vc["z_dim"], dim=vc["dim"])
    vae.scale = [fx["vae_mean"].float().cuda(), fx["vae_inv_std"].float().cuda()]  # the reference's bf16 values
    ae = None
    if with_action_vae:
        ae = M.ActionAE(M.ActionAEConfig(**fx["action_vae"]["config"]))
        ae.load_state_dict(fx["action_vae"]["model"])
    model = FW.FastWAM(video, action, mot, vae, text_dim=96, proprio_dim=8, action_vae=ae, device="cuda",
                       torch_dtype=torch.bfloat16, action_infer_shift=fx["action_infer_shift"])
    model.load_checkpoint(fx["checkpoint"])
    return model


def _infer(model, fx, **kw):
    return model.infer_action(prompt=None, input_image=fx["input_image"], action_horizon=fx["action_horizon"],
                              proprio=fx["proprio"], context=fx["context"], context_mask=fx["context_mask"],
                              num_inference_steps=fx["num_inference_steps"], seed=fx["seed"],
                              return_action_latents=True, **kw)


def test_infer_action_reproduces_reference_run():
    fx = torch.load(GOLDEN / "fastwam_infer_action.pt")
    model = _model(fx)
    out = _infer(model, fx)
    assert out["action"].shape == fx["action"].shape and out["action"].device.type == "cpu"
    assert out["action"].dtype == torch.float32
    _close("fastwam infer_action latents", out["action_latents"], fx["action_latents"])
    _close("fastwam infer_action chunk", out["action"], fx["action"])
    # a harness replacing the denoise step on the instance sees every Euler step
    calls = []
    step = model._denoise_action_with_video_cache

    def patched(**kwargs):
        calls.append(kwargs["timestep_action"])
        return step(**kwargs)

    model._denoise_action_with_video_cache = patched
    out2 = _infer(model, fx)
    assert len(calls) == fx["num_inference_steps"]
    _close("fastwam infer_action (per-step replacement)", out2["action"], fx["action"])


def test_infer_action_multi_matches_serial_calls():
    """Batched twin: B distinct observations with per-row seeds reproduce B serial
    infer_action calls (no Action-VAE: both return the action latents)."""
    fx = torch.load(GOLDEN / "fastwam_infer_action.pt")
    model = _model(fx, with_action_vae=False)
    g = torch.Generator().manual_seed(3)
    imgs = torch.cat([fx["input_image"], (torch.rand(1, 3, 64, 96, generator=g) * 2 - 1).bfloat16()])
    ctx = torch.cat([fx["context"], torch.randn(1, *fx["context"].shape[1:], generator=g).bfloat16()])
    cm = torch.ones(2, ctx.shape[1], dtype=torch.bool)
    prop = torch.cat([fx["proprio"], torch.randn(1, 8, generator=g).bfloat16()])
    seeds = [42, 7]
    out = FW.infer_action_multi(model, None, imgs, 16, prop, 4, seeds=seeds, context=ctx, context_mask=cm)["action"]
    assert out.shape == (2, 16, model.action_expert.action_dim)
    for i in range(2):
        ref = model.infer_action(prompt=None, input_image=imgs[i:i + 1], action_horizon=16, proprio=prop[i],
                                 context=ctx[i:i + 1], context_mask=cm[i:i + 1], num_inference_steps=4,
                                 seed=seeds[i])["action"]
        _close(f"infer_action_multi row {i}", out[i].float().cpu(), ref)
