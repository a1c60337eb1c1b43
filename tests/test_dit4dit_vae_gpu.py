"""DiT4DiT's Action-VAE decode (BASELINE config 3's compact path) on the GPU, against the
golden made from the reference module (DiT4DiT/model/modules/action_model/action_vae.py:
136-197, tests/golden/dit4dit_action_vae.pt): the checkpoint is read by
ActionAE.from_dit4dit and decoded by the separate decoder launches and by the CAE step
kernel's epilogue.  To feed the golden latents through the epilogue unchanged, the chunk
runs one Euler step with delta 0 (latent + velocity * 0 is the latent exactly).  Gate
(fp32 path): max|d| <= 2e-3 * max(1, max|ref|), cosine >= 0.999."""
import importlib
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

M = importlib.import_module("faster-action-models_b200.models")
GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ["c3_task_conditioned", "encoder_only", "stride3_crop", "two_stage_crop"]


def _check(name, got, ref, rel=2e-3):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert got.shape == ref.shape, (got.shape, ref.shape)
    err = (got - ref).abs().max().item()
    scale = max(1.0, ref.abs().max().item())
    cos = torch.nn.functional.cosine_similarity(got.double().flatten(), ref.double().flatten(), dim=0).item()
    print(f"PARITY dit4dit {name}: max|d| {err:.3g} cos {cos:.6f}")
    assert err <= rel * scale and cos >= 0.999, f"{name}: max|d| {err} cos {cos}"


def _case(name):
    return torch.load(GOLDEN / "dit4dit_action_vae.pt", weights_only=False)["cases"][name]


def _task_ids(fx):
    return fx["task_ids"].cuda() if fx["task_ids"] is not None else None


@pytest.mark.parametrize("case", CASES)
def test_separate_decode_matches_reference(case):
    fx = _case(case)
    ck = dict(fx["checkpoint"])
    ids = _task_ids(fx)
    if "actions_denorm" in fx:
        ae = M.ActionAE.from_dit4dit(ck).cuda()
        _check(f"{case} decode(z * std + mean)", ae.decode(fx["latent"].cuda(), ids), fx["actions_denorm"])
        ck["apply_latent_normalization"] = False
    ae = M.ActionAE.from_dit4dit(ck).cuda()
    _check(f"{case} decode", ae.decode(fx["latent"].cuda(), ids), fx["actions"])
    if ae.decoder.require_suite_ids:
        with pytest.raises(ValueError, match="task_ids"):
            ae.decode(fx["latent"].cuda())


@pytest.mark.parametrize("case", CASES)
def test_step_kernel_epilogue_decode_matches_reference(case):
    """The golden latents through fam_cae_chunk_decode(decode="fused"): one-stage decoders
    of stride 2 or 4 (c3: 2, encoder_only: 4) decode in the epilogue; stride 3 and
    two-stage decoders take the separate launches.  Same chunk either way."""
    fx = _case(case)
    ck = fx["checkpoint"]
    c = ck["config"]
    ids = _task_ids(fx)
    torch.manual_seed(7)
    head = M.ActionDiT(hidden_dim=32, action_dim=c["latent_dim"], ffn_dim=128, text_dim=64, freq_dim=256, eps=1e-6,
                       num_heads=4, attn_head_dim=8, num_layers=2).cuda()
    feats = torch.randn(fx["latent"].shape[0], 40, 64, device="cuda")
    eng = head.engine()
    want_fused = case in ("c3_task_conditioned", "encoder_only")
    runs = [(ck, "actions_denorm" if "actions_denorm" in fx else "actions")]
    if "actions_denorm" in fx:
        runs.append((dict(ck, apply_latent_normalization=False), "actions"))
    for ckpt, key in runs:
        ae = M.ActionAE.from_dit4dit(ckpt).cuda()
        for _ in range(2):
            lat, chunk = eng.chunk_decode(fx["latent"].cuda(), [1000.0], [0.0], feats, ae, suite_ids=ids,
                                          decode="fused")
            torch.cuda.synchronize()
            assert eng.decode_fused == want_fused
            assert torch.equal(lat.cpu(), fx["latent"])
            _check(f"{case} epilogue {key}", chunk, fx[key])
