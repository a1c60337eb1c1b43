"""Host-side interface checks that need no GPU: the module mirror keeps the
reference's state_dict layout (and its seeded initial weights), the schedule
helper matches the oracle, and the C-ABI library loads and exports every
symbol that include/fam.h declares."""
import ctypes
import importlib
import re
from pathlib import Path

import pytest
import torch

from oracle import fam_oracle as O

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
M = importlib.import_module("faster-action-models_b200.models")


def test_action_dit_state_dict_matches_reference_layout_and_init():
    fx = torch.load(GOLDEN / "c1_action_cache.pt", weights_only=False)
    torch.manual_seed(1)  # the seed make_golden.py used before constructing the reference module
    dit = M.ActionDiT(**fx["dit_cfg"]).to(torch.bfloat16)
    sd = dit.state_dict()
    assert list(sd.keys()) == list(fx["dit"].keys())
    for k, v in fx["dit"].items():
        assert sd[k].shape == v.shape, k
        assert torch.equal(sd[k], v), f"seeded init differs at {k}"
    # load_state_dict round trip drops the packed kernel weights
    dit._engine = object()
    dit.load_state_dict(fx["dit"])
    assert dit._engine is None


def test_cae_expert_and_action_ae_layout_and_init():
    fx = torch.load(GOLDEN / "c0_cae_expert.pt", weights_only=False)
    torch.manual_seed(0)  # make_golden.py: seed, ActionDiT, then ActionAE, then bf16 rounding
    dit = M.ActionDiT(**fx["dit_cfg"])
    c = fx["dec_cfg"]
    ae = M.ActionAE(M.ActionAEConfig(action_dim=c["action_dim"], action_horizon=c["action_horizon"],
                                     num_tokens=c["num_tokens"], latent_dim=c["latent_dim"],
                                     decoder_hidden=c["decoder_hidden"], video_cond_dim=0,
                                     variational=True))
    for mod, key in ((dit, "dit"), (ae, "ae")):
        sd = {k: v.to(torch.bfloat16) for k, v in mod.state_dict().items()}
        assert list(sd.keys()) == list(fx[key].keys()), key
        for k, v in fx[key].items():
            assert torch.equal(sd[k], v), f"{key}: {k}"
    assert dit.is_compact()


def test_wan_video_dit_layout_init_and_rope():
    fx = torch.load(GOLDEN / "c2_video_prefill.pt", weights_only=False)
    c = fx["dit_cfg"]
    torch.manual_seed(2)  # make_golden.py seeds, then builds WanVideoDiT first
    dit = M.WanVideoDiT(hidden_dim=c["hidden_dim"], in_dim=c["in_dim"], ffn_dim=c["ffn_dim"],
                        out_dim=c["out_dim"], text_dim=c["text_dim"], freq_dim=c["freq_dim"],
                        eps=c["eps"], patch_size=tuple(c["patch_size"]), num_heads=c["num_heads"],
                        attn_head_dim=c["attn_head_dim"], num_layers=c["num_layers"],
                        has_image_input=False, seperated_timestep=True,
                        video_attention_mask_mode="first_frame_causal").to(torch.bfloat16)
    sd = dit.state_dict()
    assert list(sd.keys()) == list(fx["video"].keys())
    for k, v in fx["video"].items():
        assert torch.equal(sd[k], v), k
    f, h, w = fx["grid"]
    tab = M.rope_table_3d(c["attn_head_dim"], f, h, w)
    ref = fx["freqs"].reshape(f * h * w, -1)
    assert torch.allclose(tab[..., 0], ref.real.float(), atol=1e-6)
    assert torch.allclose(tab[..., 1], ref.imag.float(), atol=1e-6)


def test_schedule_helper_matches_oracle():
    for n, s in ((10, 1.0), (4, 5.0), (7, 3.0)):
        for dt in (torch.float32, torch.bfloat16):
            t, d = M.build_inference_schedule(n, s, dtype=dt)
            rt, rd = O.build_inference_schedule(n, s, dtype=dt)
            assert t == rt.float().tolist() and d == rd.float().tolist()


def test_rope_table_matches_reference_freqs():
    tab = M.rope_table(64)
    ref = O.precompute_freqs_cis(64, end=1024)
    assert torch.allclose(tab[..., 0], ref.real.float(), atol=1e-7)
    assert torch.allclose(tab[..., 1], ref.imag.float(), atol=1e-7)


def test_library_loads_and_exports_every_declared_symbol():
    lib_path = ROOT / "faster-action-models_b200" / "libfam.so"
    if not lib_path.exists():
        pytest.skip("libfam.so not built (run __graft_entry__.build())")
    lib = ctypes.CDLL(str(lib_path))
    header = (ROOT / "include" / "fam.h").read_text()
    names = re.findall(r"FAM_API\s+\w+\s+(fam_\w+)\s*\(", header)
    assert len(names) >= 8
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/fam.h but not exported"
    fam = importlib.import_module("faster-action-models_b200")
    assert fam.version()[0] == 0


def test_elide_backbone_shares_parameters():
    """DiT4DiT tail elision: the elided backbone holds blocks 0..k of the original module
    (the same parameter tensors) and leaves the original untouched."""
    P = importlib.import_module("faster-action-models_b200.pipeline")
    Mm = importlib.import_module("faster-action-models_b200.models")
    vid = Mm.WanVideoDiT(hidden_dim=64, in_dim=4, ffn_dim=128, out_dim=4, text_dim=32, freq_dim=256, eps=1e-6,
                         patch_size=(1, 2, 2), num_heads=2, attn_head_dim=32, num_layers=4,
                         has_image_input=False)
    el = P.elide_backbone(vid, 1)
    assert el.num_layers == 2 and vid.num_layers == 4
    full = dict(vid.named_parameters())
    for name, p in el.named_parameters():
        assert p is full[name]
    names = {n for n, _ in el.named_parameters()}
    assert not any(n.startswith(("blocks.2.", "blocks.3.")) for n in names)
    assert any(n.startswith("blocks.1.") for n in names)
    import pytest as _pt
    with _pt.raises(ValueError):
        P.elide_backbone(vid, 4)


def test_vae_encoder_param_table_matches_reference_state_dict():
    """encoder_param_shapes lists exactly the reference VideoVAE38_ encoder parameters
    (names and shapes of the state dict recorded from the reference in the fixture)."""
    import importlib
    from pathlib import Path
    import torch
    V = importlib.import_module("faster-action-models_b200.vae")
    fx = torch.load(Path(__file__).resolve().parent / "golden" / "vae_encode.pt", weights_only=False)
    want = {k: tuple(v.shape) for k, v in fx["params"].items()}
    got = V.encoder_param_shapes(dim=fx["cfg"]["dim"], z_dim=fx["cfg"]["z_dim"])
    assert got == want
    # the host-side packing accepts them (no device work)
    enc = V.VideoVAE38Encoder(fx["params"], dim=fx["cfg"]["dim"], z_dim=fx["cfg"]["z_dim"], device="cpu")
    assert enc.conv_in.w.shape == (fx["cfg"]["dim"], 9 * 64)
    assert all(s[0] > 0 and s[2] % 8 == 0 for s in enc._gemm_shapes(64, 96))


def test_fastwam_checkpoint_layout_and_mot_checks():
    """The MoT holder's state_dict keys are the reference checkpoint's (`mixtures.video.` /
    `mixtures.action.`), load_checkpoint takes the reference payload unchanged, and the
    expert-compatibility checks of mot.py:33-52 hold."""
    import torch
    FW = importlib.import_module("faster-action-models_b200.fastwam")
    M = importlib.import_module("faster-action-models_b200.models")
    fx = torch.load(Path(__file__).resolve().parent / "golden" / "fastwam_infer_action.pt")
    video = M.WanVideoDiT(**fx["video_cfg"]).to(torch.bfloat16)
    action = M.ActionDiT(**fx["action_cfg"]).to(torch.bfloat16)
    mot = FW.MoT({"video": video, "action": action})
    assert set(mot.state_dict().keys()) == set(fx["checkpoint"]["mot"].keys())
    model = FW.FastWAM(video, action, mot, vae=None, text_dim=96, proprio_dim=8, device="cpu")
    model.load_checkpoint(fx["checkpoint"])
    for k, v in fx["checkpoint"]["mot"].items():
        assert torch.equal(mot.state_dict()[k], v), k
    assert torch.equal(model.proprio_encoder.weight, fx["checkpoint"]["proprio_encoder"]["weight"])
    bad = M.ActionDiT(**{**fx["action_cfg"], "num_layers": 3})
    with pytest.raises(ValueError, match="same number of layers"):
        FW.MoT({"video": video, "action": bad})
    with pytest.raises(ValueError, match="must include both"):
        FW.MoT({"video": video})
    with pytest.raises(ValueError, match="multiples of 16"):
        model.infer_action(None, torch.zeros(1, 3, 60, 96), 32, context=torch.zeros(1, 4, 96),
                           context_mask=torch.ones(1, 4, dtype=torch.bool))
    with pytest.raises(ValueError, match="last dim must be 8"):
        model.infer_action(None, torch.zeros(1, 3, 64, 96), 32, proprio=torch.zeros(1, 5))


def test_dit4dit_action_vae_loader():
    """ActionAE.from_dit4dit reads DiT4DiT's ActionVAE checkpoint layout: decoder weights with
    the task embedding as the suite embedding, task ids required when the decoder holds one,
    the latent statistics held for the kernels, and DiT4DiT's config checks."""
    fx = torch.load(GOLDEN / "dit4dit_action_vae.pt", weights_only=False)["cases"]
    ck = fx["c3_task_conditioned"]["checkpoint"]
    ae = M.ActionAE.from_dit4dit(ck)
    assert ae.encoder is None and ae.decoder.require_suite_ids
    assert (ae.cfg.action_dim, ae.cfg.action_horizon, ae.cfg.num_tokens, ae.cfg.latent_dim) == (29, 16, 8, 48)
    assert torch.equal(ae.decoder.suite_embed.weight, ck["model"]["decoder.task_embedding.weight"])
    assert torch.equal(ae.decoder.latent_std, ck["latent_std"].clamp_min(1e-4))
    assert torch.equal(ae.decoder.latent_mean, ck["latent_mean"])
    assert "latent_std" not in ae.decoder.state_dict()
    with pytest.raises(ValueError, match="task_ids are required"):
        ae.decoder.check_ids(None)
    eo = M.ActionAE.from_dit4dit(fx["encoder_only"]["checkpoint"])
    assert eo.decoder.suite_embed is None and not eo.decoder.require_suite_ids and eo.decoder.latent_std is None
    bad = {"config": dict(ck["config"], action_horizon=18), "model": ck["model"]}
    with pytest.raises(ValueError, match="divisible"):
        M.ActionAE.from_dit4dit(bad)
    with pytest.raises(ValueError, match="requires num_tasks"):
        M.ActionAE.from_dit4dit({"config": dict(ck["config"], num_tasks=0), "model": ck["model"]})
