"""Wan2.2 VAE encode of the observation frame (VideoVAE38_.encode, T = 1) on the
GPU against the reference's recorded output (golden fixture) and the CPU oracle.

Tolerance: activations are bf16 between layers (fp32 accumulation, fp32
residual stream), as the reference runs the VAE in bf16; the bound is the
north-star parity bar, max |d| <= 2e-2 * max(1, max |ref|) and cosine >= 0.999
against the fp32 result, which the reference's own bf16 run also meets."""
import importlib
from pathlib import Path

import pytest
import torch

from oracle import fam_oracle as O

pytestmark = pytest.mark.gpu

V = importlib.import_module("faster-action-models_b200.vae")
GOLDEN = Path(__file__).resolve().parent / "golden"


def _check(got, ref):
    got, ref = got.float().cpu().flatten(), ref.float().cpu().flatten()
    assert got.shape == ref.shape
    err = (got - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(got, ref, dim=0).item()
    assert err <= 2e-2 * max(1.0, ref.abs().max().item()), f"max |d| = {err}"
    assert cos >= 0.999, f"cosine {cos}"


@pytest.mark.parametrize("use_graph", [False, True])
def test_vae_encode_golden(use_graph):
    fx = torch.load(GOLDEN / "vae_encode.pt", weights_only=False)
    c = fx["cfg"]
    vae = V.WanVideoVAE38(fx["params"], fx["mean"], 1.0 / fx["inv_std"], z_dim=c["z_dim"], dim=c["dim"])
    mu = vae.model.encode(fx["image"].cuda(), vae.scale, use_graph=use_graph)
    torch.cuda.synchronize()
    assert mu.shape == fx["mu_f32"].shape
    _check(mu, fx["mu_f32"])
    # the reference's own bf16 run meets the same bar
    _check(fx["mu_bf16"], fx["mu_f32"])


def _random_params(dim, z_dim, g):
    """Seeded parameters with the reference's names and shapes (Encoder3d_38 + conv1)."""
    cfg = O.VaeConfig(dim=dim, z_dim=z_dim)
    dims = [dim * u for u in (1,) + cfg.dim_mult]
    p = {}

    def conv(name, cout, cin, k3, k=3):
        shape = (cout, cin, k, k, k) if k3 else (cout, cin, k, k)
        p[name + ".weight"] = (torch.randn(shape, generator=g) / (cin * k * k * (k if k3 else 1)) ** 0.5).bfloat16()
        p[name + ".bias"] = (0.05 * torch.randn(cout, generator=g)).bfloat16()

    def gamma(name, c, img=False):
        shape = (c, 1, 1) if img else (c, 1, 1, 1)
        p[name + ".gamma"] = (1.0 + 0.1 * torch.randn(shape, generator=g)).bfloat16()

    def rb(pre, cin, cout):
        gamma(pre + ".residual.0", cin)
        conv(pre + ".residual.2", cout, cin, True)
        gamma(pre + ".residual.3", cout)
        conv(pre + ".residual.6", cout, cout, True)
        if cin != cout:
            conv(pre + ".shortcut", cout, cin, True, k=1)

    conv("encoder.conv1", dims[0], 12, True)
    for i, (din, dout) in enumerate(zip(dims[:-1], dims[1:])):
        pre = f"encoder.downsamples.{i}.downsamples"
        rb(f"{pre}.0", din, dout)
        rb(f"{pre}.1", dout, dout)
        if i != len(cfg.dim_mult) - 1:
            conv(f"{pre}.2.resample.1", dout, dout, False)
    c = dims[-1]
    rb("encoder.middle.0", c, c)
    gamma("encoder.middle.1.norm", c, img=True)
    conv("encoder.middle.1.to_qkv", 3 * c, c, False, k=1)
    conv("encoder.middle.1.proj", c, c, False, k=1)
    rb("encoder.middle.2", c, c)
    gamma("encoder.head.0", c)
    conv("encoder.head.2", 2 * z_dim, c, True)
    conv("conv1", 2 * z_dim, 2 * z_dim, True, k=1)
    return cfg, p


def test_vae_encode_wider_against_oracle():
    """dim 32 / z 16 on a 128 x 192 frame: every channel count above one GEMM tile row."""
    g = torch.Generator().manual_seed(11)
    cfg, p = _random_params(32, 16, g)
    image = (torch.rand(1, 3, 1, 128, 192, generator=g) * 2 - 1).bfloat16()
    mean = (0.2 * torch.randn(16, generator=g)).bfloat16().float()
    std = (0.5 + torch.rand(16, generator=g)).bfloat16().float()
    ref = O.vae_encode_first_frame({k: v.float() for k, v in p.items()}, cfg, image.float(), mean, 1.0 / std)
    vae = V.WanVideoVAE38(p, mean, std, z_dim=16, dim=32)
    mu = vae.model.encode(image.cuda(), vae.scale)
    torch.cuda.synchronize()
    _check(mu, ref)
    # a second call replays the captured graph with new inputs
    image2 = (torch.rand(1, 3, 1, 128, 192, generator=g) * 2 - 1).bfloat16()
    ref2 = O.vae_encode_first_frame({k: v.float() for k, v in p.items()}, cfg, image2.float(), mean, 1.0 / std)
    mu2 = vae.model.encode(image2.cuda(), vae.scale)
    torch.cuda.synchronize()
    _check(mu2, ref2)


def test_vae_encode_rejects_multi_frame():
    g = torch.Generator().manual_seed(12)
    _, p = _random_params(8, 8, g)
    vae = V.WanVideoVAE38(p, torch.zeros(8), torch.ones(8), z_dim=8, dim=8)
    with pytest.raises(NotImplementedError):
        vae.model.encode(torch.zeros(1, 3, 5, 64, 64).bfloat16().cuda(), vae.scale)
