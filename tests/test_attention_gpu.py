"""fam_attention (split-KV flash attention, two key sources, masks) against torch fp32 SDPA."""
import pytest
import torch

from oracle import fam_oracle as O

pytestmark = pytest.mark.gpu


def _ref(q, k, v, heads, mask=None):
    return O.flash_attention(q.float(), k.float(), v.float(), heads, mask)


@pytest.mark.parametrize("B,H,hd,Sq,S1,S2,splits", [
    (1, 16, 64, 32, 1760, 32, 0), (2, 4, 64, 8, 130, 8, 3), (1, 24, 128, 200, 200, 0, 1),
    (2, 2, 128, 70, 300, 17, 0), (3, 4, 64, 32, 0, 40, 0)])
def test_attention_matches_sdpa(fam_ops, B, H, hd, Sq, S1, S2, splits):
    g = torch.Generator(device="cuda").manual_seed(B * 100 + Sq + S1)
    HD = H * hd
    q = torch.randn(B, Sq, HD, device="cuda", generator=g).bfloat16()
    k1 = torch.randn(B, max(S1, 1), HD, device="cuda", generator=g).bfloat16()[:, :S1]
    v1 = torch.randn(B, max(S1, 1), HD, device="cuda", generator=g).bfloat16()[:, :S1]
    k2 = torch.randn(B, S2, HD, device="cuda", generator=g).bfloat16() if S2 else None
    v2 = torch.randn(B, S2, HD, device="cuda", generator=g).bfloat16() if S2 else None
    mask = (torch.rand(Sq, S1 + S2, device="cuda", generator=g) > 0.3)
    mask[:, -1] = True  # every query keeps at least one key
    out = fam_ops.attention(q, k1, v1, H, k2, v2, mask=mask.to(torch.uint8), kv_splits=splits)
    torch.cuda.synchronize()
    kk = torch.cat([k1, k2], 1) if S2 else k1
    vv = torch.cat([v1, v2], 1) if S2 else v1
    ref = _ref(q, kk, vv, H, mask)
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, err


def test_first_frame_causal_and_key_mask(fam_ops):
    g = torch.Generator(device="cuda").manual_seed(9)
    B, H, hd, S, ff = 2, 4, 128, 300, 44
    q = torch.randn(B, S, H * hd, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, S, H * hd, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, S, H * hd, device="cuda", generator=g).bfloat16()
    out = fam_ops.attention(q, k, v, H, first_frame_tokens=ff)
    ref = _ref(q, k, v, H, O.build_video_to_video_mask(S, ff).cuda())
    assert (out.float() - ref).abs().max().item() < 2e-2
    km = torch.ones(B, S, dtype=torch.uint8, device="cuda")
    km[1, 250:] = 0
    out2 = fam_ops.attention(q, k, v, H, key_mask=km)
    ref2 = torch.cat([_ref(q[:1], k[:1], v[:1], H), _ref(q[1:], k[1:, :250], v[1:, :250], H)])
    torch.cuda.synchronize()
    assert (out2.float() - ref2).abs().max().item() < 2e-2


@pytest.mark.parametrize("B,S,H,ff", [(1, 1760, 4, 352), (2, 700, 3, 176), (1, 512, 2, 0), (2, 1000, 2, 0),
                                      (2, 600, 2, 0)])
def test_tcgen05_self_attention(fam_ops, B, S, H, ff):
    """Long self attention (one key source, head_dim 128) runs the tcgen05 kernel
    (TMEM scores and output, V transposed once); ragged last tiles, several
    batches and the first-frame-causal rule."""
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + S + ff)
    HD = H * 128
    q = torch.randn(B, S, HD, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, S, HD, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, S, HD, device="cuda", generator=g).bfloat16()
    out = fam_ops.attention(q, k, v, H, first_frame_tokens=ff)
    torch.cuda.synchronize()
    mask = torch.ones(S, S, dtype=torch.bool, device="cuda")
    if ff:
        mask[:ff, ff:] = False
    ref = _ref(q, k, v, H, mask)
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, err


def test_tcgen05_self_attention_sharp_rising_logits(fam_ops):
    """Scores that grow along the keys (so the running row maximum keeps moving by more
    than the lazy-rescale margin and the O rows are rescaled) and sharp softmaxes."""
    B, S, H = 1, 1024, 2
    g = torch.Generator(device="cuda").manual_seed(7)
    HD = H * 128
    q = (3.0 * torch.randn(B, S, HD, device="cuda", generator=g)).bfloat16()
    ramp = torch.linspace(0.2, 3.0, S, device="cuda").view(1, S, 1)
    k = (torch.randn(B, S, HD, device="cuda", generator=g) * ramp).bfloat16()
    v = torch.randn(B, S, HD, device="cuda", generator=g).bfloat16()
    out = fam_ops.attention(q, k, v, H)
    torch.cuda.synchronize()
    ref = _ref(q, k, v, H, torch.ones(S, S, dtype=torch.bool, device="cuda"))
    err = (out.float() - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(out.double().flatten(), ref.double().flatten(), dim=0).item()
    assert err < 2e-2 and cos >= 0.999, (err, cos)


@pytest.mark.parametrize("B,S,C,H", [(4, 1760, 64, 24), (4, 600, 300, 64), (1, 600, 300, 2)])
def test_tcgen05_attention_over_second_key_source(fam_ops, B, S, C, H):
    """Queries over a separate key source (the backbone's cross attention over the context
    tokens): C keys padded to 128-key blocks, a per-batch key mask.  The first two shapes
    launch >= 4 waves of CTAs and run the tcgen05 kernel, the last the split-KV kernel."""
    g = torch.Generator(device="cuda").manual_seed(S + C)
    HD = H * 128
    q = torch.randn(B, S, HD, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, C, HD, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, C, HD, device="cuda", generator=g).bfloat16()
    km = torch.ones(B, C, dtype=torch.uint8, device="cuda")
    km[-1, C - 7:] = 0
    km[0, 3] = 0
    out = fam_ops.attention(q, k, v, H, key_mask=km)
    torch.cuda.synchronize()
    ref = torch.cat([_ref(q[i:i + 1], k[i:i + 1], v[i:i + 1], H,
                          km[i].bool().view(1, C).expand(S, C).contiguous()) for i in range(B)])
    err = (out.float() - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(out.double().flatten(), ref.double().flatten(), dim=0).item()
    assert err < 2e-2 and cos >= 0.999, (err, cos)


def _workspace_bytes(fam_ops, q, k1, v1, H, k2=None, v2=None, mask=None, key_mask=None):
    import ctypes as C
    from importlib import import_module
    d, _ = fam_ops.attention_desc(q, k1, v1, H, k2, v2, mask, key_mask)
    n = C.c_size_t()
    lib = import_module("faster-action-models_b200._lib").lib()
    assert lib.fam_attention_workspace_size(C.byref(d), C.byref(n)) == 0
    return n.value


@pytest.mark.parametrize("B,H,Sq,S1,S2,use_mask,use_km", [
    (8, 16, 32, 1760, 32, True, False),   # the action expert's joint attention at batch 8
    (8, 16, 32, 64, 0, False, True),      # its cross attention over the context tokens
    (4, 32, 20, 300, 17, True, True),     # ragged: 20 queries, sources not multiples of 128 keys
    (2, 64, 32, 129, 0, False, False),
    (128, 1, 1, 5, 3, True, False),
    (32, 16, 32, 1760, 32, True, False),  # > 2 waves: the compact two-CTAs-per-SM variant
    (20, 16, 20, 300, 17, True, True)])
def test_tcgen05_short_query_attention(fam_ops, B, H, Sq, S1, S2, use_mask, use_km):
    """At most 32 queries per (batch, head), head dim 64, >= 128 (batch, head) pairs: the
    tcgen05 kernel with the queries replicated over the four TMEM lane quarters (each
    softmax warp owns a quarter of every key block), V as an MN-major operand, two key
    sources read through 3-D tensor maps, masks per query row and per batch key.  It needs
    no split workspace, which is how the test knows it ran; one query row is fully masked
    (output zero, as in the split-KV kernel)."""
    g = torch.Generator(device="cuda").manual_seed(B * 7 + Sq + S1 + S2)
    HD = H * 64
    q = torch.randn(B, Sq, HD, device="cuda", generator=g).bfloat16()
    k1 = torch.randn(B, S1, HD, device="cuda", generator=g).bfloat16()
    v1 = torch.randn(B, S1, HD, device="cuda", generator=g).bfloat16()
    k2 = torch.randn(B, S2, HD, device="cuda", generator=g).bfloat16() if S2 else None
    v2 = torch.randn(B, S2, HD, device="cuda", generator=g).bfloat16() if S2 else None
    S = S1 + S2
    mask = torch.ones(Sq, S, dtype=torch.bool, device="cuda")
    if use_mask:
        mask = torch.rand(Sq, S, device="cuda", generator=g) > 0.3
        mask[:, -1] = True
        if Sq > 1:
            mask[Sq // 2] = False  # a fully masked query row
    km = None
    if use_km:
        km = (torch.rand(B, S, device="cuda", generator=g) > 0.2).to(torch.uint8)
        km[:, -1] = 1
    m8 = mask.to(torch.uint8) if use_mask else None
    assert _workspace_bytes(fam_ops, q, k1, v1, H, k2, v2, m8, km) == 0
    out = fam_ops.attention(q, k1, v1, H, k2, v2, mask=m8, key_mask=km)
    torch.cuda.synchronize()
    kk = torch.cat([k1, k2], 1) if S2 else k1
    vv = torch.cat([v1, v2], 1) if S2 else v1
    refs = []
    for i in range(B):
        mi = mask & km[i].bool().view(1, S) if km is not None else mask
        refs.append(_ref(q[i:i + 1], kk[i:i + 1], vv[i:i + 1], H, mi.contiguous()))
    ref = torch.cat(refs)
    live = mask.any(1) if km is None else torch.ones(Sq, dtype=torch.bool, device="cuda")
    if use_mask and Sq > 1:
        assert torch.all(out[:, Sq // 2] == 0)
        live = live.clone()
        live[Sq // 2] = False
    o, r = out.float()[:, live], ref[:, live]
    err = (o - r).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(o.double().flatten(), r.double().flatten(), dim=0).item()
    assert err < 2e-2 and cos >= 0.999, (err, cos)
    # the same call with explicit splits takes the split-KV kernel: both agree
    alt = fam_ops.attention(q, k1, v1, H, k2, v2, mask=m8, key_mask=km, kv_splits=2)
    torch.cuda.synchronize()
    assert (alt.float()[:, live] - o).abs().max().item() < 2e-2


@pytest.mark.parametrize("B", [8, 32])
def test_tcgen05_short_query_attention_sharp_rising_logits(fam_ops, B):
    """Scores that grow along the keys move each quarter's running maximum by more than
    the lazy-rescale margin again and again (O rows rescaled in TMEM); batch 8 runs the
    double-buffered variant, batch 32 the compact one."""
    H, Sq, S = 16, 32, 1792
    g = torch.Generator(device="cuda").manual_seed(11)
    HD = H * 64
    q = (3.0 * torch.randn(B, Sq, HD, device="cuda", generator=g)).bfloat16()
    ramp = torch.linspace(0.2, 3.0, S, device="cuda").view(1, S, 1)
    k = (torch.randn(B, S, HD, device="cuda", generator=g) * ramp).bfloat16()
    v = torch.randn(B, S, HD, device="cuda", generator=g).bfloat16()
    assert _workspace_bytes(fam_ops, q, k, v, H) == 0
    out = fam_ops.attention(q, k, v, H)
    torch.cuda.synchronize()
    ref = _ref(q, k, v, H, torch.ones(Sq, S, dtype=torch.bool, device="cuda"))
    err = (out.float() - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(out.double().flatten(), ref.double().flatten(), dim=0).item()
    assert err < 2e-2 and cos >= 0.999, (err, cos)
