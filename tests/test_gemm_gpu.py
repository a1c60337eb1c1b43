"""tcgen05 GEMM against a torch fp32 matmul of the same bf16 operands."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(x, w, bias=None, act="none"):
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    if act == "gelu_tanh":
        y = torch.nn.functional.gelu(y, approximate="tanh")
    return y


def _close(got, ref, tol=2e-2):
    err = (got.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err} vs scale {scale}"


@pytest.mark.parametrize("T,F,K", [(32, 1024, 1024), (32, 3072, 1024), (8, 256, 64),
                                   (17, 200, 136), (256, 4096, 1024), (64, 1024, 4096)])
@pytest.mark.parametrize("act", ["none", "gelu_tanh"])
def test_weights_as_a_store(fam_ops, T, F, K, act):
    g = torch.Generator(device="cuda").manual_seed(T * 7 + F + K)
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(F, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    b = torch.randn(F, device="cuda", generator=g).bfloat16()
    y = fam_ops.gemm(w, x, bias=b, act=act, weights_as_a=True)
    torch.cuda.synchronize()
    _close(y, _ref(x, w, b, act))


@pytest.mark.parametrize("T,F,K", [(1760, 3072, 3072), (300, 256, 192), (128, 128, 64), (1000, 520, 4096)])
def test_activations_as_a_store(fam_ops, T, F, K):
    g = torch.Generator(device="cuda").manual_seed(T + F + K)
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(F, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    b = torch.randn(F, device="cuda", generator=g).bfloat16()
    y = fam_ops.gemm(x, w, bias=b)
    torch.cuda.synchronize()
    _close(y, _ref(x, w, b))


@pytest.mark.parametrize("splits", [2, 4, 16])
def test_split_k_partials(fam_ops, splits):
    g = torch.Generator(device="cuda").manual_seed(splits)
    T, F, K = 32, 1024, 4096
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(F, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    p = fam_ops.gemm(w, x, weights_as_a=True, splits=splits)
    torch.cuda.synchronize()
    assert p.shape == (splits, T, F)
    _close(p.sum(0), _ref(x, w))


def test_residual_gate(fam_ops):
    g = torch.Generator(device="cuda").manual_seed(5)
    B, S, K, F, ff = 2, 96, 256, 384, 40
    x = torch.randn(B * S, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(F, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    b = torch.randn(F, device="cuda", generator=g).bfloat16()
    gw = torch.randn(F, device="cuda", generator=g).bfloat16()
    gt = torch.randn(B, 2, F, device="cuda", generator=g)
    r0 = torch.randn(B * S, F, device="cuda", generator=g)
    r = r0.clone()
    fam_ops.gemm(x, w, bias=b, residual=r, gate_w=gw, gate_t=gt, tokens_per_batch=S,
                 first_frame_tokens=ff, gate_batch_stride=2 * F, gate_group_stride=F)
    torch.cuda.synchronize()
    tok = torch.arange(B * S, device="cuda")
    grp = ((tok % S) >= ff).long()
    gate = gw.float()[None, :] + gt[tok // S, grp]
    ref = r0 + gate * _ref(x, w, b)
    _close(r, ref)
    # swap-AB orientation with a per-batch gate
    r = r0[:64].clone()
    fam_ops.gemm(w, x[:64], bias=b, residual=r, gate_w=gw, gate_t=gt, weights_as_a=True,
                 tokens_per_batch=32, gate_batch_stride=2 * F)
    torch.cuda.synchronize()
    tok = torch.arange(64, device="cuda")
    gate = gw.float()[None, :] + gt[tok // 32, 0]
    _close(r, r0[:64] + gate * _ref(x[:64], w, b))


@pytest.mark.parametrize("tile_n", [0, 128, 160, 192, 256])
def test_persistent_residual_and_store(fam_ops, tile_n):
    """Many-tile problems run the persistent kernel (two TMEM accumulators, vector
    residual epilogue); tile widths 128 / 160 / 192 / 256 and the automatic choice."""
    g = torch.Generator(device="cuda").manual_seed(11 + tile_n)
    B, S, K, F, ff = 2, 880, 512, 3072, 352
    x = torch.randn(B * S, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(F, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    b = torch.randn(F, device="cuda", generator=g).bfloat16()
    gw = torch.randn(F, device="cuda", generator=g).bfloat16()
    gt = torch.randn(B, 2, F, device="cuda", generator=g)
    r0 = torch.randn(B * S, F, device="cuda", generator=g)
    r = r0.clone()
    fam_ops.gemm(x, w, bias=b, residual=r, gate_w=gw, gate_t=gt, tokens_per_batch=S,
                 first_frame_tokens=ff, gate_batch_stride=2 * F, gate_group_stride=F, tile_n=tile_n)
    y = fam_ops.gemm(x, w, bias=b, act="gelu_tanh", tile_n=tile_n)
    torch.cuda.synchronize()
    tok = torch.arange(B * S, device="cuda")
    grp = ((tok % S) >= ff).long()
    gate = gw.float()[None, :] + gt[tok // S, grp]
    _close(r, r0 + gate * _ref(x, w, b))
    _close(y, _ref(x, w, b, "gelu_tanh"))


@pytest.mark.parametrize("F,K", [(3072, 512), (3072, 1344), (9216, 512), (14336, 256)])
def test_split_round(fam_ops, F, K):
    """Split last round: 256-wide tiles round-robin, each tile of the partial last
    round cut into 4 / 2 / 3 k-pieces (F = 3072 / 9216 / 14336 at 1760 tokens) and
    finished from the later pieces' fp32 partials; residual and GELU-store
    epilogues, deterministic across launches; the model-chosen schedule agrees."""
    g = torch.Generator(device="cuda").manual_seed(K)
    B, S, ff = 2, 880, 352
    x = torch.randn(B * S, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(F, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    b = torch.randn(F, device="cuda", generator=g).bfloat16()
    gw = torch.randn(F, device="cuda", generator=g).bfloat16()
    gt = torch.randn(B, 2, F, device="cuda", generator=g)
    r0 = torch.randn(B * S, F, device="cuda", generator=g)
    outs = []
    for _ in range(2):
        r = r0.clone()
        fam_ops.gemm(x, w, bias=b, residual=r, gate_w=gw, gate_t=gt, tokens_per_batch=S,
                     first_frame_tokens=ff, gate_batch_stride=2 * F, gate_group_stride=F,
                     split_round="always")
        y = fam_ops.gemm(x, w, bias=b, act="gelu_tanh", split_round="always")
        torch.cuda.synchronize()
        outs.append((r, y))
    y_auto = fam_ops.gemm(x, w, bias=b, act="gelu_tanh", split_round="auto")
    tok = torch.arange(B * S, device="cuda")
    grp = ((tok % S) >= ff).long()
    gate = gw.float()[None, :] + gt[tok // S, grp]
    _close(outs[0][0], r0 + gate * _ref(x, w, b))
    _close(outs[0][1], _ref(x, w, b, "gelu_tanh"))
    _close(y_auto, _ref(x, w, b, "gelu_tanh"))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("M,K,N", [(1760, 512, 3072), (600, 1344, 1024), (1024, 3072, 9216)])
def test_cta_pair(fam_ops, M, K, N):
    """CTA-pair kernel (tcgen05 cta_group::2, 256 x 256 tiles, half of B per CTA):
    store, GELU-store and gated-residual epilogues, ragged M, deterministic."""
    g = torch.Generator(device="cuda").manual_seed(M + K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    b = torch.randn(N, device="cuda", generator=g).bfloat16()
    gt = torch.randn(1, N, device="cuda", generator=g)
    r0 = torch.randn(M, N, device="cuda", generator=g)
    outs = []
    for _ in range(2):
        y = fam_ops.gemm(x, w, bias=b, pair=True, tile_n=256)
        yg = fam_ops.gemm(x, w, bias=b, act="gelu_tanh", pair=True, tile_n=256)
        r = r0.clone()
        fam_ops.gemm(x, w, bias=b, residual=r, gate_t=gt, tokens_per_batch=M, pair=True, tile_n=256)
        torch.cuda.synchronize()
        outs.append((y, yg, r))
    _close(outs[0][0], _ref(x, w, b))
    _close(outs[0][1], _ref(x, w, b, "gelu_tanh"))
    _close(outs[0][2], r0 + gt[0][None, :] * _ref(x, w, b))
    for a, c in zip(outs[0], outs[1]):
        assert torch.equal(a, c)
