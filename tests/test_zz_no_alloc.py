"""fam_attention_static_scratch: the attention entry point for callers that cannot
allocate device memory (a plugin that does not own its host process's allocator, a
control loop that forbids allocation once running, an FFI host with no device
allocator).  It must give the same result as fam_attention with a caller workspace,
on two calls in a row (the second finds the first call's leftovers in the shared
static scratch), and reject a problem larger than its fixed scratch.

This file is collected last on purpose (tests/test_zz_*), and passes both alone in a
fresh process and after the rest of the suite."""
import ctypes as C
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu

ops = importlib.import_module("faster-action-models_b200.ops")
_lib = importlib.import_module("faster-action-models_b200._lib")


def _case(B, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    H, hd, Sq, S1, S2 = 16, 64, 32, 1760, 32
    HD = H * hd
    q = torch.randn(B, Sq, HD, device="cuda", generator=g).bfloat16()
    k1 = torch.randn(B, S1, HD, device="cuda", generator=g).bfloat16()
    v1 = torch.randn(B, S1, HD, device="cuda", generator=g).bfloat16()
    k2 = torch.randn(B, S2, HD, device="cuda", generator=g).bfloat16()
    v2 = torch.randn(B, S2, HD, device="cuda", generator=g).bfloat16()
    mask = (torch.rand(Sq, S1 + S2, device="cuda", generator=g) > 0.2).to(torch.uint8)
    mask[:, -1] = 1
    return q, k1, v1, H, k2, v2, mask


def _sdpa_fp32(q, k1, v1, H, k2, v2, mask):
    B, Sq, HD = q.shape
    k = torch.cat([k1, k2], 1).float().view(B, -1, H, HD // H).transpose(1, 2)
    v = torch.cat([v1, v2], 1).float().view(B, -1, H, HD // H).transpose(1, 2)
    qh = q.float().view(B, Sq, H, HD // H).transpose(1, 2)
    o = torch.nn.functional.scaled_dot_product_attention(qh, k, v, attn_mask=mask.bool())
    return o.transpose(1, 2).reshape(B, Sq, HD)


def test_static_scratch_matches_workspace_entry_point_twice():
    lib = _lib.lib()
    for call, seed in ((0, 11), (1, 12)):
        q, k1, v1, H, k2, v2, mask = _case(2, seed)
        ref = ops.attention(q, k1, v1, H, k2, v2, mask=mask)
        d, out = ops.attention_desc(q, k1, v1, H, k2, v2, mask=mask)
        n = C.c_size_t()
        _lib.check(lib.fam_attention_workspace_size(C.byref(d), C.byref(n)), "workspace size")
        assert n.value > 0, "the case must use split scratch"
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(lib.fam_attention_static_scratch(C.byref(d), C.c_void_p(stream)),
                   "fam_attention_static_scratch")
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= 2e-2, f"call {call}: max|d| {err}"
        # and against plain fp32 attention of the same inputs (masked SDPA over the
        # concatenated keys), independent of the library's own kernels
        sd = _sdpa_fp32(q, k1, v1, H, k2, v2, mask)
        err_sd = (out.float() - sd).abs().max().item()
        cos = torch.nn.functional.cosine_similarity(out.float().flatten(), sd.flatten(), dim=0).item()
        assert err_sd <= 2e-2 and cos >= 0.999, f"call {call}: vs fp32 SDPA max|d| {err_sd} cos {cos}"


def test_static_scratch_short_query_shape_runs_tcgen05_without_scratch():
    """Batch 8 x 16 heads of 32 queries: the descriptor the tcgen05 short-query kernel
    takes (no split workspace), through the allocation-free entry point, twice."""
    lib = _lib.lib()
    for call, seed in ((0, 21), (1, 22)):
        q, k1, v1, H, k2, v2, mask = _case(8, seed)
        d, out = ops.attention_desc(q, k1, v1, H, k2, v2, mask=mask)
        n = C.c_size_t()
        _lib.check(lib.fam_attention_workspace_size(C.byref(d), C.byref(n)), "workspace size")
        assert n.value == 0, "the case must take the scratch-free tcgen05 kernel"
        _lib.check(lib.fam_attention_static_scratch(C.byref(d), C.c_void_p(torch.cuda.current_stream().cuda_stream)),
                   "fam_attention_static_scratch")
        torch.cuda.synchronize()
        sd = _sdpa_fp32(q, k1, v1, H, k2, v2, mask)
        err = (out.float() - sd).abs().max().item()
        cos = torch.nn.functional.cosine_similarity(out.float().flatten(), sd.flatten(), dim=0).item()
        assert err <= 2e-2 and cos >= 0.999, f"call {call}: vs fp32 SDPA max|d| {err} cos {cos}"


def test_static_scratch_rejects_oversized_problem():
    lib = _lib.lib()
    q, k1, v1, H, k2, v2, mask = _case(4, 13)
    # 28 key splits x 4 batches x 16 heads of partials: ~30 MB, beyond the 8 MiB array
    d, out = ops.attention_desc(q, k1, v1, H, k2, v2, mask=mask, kv_splits=28)
    rc = lib.fam_attention_static_scratch(C.byref(d), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 1  # FAM_ERR_INVALID
    assert "scratch" in _lib.last_error()
