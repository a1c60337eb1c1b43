"""Op-level wrappers over the C ABI, taking torch CUDA tensors.

torch is used only for device memory and the current stream; all arithmetic
runs in libfam.so kernels.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib
from ._lib import GemmDesc, check, lib


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")


def gemm(a: torch.Tensor, b: torch.Tensor, *, out: Optional[torch.Tensor] = None,
         bias: Optional[torch.Tensor] = None, act: str = "none", out_dtype=torch.bfloat16,
         weights_as_a: bool = False, splits: int = 1, tile_n: int = 0,
         residual: Optional[torch.Tensor] = None, gate_w: Optional[torch.Tensor] = None,
         gate_t: Optional[torch.Tensor] = None, tokens_per_batch: int = 0,
         first_frame_tokens: int = 0, gate_batch_stride: int = 0, gate_group_stride: int = 0,
         pdl: bool = False, split_round: str = "off", pair: bool = False) -> torch.Tensor:
    """Linear layer on the tensor cores.

    weights_as_a=False:  a = activations [T, K], b = weight [F, K] -> [T, F]
    weights_as_a=True:   a = weight [F, K], b = activations [T, K] -> [T, F]
    splits > 1 returns fp32 split-K partials [splits, T, F] (no bias).
    residual (fp32 [T, F]) is updated in place: residual += gate * (x W^T + bias).
    split_round: "auto" / "always" let a many-tile problem run 256-wide tiles and split
    each tile of the last, partial round into k-pieces on the idle SMs ("auto": only
    where the tile-time model predicts a gain); a zeroed per-device scratch is kept for it.
    """
    _require(a, torch.bfloat16, "a")
    _require(b, torch.bfloat16, "b")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError(f"gemm shapes {tuple(a.shape)} x {tuple(b.shape)}")
    if a.stride(1) != 1 or b.stride(1) != 1:
        raise ValueError("gemm operands must be K-contiguous")
    M, K = a.shape
    N = b.shape[0]
    T, F = (N, M) if weights_as_a else (M, N)
    d = GemmDesc()
    d.a, d.lda, d.b, d.ldb = a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0)
    d.m, d.n, d.k = M, N, K
    d.splits, d.tile_n = splits, tile_n
    d.activation = _lib.FAM_ACT_GELU_TANH if act == "gelu_tanh" else _lib.FAM_ACT_NONE
    d.features_on_a = 1 if weights_as_a else 0
    d.a_is_const = 1 if weights_as_a else 0
    d.b_is_const = 0 if weights_as_a else 1
    d.pdl = 1 if pdl else 0
    d.pair = 1 if pair else 0
    d.bias = _ptr(bias)
    if residual is not None:
        _require(residual, torch.float32, "residual")
        out = residual
        d.epilogue = _lib.FAM_EPI_RESIDUAL
        d.out_dtype = _lib.FAM_DTYPE_F32
        d.gate_w, d.gate_t = _ptr(gate_w), _ptr(gate_t)
        d.tokens_per_batch = tokens_per_batch if tokens_per_batch > 0 else T
        d.first_frame_tokens = first_frame_tokens
        d.gate_batch_stride, d.gate_group_stride = gate_batch_stride, gate_group_stride
    elif splits > 1:
        d.epilogue = _lib.FAM_EPI_PARTIAL
        d.out_dtype = _lib.FAM_DTYPE_F32
        if out is None:
            out = torch.empty((splits, T, F), device=a.device, dtype=torch.float32)
        d.out_stride_split = T * F
    else:
        d.epilogue = _lib.FAM_EPI_STORE
        d.out_dtype = _lib.FAM_DTYPE_BF16 if out_dtype == torch.bfloat16 else _lib.FAM_DTYPE_F32
        if out is None:
            out = torch.empty((T, F), device=a.device, dtype=out_dtype)
    ld = out.stride(-2)
    if weights_as_a:
        d.out_stride_a, d.out_stride_b = 1, ld
    else:
        d.out_stride_a, d.out_stride_b = ld, 1
    d.out = out.data_ptr()
    if split_round not in ("off", "auto", "always"):
        raise ValueError(f"split_round {split_round!r}")
    if split_round != "off":
        sk = _split_scratch(a.device)
        d.scratch, d.scratch_bytes = sk.data_ptr(), sk.numel()
        d.split_round = 1 if split_round == "always" else 0
    check(lib().fam_gemm(C.byref(d), C.c_void_p(_stream())), "fam_gemm")
    return out


def conv3x3(act: torch.Tensor, cin: int, wp: int, H: int, w: torch.Tensor, *, out: torch.Tensor,
            bias: Optional[torch.Tensor] = None, accumulate: bool = False, splits: int = 1) -> torch.Tensor:
    """Implicit-GEMM 3x3 stride-1 convolution on the tensor cores.

    act: bf16 zero-bordered channels-last buffer, row (y + 1) * wp + (x + 1) holds
    position (y, x) of an H x (wp - 2) frame (cin channels, row stride act.stride(0));
    w: bf16 [N, 9 * ceil(cin / 64) * 64], K order (dy, dx, c) with each tap's
    channels zero-padded to whole 64-blocks.  out: fp32 [H * (wp - 2), N] stored, or
    accumulated into when `accumulate`; with splits > 1, out is the fp32 partial
    buffer [splits, H * (wp - 2), N] (no bias)."""
    _require(act, torch.bfloat16, "act")
    _require(w, torch.bfloat16, "w")
    kpt = (cin + 63) // 64
    N, K = w.shape
    if K != 9 * kpt * 64 or act.stride(-1) != 1 or w.stride(1) != 1:
        raise ValueError(f"conv3x3: weight {tuple(w.shape)} for {cin} channels")
    M = H * wp
    Mo = H * (wp - 2)
    d = GemmDesc()
    d.a, d.lda, d.b, d.ldb = act.data_ptr(), act.stride(0), w.data_ptr(), w.stride(0)
    d.m, d.n, d.k = M, N, K
    d.splits = splits
    d.activation = _lib.FAM_ACT_NONE
    d.b_is_const = 1
    d.conv_wp, d.conv_cin, d.conv_a_rows = wp, cin, act.shape[0]
    d.out_dtype = _lib.FAM_DTYPE_F32
    if splits > 1:
        d.epilogue = _lib.FAM_EPI_PARTIAL
        d.out_stride_split = Mo * N
    else:
        d.epilogue = _lib.FAM_EPI_RESIDUAL if accumulate else _lib.FAM_EPI_STORE
        d.bias = _ptr(bias)
        d.tokens_per_batch = Mo
    _require(out, torch.float32, "out")
    d.out, d.out_stride_a, d.out_stride_b = out.data_ptr(), out.stride(-2), 1
    check(lib().fam_gemm(C.byref(d), C.c_void_p(_stream())), "fam_gemm (conv3x3)")
    return out


_SK = {}


def _split_scratch(dev) -> torch.Tensor:
    """Zeroed split-round scratch of the device (every launch leaves it zeroed)."""
    if dev not in _SK:
        n = C.c_size_t()
        check(lib().fam_gemm_split_round_scratch_bytes(C.byref(n)), "fam_gemm_split_round_scratch_bytes")
        _SK[dev] = torch.zeros(n.value, dtype=torch.uint8, device=dev)
    return _SK[dev]


def attention_desc(q, k1, v1, heads, k2=None, v2=None, mask=None, key_mask=None,
                   first_frame_tokens: int = 0, kv_splits: int = 0, out=None):
    """Descriptor for fam_attention over token-major [B, S, H*d] bf16 tensors."""
    from ._abi import AttentionDesc
    B, Sq, HD = q.shape
    hd = HD // heads
    if out is None:
        out = torch.empty_like(q)
    d = AttentionDesc()
    d.batch, d.heads, d.head_dim, d.q_tokens = B, heads, hd, Sq
    d.q, d.q_batch_stride, d.q_token_stride = q.data_ptr(), q.stride(0), q.stride(1)
    d.k1, d.v1 = k1.data_ptr(), v1.data_ptr()
    d.kv1_batch_stride, d.kv1_token_stride, d.kv1_tokens = k1.stride(0), k1.stride(1), k1.shape[1]
    if k2 is not None:
        d.k2, d.v2 = k2.data_ptr(), v2.data_ptr()
        d.kv2_batch_stride, d.kv2_token_stride, d.kv2_tokens = k2.stride(0), k2.stride(1), k2.shape[1]
    if mask is not None:
        d.mask, d.mask_row_stride = mask.data_ptr(), mask.stride(0)
    if key_mask is not None:
        d.key_mask, d.key_mask_batch_stride = key_mask.data_ptr(), key_mask.stride(0)
    d.first_frame_tokens, d.kv_splits = first_frame_tokens, kv_splits
    d.out, d.out_batch_stride, d.out_token_stride = out.data_ptr(), out.stride(0), out.stride(1)
    return d, out


def attention(q, k1, v1, heads, k2=None, v2=None, mask=None, key_mask=None,
              first_frame_tokens: int = 0, kv_splits: int = 0, out=None) -> torch.Tensor:
    """Masked attention (flash_attention of wan_video_dit.py:13-22) through fam_attention.
    Masks are uint8 (nonzero = attend); the caller keeps every tensor alive."""
    for t in (q, k1, v1) + ((k2, v2) if k2 is not None else ()):
        _require(t, torch.bfloat16, "attention operand")
    d, out = attention_desc(q, k1, v1, heads, k2, v2, mask, key_mask, first_frame_tokens,
                            kv_splits, out)
    n = C.c_size_t()
    check(lib().fam_attention_workspace_size(C.byref(d), C.byref(n)), "fam_attention_workspace_size")
    ws = torch.empty(max(1, n.value), dtype=torch.uint8, device=q.device)
    check(lib().fam_attention(C.byref(d), ws.data_ptr(), ws.numel(), C.c_void_p(_stream())),
          "fam_attention")
    out._fam_ws = ws  # keep the workspace alive until the caller drops the output
    return out
