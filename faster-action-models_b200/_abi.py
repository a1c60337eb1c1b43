"""ctypes declarations of the model-level entry points of include/fam.h."""
from __future__ import annotations

import ctypes as C

vp = C.c_void_p


class ActionConfig(C.Structure):
    _fields_ = [("hidden_dim", C.c_int32), ("action_dim", C.c_int32), ("ffn_dim", C.c_int32),
                ("text_dim", C.c_int32), ("freq_dim", C.c_int32), ("num_heads", C.c_int32),
                ("head_dim", C.c_int32), ("num_layers", C.c_int32), ("eps", C.c_float)]


class ActionLayer(C.Structure):
    _fields_ = [(n, vp) for n in (
        "modulation", "qkv_w", "qkv_b", "norm_q", "norm_k", "o_w", "o_b", "norm3_w", "norm3_b",
        "cq_w", "cq_b", "cnorm_q", "cnorm_k", "ckv_w", "ckv_b", "co_w", "co_b", "ffn0_w",
        "ffn0_b", "ffn2_w", "ffn2_b")]


class ActionWeights(C.Structure):
    _fields_ = [(n, vp) for n in (
        "enc_w", "enc_b", "text0_w", "text0_b", "text2_w", "text2_b", "time0_w", "time0_b",
        "time2_w", "time2_b", "tproj_w", "tproj_b", "head_w", "head_b")] + [
        ("layers", C.POINTER(ActionLayer)), ("rope", vp), ("rope_positions", C.c_int32)]


class ActionIO(C.Structure):
    _fields_ = [("batch", C.c_int32), ("action_tokens", C.c_int32),
                ("context_tokens", C.c_int32), ("video_tokens", C.c_int32),
                ("context", vp), ("context_mask", vp), ("video_k", C.POINTER(vp)),
                ("video_v", C.POINTER(vp)), ("video_batch_stride", C.c_int64),
                ("video_token_stride", C.c_int64), ("attn_mask", vp), ("workspace", vp),
                ("workspace_bytes", C.c_size_t)]


def declare(lib) -> None:
    i32, sz = C.c_int32, C.c_size_t
    lib.fam_action_expert_create.argtypes = [C.POINTER(ActionConfig), C.POINTER(ActionWeights),
                                             C.POINTER(vp)]
    lib.fam_action_expert_destroy.argtypes = [vp]
    lib.fam_action_workspace_size.argtypes = [vp, i32, i32, i32, i32, C.POINTER(sz)]
    lib.fam_action_chunk.argtypes = [vp, C.POINTER(ActionIO), vp, C.POINTER(C.c_float),
                                     C.POINTER(C.c_float), i32, vp, i32, vp]
    lib.fam_action_denoise_step.argtypes = [vp, C.POINTER(ActionIO), vp, C.c_float, vp, vp]
    for n in ("fam_action_expert_create", "fam_action_expert_destroy", "fam_action_workspace_size",
              "fam_action_chunk", "fam_action_denoise_step"):
        getattr(lib, n).restype = C.c_int
    declare_counts(lib)
    declare_ops(lib)


def declare_counts(lib) -> None:
    lib.fam_action_launch_count.argtypes = [C.c_void_p, C.POINTER(C.c_int32)]
    lib.fam_action_launch_count.restype = C.c_int


class AttentionDesc(C.Structure):
    _fields_ = [("batch", C.c_int32), ("heads", C.c_int32), ("head_dim", C.c_int32),
                ("q_tokens", C.c_int32), ("q", vp), ("q_batch_stride", C.c_int64),
                ("q_token_stride", C.c_int64), ("k1", vp), ("v1", vp),
                ("kv1_batch_stride", C.c_int64), ("kv1_token_stride", C.c_int64),
                ("kv1_tokens", C.c_int32), ("k2", vp), ("v2", vp),
                ("kv2_batch_stride", C.c_int64), ("kv2_token_stride", C.c_int64),
                ("kv2_tokens", C.c_int32), ("mask", vp), ("mask_row_stride", C.c_int64),
                ("key_mask", vp), ("key_mask_batch_stride", C.c_int64),
                ("first_frame_tokens", C.c_int32), ("kv_splits", C.c_int32), ("out", vp),
                ("out_batch_stride", C.c_int64), ("out_token_stride", C.c_int64)]


def declare_ops(lib) -> None:
    lib.fam_attention_workspace_size.argtypes = [C.POINTER(AttentionDesc), C.POINTER(C.c_size_t)]
    lib.fam_attention.argtypes = [C.POINTER(AttentionDesc), vp, C.c_size_t, vp]
    lib.fam_attention_static_scratch.argtypes = [C.POINTER(AttentionDesc), vp]
    for n in ("fam_attention_workspace_size", "fam_attention", "fam_attention_static_scratch"):
        getattr(lib, n).restype = C.c_int
