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


class ActionStacks(C.Structure):
    _fields_ = [(n, vp) for n in (
        "qkv_w", "o_w", "cq_w", "co_w", "ffn0_w", "ffn2_w", "qkv_b", "o_b", "cq_b", "co_b",
        "ffn0_b", "ffn2_b", "norm_q", "norm_k", "cnorm_q", "norm3_w", "norm3_b", "modulation",
        "ckv_w", "ckv_b", "cnorm_k")]


class ActionWeights(C.Structure):
    _fields_ = [(n, vp) for n in (
        "enc_w", "enc_b", "text0_w", "text0_b", "text2_w", "text2_b", "time0_w", "time0_b",
        "time2_w", "time2_b", "tproj_w", "tproj_b", "head_w", "head_b")] + [
        ("layers", C.POINTER(ActionLayer)), ("rope", vp), ("rope_positions", C.c_int32),
        ("stacks", C.POINTER(ActionStacks))]


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
    declare_vae(lib)
    declare_ops(lib)
    declare_cae(lib)
    declare_video(lib)


def declare_counts(lib) -> None:
    lib.fam_action_launch_count.argtypes = [C.c_void_p, C.POINTER(C.c_int32)]
    lib.fam_action_launch_count.restype = C.c_int
    lib.fam_action_set_mode.argtypes = [C.c_void_p, C.c_int32]
    lib.fam_action_set_mode.restype = C.c_int
    lib.fam_action_last_path.argtypes = [C.c_void_p, C.POINTER(C.c_int32)]
    lib.fam_action_last_path.restype = C.c_int
    lib.fam_selftest_bounded_wait.argtypes = [C.c_void_p]
    lib.fam_selftest_bounded_wait.restype = C.c_int
    lib.fam_action_set_kernel_events.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
    lib.fam_action_set_kernel_events.restype = C.c_int


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


fp = C.c_void_p  # const float* (device)


class CaeLayer(C.Structure):
    _fields_ = [(n, fp) for n in (
        "modulation", "qkv_w", "qkv_b", "norm_q", "norm_k", "o_w", "o_b", "norm3_w", "norm3_b",
        "cq_w", "cq_b", "cnorm_q", "cnorm_k", "ckv_w", "ckv_b", "co_w", "co_b", "ffn0_w",
        "ffn0_b", "ffn2_w", "ffn2_b")]


class CaeWeights(C.Structure):
    _fields_ = [(n, fp) for n in (
        "enc_w", "enc_b", "text0_w", "text0_b", "text2_w", "text2_b", "time0_w", "time0_b",
        "time2_w", "time2_b", "tproj_w", "tproj_b", "head_w", "head_b")] + [
        ("layers", C.POINTER(CaeLayer)), ("rope", fp), ("rope_positions", C.c_int32)]


class DecoderConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("action_dim", "action_horizon", "num_tokens",
                                         "latent_dim", "hidden", "num_suites")]


class DecoderStage(C.Structure):
    _fields_ = [(n, fp) for n in ("convt_w", "convt_b", "gn0_w", "gn0_b", "c1_w", "c1_b",
                                  "gn1_w", "gn1_b", "c2_w", "c2_b", "gn2_w", "gn2_b")] + [
        ("stride", C.c_int32)]


class DecoderWeights(C.Structure):
    _fields_ = [("in_w", fp), ("in_b", fp), ("out_w", fp), ("out_b", fp), ("suite_embed", fp),
                ("stages", C.POINTER(DecoderStage)), ("num_stages", C.c_int32),
                ("latent_std", fp), ("latent_mean", fp)]


def declare_cae(lib) -> None:
    i32, sz = C.c_int32, C.c_size_t
    lib.fam_cae_workspace_size.argtypes = [C.POINTER(ActionConfig), i32, i32, C.POINTER(sz)]
    lib.fam_cae_chunk.argtypes = [C.POINTER(ActionConfig), C.POINTER(CaeWeights), i32, i32, vp,
                                  i32, i32, vp, vp, C.POINTER(C.c_float), C.POINTER(C.c_float),
                                  i32, vp, vp, sz, vp]
    lib.fam_cae_status.argtypes = [C.POINTER(ActionConfig), i32, i32, vp, C.POINTER(i32), vp]
    lib.fam_decoder_workspace_size.argtypes = [C.POINTER(DecoderConfig), C.POINTER(DecoderWeights),
                                               i32, C.POINTER(sz)]
    lib.fam_action_decode.argtypes = [C.POINTER(DecoderConfig), C.POINTER(DecoderWeights), i32,
                                      vp, vp, vp, vp, sz, vp]
    lib.fam_cae_decode_workspace_size.argtypes = [C.POINTER(ActionConfig), C.POINTER(DecoderConfig),
                                                  C.POINTER(DecoderWeights), i32, i32, C.POINTER(sz)]
    lib.fam_cae_chunk_decode.argtypes = [C.POINTER(ActionConfig), C.POINTER(CaeWeights), i32, i32, vp,
                                         i32, i32, vp, vp, C.POINTER(C.c_float), C.POINTER(C.c_float),
                                         i32, vp, C.POINTER(DecoderConfig), C.POINTER(DecoderWeights), vp, vp,
                                         i32, C.POINTER(i32), vp, sz, vp]
    for n in ("fam_cae_workspace_size", "fam_cae_chunk", "fam_cae_status", "fam_decoder_workspace_size",
              "fam_action_decode", "fam_cae_decode_workspace_size", "fam_cae_chunk_decode"):
        getattr(lib, n).restype = C.c_int


class VideoConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("hidden_dim", "in_dim", "ffn_dim", "text_dim", "freq_dim",
                                         "num_heads", "head_dim", "num_layers", "patch_t",
                                         "patch_h", "patch_w")] + [("eps", C.c_float)]


class VideoWeights(C.Structure):
    _fields_ = [(n, vp) for n in ("patch_w", "patch_b", "text0_w", "text0_b", "text2_w", "text2_b",
                                  "time0_w", "time0_b", "time2_w", "time2_b", "tproj_w",
                                  "tproj_b")] + [("layers", C.POINTER(ActionLayer))]


class VideoIO(C.Structure):
    _fields_ = [("batch", C.c_int32), ("frames", C.c_int32), ("height", C.c_int32),
                ("width", C.c_int32), ("context_tokens", C.c_int32), ("latents", vp),
                ("timesteps", C.POINTER(C.c_float)), ("context", vp), ("context_mask", vp),
                ("rope", vp), ("first_frame_causal", C.c_int32), ("cache_k", C.POINTER(vp)),
                ("cache_v", C.POINTER(vp)), ("hidden_out", vp), ("workspace", vp),
                ("workspace_bytes", C.c_size_t), ("t_out", vp)]


def declare_video(lib) -> None:
    i32, sz = C.c_int32, C.c_size_t
    lib.fam_video_expert_create.argtypes = [C.POINTER(VideoConfig), C.POINTER(VideoWeights),
                                            C.POINTER(vp)]
    lib.fam_video_expert_destroy.argtypes = [vp]
    lib.fam_video_workspace_size.argtypes = [vp, i32, i32, i32, C.POINTER(sz)]
    lib.fam_video_prefill.argtypes = [vp, C.POINTER(VideoIO), i32, vp]
    lib.fam_video_launch_count.argtypes = [vp, C.POINTER(C.c_int32)]
    lib.fam_video_head_norm.argtypes = [vp, vp, vp, i32, i32, i32, i32, C.c_float, vp, vp]
    lib.fam_video_unpatchify.argtypes = [vp, i32, i32, i32, i32, i32, i32, i32, i32, vp, vp]
    for n in ("fam_video_expert_create", "fam_video_expert_destroy", "fam_video_workspace_size",
              "fam_video_prefill", "fam_video_launch_count", "fam_video_head_norm", "fam_video_unpatchify"):
        getattr(lib, n).restype = C.c_int


def declare_vae(lib) -> None:
    """Wan2.2 VAE encode pieces (include/fam.h, fam_vae_*)."""
    i32, i64, f32 = C.c_int32, C.c_int64, C.c_float
    fp = C.POINTER(C.c_float)
    lib.fam_vae_patchify.argtypes = [vp, i32, i32, vp, i64, i32, vp]
    lib.fam_vae_im2col.argtypes = [vp, i64, i32, i32, i32, i32, i32, i32, i32, vp, i64, vp]
    lib.fam_vae_rms.argtypes = [vp, i64, i64, i32, vp, i32, vp, i64, i32, vp, i64, vp]
    lib.fam_vae_avg_down_add.argtypes = [vp, i64, i32, i32, i32, i32, i32, i32, vp, i64, vp]
    lib.fam_vae_softmax.argtypes = [vp, i64, i32, i32, f32, vp, i64, vp]
    lib.fam_vae_transpose.argtypes = [vp, i64, i32, i32, vp, i64, vp]
    lib.fam_vae_latent.argtypes = [vp, i64, i64, i32, vp, vp, vp, vp]
    lib.fam_vae_splitk_reduce.argtypes = [vp, i32, i64, i32, vp, vp, i64, i32, vp]
    for n in ("fam_vae_patchify", "fam_vae_im2col", "fam_vae_rms", "fam_vae_avg_down_add", "fam_vae_softmax",
              "fam_vae_transpose", "fam_vae_latent", "fam_vae_splitk_reduce"):
        getattr(lib, n).restype = C.c_int
