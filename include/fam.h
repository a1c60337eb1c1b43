/*
 * libfam — B200 (sm_100a) kernels for the per-action-chunk denoising path of
 * the FastWAM world action models.  Plain C ABI: device pointers, sizes and a
 * cudaStream_t passed as void*; no torch types; every entry point returns an
 * int status (FAM_OK == 0) and fam_last_error() describes the last failure of
 * the calling thread.  No entry point allocates device memory during a call
 * except the one-time status word per device and the packed-weight handles
 * documented below; outputs and workspaces are caller-owned.
 *
 * Reference interfaces replaced (paths relative to the reference project):
 *   fam_gemm                  nn.Linear calls of DiTBlock / ActionDiT / WanVideoDiT
 *                             (FastWAM/src/fastwam/models/wan22/wan_video_dit.py:170-246,
 *                              action_dit.py:73-97)
 * The model-level entry points are declared further down with their own
 * citations.
 */
#ifndef FAM_H_
#define FAM_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FAM_API __attribute__((visibility("default")))
#else
#define FAM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FAM_VERSION_MAJOR 0
#define FAM_VERSION_MINOR 1
#define FAM_VERSION_PATCH 0

/* status codes */
#define FAM_OK 0
#define FAM_ERR_INVALID 1  /* bad argument or unsupported shape */
#define FAM_ERR_CUDA 2     /* a CUDA runtime call failed */
#define FAM_ERR_DEVICE 3   /* a kernel reported an error through the status word */

/* dtypes */
#define FAM_DTYPE_BF16 0
#define FAM_DTYPE_F32 1

/* GEMM epilogues */
#define FAM_EPI_STORE 0    /* out = act(acc + bias) */
#define FAM_EPI_PARTIAL 1  /* out[split] = acc (fp32 split-K partials, no bias) */
#define FAM_EPI_RESIDUAL 2 /* out_f32 += gate * (acc + bias) */

#define FAM_ACT_NONE 0
#define FAM_ACT_GELU_TANH 1
#define FAM_ACT_SILU 2

FAM_API int fam_version(int* major, int* minor, int* patch);

/* Copies the calling thread's last error message (NUL-terminated). */
FAM_API int fam_last_error(char* buf, size_t len);

/* Reads the current device's status word (0 = healthy; otherwise the code of
 * the first kernel that gave up a bounded wait or rejected its arguments).
 * Synchronizes `stream`.  reset != 0 clears the word afterwards. */
FAM_API int fam_device_status(int* code, int reset, void* stream);

/* Self-test of the failure path (no counterpart in the reference): launches
 * one thread that waits on an mbarrier nothing completes.  The wait gives up
 * after its 1 s %globaltimer limit, records code 1 (a consumer wait expired)
 * in the device status word and the kernel returns: no fault, the context
 * stays usable.  Read the outcome with fam_device_status after the stream. */
FAM_API int fam_selftest_bounded_wait(void* stream);

/* D[m][n] = sum_k A[m][k] * B[n][k]  on the tcgen05 tensor cores.
 * A: bf16 [m, k] row stride lda; B: bf16 [n, k] row stride ldb (both K-major,
 * 16-byte aligned, k and strides multiples of 8).  The output element for
 * (m, n) is out[m * out_stride_a + n * out_stride_b] (+ split * out_stride_split
 * for FAM_EPI_PARTIAL).  features_on_a says which index is the output feature
 * (selects bias[feature] and the residual gate); the other index is the token.
 * Residual gate for token t, feature f:
 *   gate_w[f] + gate_t[(t / tokens_per_batch) * gate_batch_stride
 *                      + (first_frame_tokens > 0 && t % tokens_per_batch >= first_frame_tokens
 *                         ? gate_group_stride : 0) + f]
 * (gate_t == NULL: gate 1).  tile_n = 0 picks the MMA N tile (16..256). */
typedef struct fam_gemm_desc {
  const void* a;
  int64_t lda;
  const void* b;
  int64_t ldb;
  int32_t m, n, k;
  int32_t splits;
  int32_t tile_n;
  int32_t epilogue;
  int32_t activation;
  int32_t out_dtype;
  int32_t features_on_a;
  int32_t a_is_const; /* operand is constant across a launch chain (prefetched before the PDL wait) */
  int32_t b_is_const;
  int32_t pdl;        /* launch with programmatic stream serialization */
  void* out;
  int64_t out_stride_a;
  int64_t out_stride_b;
  int64_t out_stride_split;
  const void* bias;   /* bf16 [features] or NULL */
  const void* gate_w; /* bf16 [features] or NULL */
  const void* gate_t; /* f32 or NULL */
  int32_t tokens_per_batch;
  int32_t first_frame_tokens;
  int64_t gate_batch_stride;
  int64_t gate_group_stride;
  /* Optional split-round scratch (NULL: none), fam_gemm_split_round_scratch_bytes
   * bytes, zeroed once before its first use (every launch leaves it zeroed).
   * With it a many-tile problem may run 256-wide tiles whole-round-robin and
   * split each tile of the last, partial round into 2..4 k-pieces on the idle
   * SMs, summed in a fixed order (deterministic).  split_round = 0: only when
   * the tile-time model predicts a gain; 1: whenever the last round is partial. */
  void* scratch;
  size_t scratch_bytes;
  int32_t split_round;
  /* Implicit 3x3 stride-1 convolution when conv_wp > 0: a is a zero-bordered
   * channels-last activation buffer [conv_a_rows, conv_cin] (row stride lda)
   * whose rows are the padded positions y * conv_wp + x of a frame of width
   * conv_wp - 2; m = H * conv_wp; b is [n, k] with k = 9 * ceil(conv_cin / 64) * 64
   * (per tap (dy, dx) a block of the input channels, zero-padded to 64);
   * output row y * (conv_wp - 2) + x for x < conv_wp - 2. */
  int32_t conv_wp;
  int32_t conv_cin;
  int64_t conv_a_rows;
  /* 1: a many-tile problem that would run 256-wide tiles may run them on CTA
   * pairs (tcgen05 cta_group::2, 256 x 256 tiles, half of B per CTA); 0: off. */
  int32_t pair;
} fam_gemm_desc;

FAM_API int fam_gemm(const fam_gemm_desc* desc, void* stream);
FAM_API int fam_gemm_split_round_scratch_bytes(size_t* bytes);

/* Masked multi-head attention, softmax(q k^T / sqrt(d)) v with a bool mask,
 * over the concatenation of two key/value sources (source 2 may be empty).
 * Replaces flash_attention / MoT._mixed_attention
 * (FastWAM/src/fastwam/models/wan22/wan_video_dit.py:13-22, mot.py:88-103,
 * 506-512, 560-566).  All tensors bf16, token-major with head h at columns
 * [h * head_dim, (h + 1) * head_dim) of each row:
 *   q[b * q_batch_stride + t * q_token_stride + h * head_dim + i]
 * Keys j < kv1_tokens come from source 1, the rest from source 2.  A key is
 * attended when mask[t * mask_row_stride + j] != 0 (NULL: all), key_mask
 * [b * key_mask_batch_stride + j] != 0 (NULL: all) and, when
 * first_frame_tokens > 0, queries t < first_frame_tokens see only keys
 * j < first_frame_tokens.  head_dim is 64 or 128.  With several key splits
 * the partial results go to the caller's workspace. */
typedef struct fam_attention_desc {
  int32_t batch, heads, head_dim, q_tokens;
  const void* q;
  int64_t q_batch_stride, q_token_stride;
  const void* k1;
  const void* v1;
  int64_t kv1_batch_stride, kv1_token_stride;
  int32_t kv1_tokens;
  const void* k2;
  const void* v2;
  int64_t kv2_batch_stride, kv2_token_stride;
  int32_t kv2_tokens;
  const uint8_t* mask;
  int64_t mask_row_stride;
  const uint8_t* key_mask;
  int64_t key_mask_batch_stride;
  int32_t first_frame_tokens;
  int32_t kv_splits; /* 0: chosen to fill the GPU */
  void* out;
  int64_t out_batch_stride, out_token_stride;
} fam_attention_desc;

/* Bytes of device workspace fam_attention needs for this descriptor: 0 when
 * the call runs without split partials (one CTA per batch and head, e.g. the
 * tcgen05 short-query kernel that a descriptor with kv_splits = 0, head_dim
 * 64, q_tokens <= 32 and batch x heads >= 128 selects). */
FAM_API int fam_attention_workspace_size(const fam_attention_desc* desc, size_t* bytes);
FAM_API int fam_attention(const fam_attention_desc* desc, void* workspace, size_t workspace_bytes,
                          void* stream);

/* fam_attention for callers that cannot allocate device memory (an embedded
 * plugin that does not own the process's allocator, a control loop that
 * forbids allocation after start-up, an FFI host without a device
 * allocator).  No counterpart in the reference: its PyTorch path allocates
 * freely.  The split partials live in a static device array of 8 MiB per GPU
 * (held by every GPU that loads the library until exit); calls needing more
 * are rejected with FAM_ERR_INVALID.  Allocates nothing.  Every call outside a
 * stream capture looks the array's address up (a reset context is followed);
 * make one call on each device before any capture there, and at start-up:
 * under CUDA's lazy module loading that first call loads the library's device
 * image, this array included.  A descriptor with kv_splits = 0 that the
 * tcgen05 short-query kernel takes (head_dim 64, q_tokens <= 32, batch x heads
 * >= 128) runs that kernel, which needs no scratch; every other descriptor
 * runs the split-KV mma.sync kernel (not the tcgen05 long-self-attention
 * kernel, which needs a transposed-V workspace).  All calls on a device share
 * the array: calls that overlap on the GPU race. */
FAM_API int fam_attention_static_scratch(const fam_attention_desc* desc, void* stream);

/* ======================================================================
 * Action expert (ActionDiT + MoT action path) — BASELINE configs 1 and 3.
 *
 * Replaces, for a bf16 model:
 *   ActionDiT.prepare / post         FastWAM/src/fastwam/models/wan22/action_dit.py:312-331
 *   MoT.forward_action_with_video_cache_tensor   .../wan22/mot.py:528-578
 *   FastWAM._denoise_action_with_video_cache     .../wan22/fastwam.py:771-804
 *   the Euler loop of FastWAM.infer_action       .../wan22/fastwam.py:1241-1263
 *   WanContinuousFlowMatchScheduler.step         .../wan22/schedulers/scheduler_continuous.py:82-88
 * Weights are the reference state_dict tensors (bf16, device resident); the
 * q/k/v projections of each block are passed concatenated ([3*HD, D] rows
 * q, k, v) and the cross-attention k/v concatenated ([2*HD, D]).  The
 * handle keeps the pointers (the caller owns the memory).
 * ====================================================================== */
typedef struct fam_action_config {
  int32_t hidden_dim;   /* D */
  int32_t action_dim;   /* A */
  int32_t ffn_dim;      /* F */
  int32_t text_dim;     /* T */
  int32_t freq_dim;     /* sinusoid width (256) */
  int32_t num_heads;    /* H */
  int32_t head_dim;     /* d (64 or 128); HD = H * d */
  int32_t num_layers;   /* L */
  float eps;            /* LayerNorm / RMSNorm eps */
} fam_action_config;

typedef struct fam_action_layer {
  const void* modulation;                  /* [6, D]            blocks.i.modulation */
  const void* qkv_w; const void* qkv_b;    /* [3HD, D], [3HD]   self_attn.{q,k,v} */
  const void* norm_q; const void* norm_k;  /* [HD]              self_attn.norm_{q,k} */
  const void* o_w; const void* o_b;        /* [D, HD], [D]      self_attn.o */
  const void* norm3_w; const void* norm3_b;/* [D]               norm3 */
  const void* cq_w; const void* cq_b;      /* [HD, D], [HD]     cross_attn.q */
  const void* cnorm_q; const void* cnorm_k;/* [HD]              cross_attn.norm_{q,k} */
  const void* ckv_w; const void* ckv_b;    /* [2HD, D], [2HD]   cross_attn.{k,v} */
  const void* co_w; const void* co_b;      /* [D, HD], [D]      cross_attn.o */
  const void* ffn0_w; const void* ffn0_b;  /* [F, D], [F]       ffn.0 */
  const void* ffn2_w; const void* ffn2_b;  /* [D, F], [D]       ffn.2 */
} fam_action_layer;

/* Optional (no counterpart in the reference, whose blocks are separate
 * modules): the same per-block tensors stacked over the blocks, contiguous
 * (block l of a stack starts at l * rows).  When given, fam_action_chunk can
 * run the fused persistent chunk kernel (batch 1, <= 32 action tokens,
 * action_dim <= 16, head_dim 64, hidden 512 or 1024, other
 * widths multiples of 128, <= 256 context tokens, <= 2560 video + action
 * keys); the layer pointers must point into these stacks. */
typedef struct fam_action_stacks {
  const void *qkv_w, *o_w, *cq_w, *co_w, *ffn0_w, *ffn2_w;   /* [L*N, K] */
  const void *qkv_b, *o_b, *cq_b, *co_b, *ffn0_b, *ffn2_b;   /* [L*N] */
  const void *norm_q, *norm_k, *cnorm_q;                     /* [L*HD] */
  const void *norm3_w, *norm3_b;                             /* [L*D] */
  const void *modulation;                                    /* [L*6*D] */
  /* optional (NULL: per-block prologue launches): cross-attention K/V
   * projection and k RMSNorm weight stacked over the blocks, for one batched
   * context K/V GEMM per chunk */
  const void *ckv_w, *ckv_b;                                 /* [L*2HD, D], [L*2HD] */
  const void *cnorm_k;                                       /* [L*HD] */
} fam_action_stacks;

typedef struct fam_action_weights {
  const void* enc_w; const void* enc_b;        /* [D, A]  action_encoder */
  const void* text0_w; const void* text0_b;    /* [D, T]  text_embedding.0 */
  const void* text2_w; const void* text2_b;    /* [D, D]  text_embedding.2 */
  const void* time0_w; const void* time0_b;    /* [D, 256] time_embedding.0 */
  const void* time2_w; const void* time2_b;    /* [D, D]  time_embedding.2 */
  const void* tproj_w; const void* tproj_b;    /* [6D, D] time_projection.1 */
  const void* head_w; const void* head_b;      /* [A, D]  head */
  const fam_action_layer* layers;              /* host array [L] */
  const void* rope;        /* f32 [rope_positions, d/2, 2] (cos, sin) of precompute_freqs_cis(d) */
  int32_t rope_positions;
  const fam_action_stacks* stacks; /* NULL: launch-chain path only */
} fam_action_weights;

/* Execution path of fam_action_chunk: FAM_ACTION_AUTO picks the fused
 * persistent kernel when the call qualifies, FAM_ACTION_CHAIN always runs the
 * chain of per-op kernels, FAM_ACTION_FUSED requires the fused kernel. */
#define FAM_ACTION_AUTO 0
#define FAM_ACTION_CHAIN 1
#define FAM_ACTION_FUSED 2

typedef struct fam_action_expert fam_action_expert;

/* Per-call inputs.  All device pointers; the K/V cache of layer l is
 * video_k[l][b * video_batch_stride + s * video_token_stride + c] (c < HD),
 * i.e. the reference's list of [B, Sv, HD] tensors (MoT.prefill_video_cache_tensor
 * output).  attn_mask is the [Sa, Sv + Sa] action-row slice of the MoT mask
 * (True = attend; NULL = all True).  context_mask [B, C] (NULL = all valid). */
typedef struct fam_action_io {
  int32_t batch;
  int32_t action_tokens;     /* Sa */
  int32_t context_tokens;    /* C */
  int32_t video_tokens;      /* Sv (0: standalone expert, no cache) */
  const void* context;       /* bf16 [B, C, T] */
  const uint8_t* context_mask;
  const void* const* video_k;/* host array [L] of device pointers */
  const void* const* video_v;
  int64_t video_batch_stride;
  int64_t video_token_stride;
  const uint8_t* attn_mask;
  void* workspace;
  size_t workspace_bytes;
} fam_action_io;

FAM_API int fam_action_expert_create(const fam_action_config* cfg, const fam_action_weights* w,
                                     fam_action_expert** out);
FAM_API int fam_action_expert_destroy(fam_action_expert* e);

/* Workspace bytes for a call with these sizes (max_steps >= num_steps of the call). */
FAM_API int fam_action_workspace_size(const fam_action_expert* e, int32_t batch,
                                      int32_t action_tokens, int32_t context_tokens,
                                      int32_t max_steps, size_t* bytes);

/* One whole action chunk: num_steps Euler steps at the given (already
 * dtype-rounded) timesteps and deltas (host arrays), latent updated in place
 * (bf16 [B, Sa, A]).  velocity_trace (bf16 [num_steps, B, Sa, A]) is optional.
 * use_graph != 0 captures the launch sequence once into a CUDA graph and
 * replays it while the pointers and sizes stay the same. */
FAM_API int fam_action_chunk(fam_action_expert* e, const fam_action_io* io, void* latent,
                             const float* timesteps, const float* deltas, int32_t num_steps,
                             void* velocity_trace, int32_t use_graph, void* stream);

/* One model evaluation (FastWAM._denoise_action_with_video_cache): the
 * velocity bf16 [B, Sa, A] for latent at the given timestep; no Euler update. */
FAM_API int fam_action_denoise_step(fam_action_expert* e, const fam_action_io* io,
                                    const void* latent, float timestep, void* velocity,
                                    void* stream);

/* Number of kernels the last fam_action_chunk / fam_action_denoise_step call
 * enqueued (a graph replay launches the same set). */
FAM_API int fam_action_launch_count(const fam_action_expert* e, int32_t* count);

/* Selects the execution path (FAM_ACTION_AUTO / _CHAIN / _FUSED) and reports
 * the path the last fam_action_chunk call took (1 chain, 2 fused). */
FAM_API int fam_action_set_mode(fam_action_expert* e, int32_t mode);
FAM_API int fam_action_last_path(const fam_action_expert* e, int32_t* path);

/* Measurement hook (no counterpart in the reference): with two cudaEvent_t
 * handles set, every fused-path fam_action_chunk called with use_graph = 0
 * records start / stop on its stream immediately around the fused kernel
 * launch, so a caller can time that kernel alone (graph replays record
 * nothing).  NULL, NULL clears the hook. */
FAM_API int fam_action_set_kernel_events(fam_action_expert* e, void* start_event, void* stop_event);

/* ======================================================================
 * Video DiT prefill (WanVideoDiT backbone) — BASELINE config 2.
 *
 * Replaces, for a bf16 model with separated per-token timesteps:
 *   WanVideoDiT.prepare              FastWAM/src/fastwam/models/wan22/wan_video_dit.py:640-720
 *   MoT.prefill_video_cache_tensor   .../wan22/mot.py:474-526
 * The first latent frame's tokens use timestep 0 (wan_video_dit.py:671-677),
 * so the time MLP runs on two rows per sample and every block reads the
 * (first frame, rest) modulation pair.  Outputs per block the post-RMSNorm +
 * RoPE K and the raw V, [B, S, H*d] bf16 each, and optionally the final token
 * states (fp32 [B, S, D]; computing them adds the last block's post block).
 * Blocks use the fam_action_layer layout.
 * ====================================================================== */
typedef struct fam_video_config {
  int32_t hidden_dim, in_dim, ffn_dim, text_dim, freq_dim, num_heads, head_dim, num_layers;
  int32_t patch_t, patch_h, patch_w;
  float eps;
} fam_video_config;

typedef struct fam_video_weights {
  const void *patch_w, *patch_b;   /* [D, in*pt*ph*pw] (Conv3d weight flattened), [D] */
  const void *text0_w, *text0_b, *text2_w, *text2_b;
  const void *time0_w, *time0_b, *time2_w, *time2_b, *tproj_w, *tproj_b;
  const fam_action_layer* layers;  /* host array [L] */
} fam_video_weights;

typedef struct fam_video_expert fam_video_expert;

typedef struct fam_video_io {
  int32_t batch, frames, height, width; /* latent grid [B, in, F, H, W] */
  int32_t context_tokens;
  const void* latents;        /* bf16 [B, in, F, H, W] */
  const float* timesteps;     /* host [B], already rounded to the model dtype */
  const void* context;        /* bf16 [B, C, T] */
  const uint8_t* context_mask;/* [B, C] or NULL */
  const float* rope;          /* f32 [S, d/2, 2] per token (3-D RoPE of the grid) */
  int32_t first_frame_causal; /* 1: first-frame tokens attend only to the first frame */
  void* const* cache_k;       /* host array [L] of device [B, S, H*d] bf16 */
  void* const* cache_v;
  float* hidden_out;          /* f32 [B, S, D] or NULL */
  void* workspace;
  size_t workspace_bytes;
  void* t_out;                /* bf16 [B, 2, D] time embedding t (first-frame t = 0 row, then the
                               * other frames' row) for the output head, or NULL */
} fam_video_io;

FAM_API int fam_video_expert_create(const fam_video_config* cfg, const fam_video_weights* w,
                                    fam_video_expert** out);
FAM_API int fam_video_expert_destroy(fam_video_expert* e);
FAM_API int fam_video_workspace_size(const fam_video_expert* e, int32_t batch, int32_t tokens,
                                     int32_t context_tokens, size_t* bytes);
FAM_API int fam_video_prefill(fam_video_expert* e, const fam_video_io* io, int32_t use_graph,
                              void* stream);
FAM_API int fam_video_launch_count(const fam_video_expert* e, int32_t* count);

/* ======================================================================
 * Compact action expert (hidden width <= 64, e.g. the CAE expert of
 * CAE-FastWAM and BASELINE config 0): the whole Euler loop of a chunk in two
 * launches — the context side (text embedding + every block's cross K/V) and
 * one persistent kernel per sample running every step x block.  fp32
 * arithmetic and fp32 weights (the reference's fp32 configuration).
 *
 * Replaces ActionDiT.forward called in the flow-matching loop
 *   FastWAM/src/fastwam/models/wan22/action_dit.py:312-362,
 *   .../wan22/wan_video_dit.py:248-267 (DiTBlock.forward),
 *   .../wan22/fastwam.py:1241-1263 and scheduler_continuous.py:82-88.
 * Limits: tokens <= 32, hidden <= 64, heads*head_dim <= 64, head_dim <= 32,
 * ffn <= 256, blocks <= 32, action channels <= 64.
 * ====================================================================== */
typedef struct fam_cae_layer {
  const float *modulation, *qkv_w, *qkv_b, *norm_q, *norm_k, *o_w, *o_b, *norm3_w, *norm3_b,
      *cq_w, *cq_b, *cnorm_q, *cnorm_k, *ckv_w, *ckv_b, *co_w, *co_b, *ffn0_w, *ffn0_b, *ffn2_w,
      *ffn2_b; /* same shapes and meaning as fam_action_layer, fp32 */
} fam_cae_layer;

typedef struct fam_cae_weights {
  const float *enc_w, *enc_b, *text0_w, *text0_b, *text2_w, *text2_b, *time0_w, *time0_b,
      *time2_w, *time2_b, *tproj_w, *tproj_b, *head_w, *head_b;
  const fam_cae_layer* layers; /* host array [num_layers] */
  const float* rope;           /* f32 [rope_positions, head_dim/2, 2] */
  int32_t rope_positions;
} fam_cae_weights;

/* Workspace bytes of fam_cae_chunk for batch x context_tokens. */
FAM_API int fam_cae_workspace_size(const fam_action_config* cfg, int32_t batch,
                                   int32_t context_tokens, size_t* bytes);

/* latent: f32 [B, S, A] updated in place; context: [B, C, T] f32 (context_bf16
 * == 0) or bf16; context_mask u8 [B, C] or NULL; velocity_trace f32
 * [num_steps, B, S, A] or NULL; timesteps / deltas host arrays [num_steps]. */
FAM_API int fam_cae_chunk(const fam_action_config* cfg, const fam_cae_weights* w, int32_t batch,
                          int32_t tokens, const void* context, int32_t context_bf16,
                          int32_t context_tokens, const uint8_t* context_mask, float* latent,
                          const float* timesteps, const float* deltas, int32_t num_steps,
                          float* velocity_trace, void* workspace, size_t workspace_bytes,
                          void* stream);

/* fam_cae_chunk followed by the Action-VAE decode of the final latents
 * (FastWAM.decode_action_latents -> ActionAE.decode, fastwam.py:855-863,
 * action_ae.py:154-187): actions f32 [B, horizon, A], suite_ids int32 [B] or
 * NULL.  The decode can run in the epilogue of the staged step kernel (no
 * further launch) when the decoder has one upsampling stage of stride 2 or 4
 * and its hidden channels split into whole GroupNorm groups over the CTAs of a
 * sample's cluster; otherwise the decoder's own kernels follow.  decode_mode:
 * FAM_DECODE_AUTO takes the epilogue when it qualifies and batch >= 4 (each
 * sample decodes on its own cluster of at most 4 SMs, flat in the batch,
 * while the separate launches grow with it: they are as fast or faster at
 * batch 1, the epilogue is faster at batch 16), FAM_DECODE_FUSED whenever it
 * qualifies, FAM_DECODE_SEPARATE never.
 * *decode_fused (may be NULL) reports which ran.  `latent` receives the final
 * latents either way.  Workspace: fam_cae_decode_workspace_size. */
#define FAM_DECODE_AUTO 0
#define FAM_DECODE_FUSED 1
#define FAM_DECODE_SEPARATE 2
FAM_API int fam_cae_decode_workspace_size(const fam_action_config* cfg, const struct fam_decoder_config* dcfg,
                                          const struct fam_decoder_weights* dw, int32_t batch,
                                          int32_t context_tokens, size_t* bytes);
FAM_API int fam_cae_chunk_decode(const fam_action_config* cfg, const fam_cae_weights* w, int32_t batch,
                                 int32_t tokens, const void* context, int32_t context_bf16,
                                 int32_t context_tokens, const uint8_t* context_mask, float* latent,
                                 const float* timesteps, const float* deltas, int32_t num_steps,
                                 float* velocity_trace, const struct fam_decoder_config* dcfg,
                                 const struct fam_decoder_weights* dw, const int32_t* suite_ids,
                                 float* actions, int32_t decode_mode, int32_t* decode_fused, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Status word of the last fam_cae_chunk on this workspace (synchronizes the
 * stream): 0, or nonzero when a bounded device wait (a bulk copy that did not
 * land within the wait limit) gave up and the outputs are not valid. */
FAM_API int fam_cae_status(const fam_action_config* cfg, int32_t batch, int32_t context_tokens,
                           const void* workspace, int32_t* status, void* stream);

/* ======================================================================
 * Action-VAE decoder (ActionAE.decode / ActionDecoder.forward,
 * FastWAM/src/fastwam/models/action_ae.py:123-166, 184-187), fp32:
 * input_proj (+ suite embedding) -> per stride s: ConvTranspose1d(h, h, 2s, s,
 * s/2) -> GroupNorm(min(8, h)) -> SiLU -> residual [Conv1d k3 -> GN -> SiLU ->
 * Conv1d k3 -> GN] -> crop / zero-pad to action_horizon -> output_proj.
 * ====================================================================== */
typedef struct fam_decoder_config {
  int32_t action_dim, action_horizon, num_tokens, latent_dim, hidden, num_suites;
} fam_decoder_config;

typedef struct fam_decoder_stage {
  const float *convt_w, *convt_b; /* up.{4i}: [h, h, 2s], [h] */
  const float *gn0_w, *gn0_b;     /* up.{4i+1} */
  const float *c1_w, *c1_b;       /* up.{4i+3}.net.0: [h, h, 3] */
  const float *gn1_w, *gn1_b;     /* up.{4i+3}.net.1 */
  const float *c2_w, *c2_b;       /* up.{4i+3}.net.3 */
  const float *gn2_w, *gn2_b;     /* up.{4i+3}.net.4 */
  int32_t stride;
} fam_decoder_stage;

typedef struct fam_decoder_weights {
  const float *in_w, *in_b;       /* input_proj [h, latent] */
  const float *out_w, *out_b;     /* output_proj [A, h] */
  const float* suite_embed;       /* [num_suites, h] or NULL */
  const fam_decoder_stage* stages;/* host array */
  int32_t num_stages;
  /* Latent un-normalisation of DiT4DiT._decode_action_predictions
   * (DiT4DiT/model/framework/DiT4DiT.py:403-406): when both are non-NULL the
   * decoder reads z * latent_std + latent_mean (f32 [num_tokens, latent]; the
   * product and the sum each rounded to f32) in place of z.  NULL for FastWAM's
   * ActionAE, which decodes z as it is. */
  const float *latent_std, *latent_mean;
} fam_decoder_weights;

FAM_API int fam_decoder_workspace_size(const fam_decoder_config* cfg, const fam_decoder_weights* w,
                                       int32_t batch, size_t* bytes);
/* z: f32 [B, num_tokens, latent]; suite_ids: int32 [B] or NULL; out: f32 [B, horizon, A]. */
FAM_API int fam_action_decode(const fam_decoder_config* cfg, const fam_decoder_weights* w,
                              int32_t batch, const float* z, const int32_t* suite_ids, float* out,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Video output head (WanVideoDiT.post_dit -> Head.forward + unpatchify,
 * wan_video_dit.py:290-306, 426-431, 634-638), the video half of a joint
 * denoising step.  fam_video_head_norm: out bf16 [B*S, D] =
 * LayerNorm(hidden) * (1 + scale) + shift with (shift, scale) = bf16(modulation
 * [2, D] + t) of the token's row of t_rows bf16 [B, 2, D] (row 0 for the first
 * first_frame_tokens tokens of a sample); then fam_gemm with head.head gives
 * [B*S, pt*ph*pw*C]; fam_video_unpatchify rearranges it to bf16 [B, C, F*pt, H*ph, W*pw]. */
FAM_API int fam_video_head_norm(const float* hidden, const void* t_rows, const void* modulation, int32_t batch,
                                int32_t tokens, int32_t first_frame_tokens, int32_t dim, float eps, void* out,
                                void* stream);
FAM_API int fam_video_unpatchify(const void* x, int32_t batch, int32_t f, int32_t h, int32_t w, int32_t pt,
                                 int32_t ph, int32_t pw, int32_t channels, void* out, void* stream);

/* ---------------------------------------------------------------------------
 * Wan2.2 VAE encode of one observation frame: the pieces around the GEMMs of
 * VideoVAE38_.encode with T = 1 (FastWAM/src/fastwam/models/wan22/
 * wan_video_vae.py:1285-1304 via Encoder3d_38.forward :678-733; called from
 * fastwam.py:296-306).  Activations are channels-last [positions, channels];
 * 3x3 convolutions are fam_vae_im2col + fam_gemm, 1x1 convolutions fam_gemm.
 * -------------------------------------------------------------------------- */
/* patchify(2) (wan_video_vae.py:199-212) of a bf16 [3, H, W] frame into
 * out bf16 rows of 16 channels c*4 + r*2 + q (12..15 zero), row stride out_ld;
 * pad = 1: the zero-bordered layout of fam_gemm's implicit convolution
 * (position (y, x) at row (y + 1) * (W/2 + 2) + x + 1). */
FAM_API int fam_vae_patchify(const void* image, int H, int W, void* out, int64_t out_ld, int pad,
                             void* stream);
/* 3x3 gather for a convolution of stride `stride` and top/left zero padding
 * `pad` (bottom/right padding follows from Ho, Wo): dst [Ho*Wo, 9*C] bf16,
 * K order (dy, dx, c).  C, row strides: multiples of 8. */
FAM_API int fam_vae_im2col(const void* src, int64_t src_ld, int H, int W, int C, int stride, int pad,
                           int Ho, int Wo, void* dst, int64_t dst_ld, void* stream);
/* RMS_norm over channels (wan_video_vae.py:55-70; + SiLU when silu_on) of the
 * fp32 stream x [P, C] into bf16 out (nullable; out_pad_w > 0: the
 * zero-bordered layout of a frame out_pad_w wide), and/or bf16(x) into raw. */
FAM_API int fam_vae_rms(const float* x, int64_t x_ld, int64_t P, int C, const void* gamma, int silu_on,
                        void* out, int64_t out_ld, int out_pad_w, void* raw, int64_t raw_ld, void* stream);
/* out += AvgDown3D(in) for a one-frame input (wan_video_vae.py:345-395). */
FAM_API int fam_vae_avg_down_add(const float* in, int64_t in_ld, int H, int W, int Cin, int Cout,
                                 int factor_t, int factor_s, float* out, int64_t out_ld, void* stream);
/* Row softmax of fp32 scores * scale into bf16 (AttentionBlock, :321-342). */
FAM_API int fam_vae_softmax(const float* s, int64_t s_ld, int rows, int cols, float scale, void* p,
                            int64_t p_ld, void* stream);
/* bf16 transpose dst[c][r] = src[r][c]. */
FAM_API int fam_vae_transpose(const void* src, int64_t src_ld, int rows, int cols, void* dst,
                              int64_t dst_ld, void* stream);
/* out f32 [M, N] (+= when accumulate) bias + sum over splits of the split-K
 * GEMM partials f32 [splits, M, N] (fam_gemm FAM_EPI_PARTIAL). */
FAM_API int fam_vae_splitk_reduce(const float* partials, int splits, int64_t M, int N, const void* bias,
                                  float* out, int64_t out_ld, int accumulate, void* stream);
/* out f32 [z, P] = (mu[:, :z] - mean) * inv_std (VideoVAE38_.encode, :1296-1303). */
FAM_API int fam_vae_latent(const float* mu, int64_t mu_ld, int64_t P, int z, const float* mean,
                           const float* inv_std, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FAM_H_ */
