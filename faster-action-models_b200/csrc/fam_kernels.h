// Argument structs and launchers of the non-GEMM kernels (internal).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fam {

// Timesteps passed by value (graph-capturable without a host copy).
constexpr int kMaxSteps = 64;
struct StepTimes {
  float t[kMaxSteps];
};

enum NormMode : int { kNormNone = 0, kNormAdaLN = 1, kNormAffine = 2 };

// Which row of the time modulation a token uses:
//   tmod + b * bstride + (token is past the first frame ? gstride : 0), then
//   chunk c (0..5) at c * D.  mod_w (bf16 [6, D], the block's `modulation`
//   parameter) is added when non-null.
struct ModRows {
  const float* tmod;
  const __nv_bfloat16* mod_w;
  int tokens_per_batch;
  int first_frame_tokens;
  long long bstride;
  long long gstride;
};

struct ResidNormArgs {
  float* x;                      // [rows, D] fp32 residual stream (updated in place)
  const float* partials;         // [nsplit, rows, D] or null (no residual update)
  long long split_stride;
  int nsplit;
  const __nv_bfloat16* bias;     // [D] or null
  int gate_chunk;                // modulation chunk used as gate, -1 = gate 1
  int round_residual;            // round x to bf16 after the add (reference residual dtype)
  int norm_mode;                 // NormMode
  int shift_chunk;               // AdaLN: shift chunk (scale = shift_chunk + 1)
  const __nv_bfloat16* norm_w;   // affine LN weight / bias
  const __nv_bfloat16* norm_b;
  ModRows mod;                   // modulation rows of the gate
  ModRows nmod;                  // modulation rows of the AdaLN shift/scale
  __nv_bfloat16* h;              // [rows, h_stride] bf16 normalized output
  long long h_stride;
  int D;
  float eps;
};

struct QkvPostArgs {
  const float* partials;         // [nsplit, rows, 3*HD] (nsplit > 0)
  const __nv_bfloat16* qkv_bf16; // [rows, 3*HD] (nsplit == 0)
  long long split_stride;
  int nsplit;
  const __nv_bfloat16* bias;     // [3*HD]
  const __nv_bfloat16* norm_q;   // [HD]
  const __nv_bfloat16* norm_k;   // [HD]
  const float2* rope;            // [positions, head_dim/2] (cos, sin)
  int rows_per_batch;            // RoPE position = row % rows_per_batch
  __nv_bfloat16* q_out;          // [rows, out_stride]
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
  long long out_stride;
  int HD;
  int head_dim;
  float eps;
};

struct RmsRowsArgs {
  const float* partials;
  long long split_stride;
  int nsplit;
  const __nv_bfloat16* in;       // nsplit == 0
  long long in_stride;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* w;
  __nv_bfloat16* out;
  long long out_stride;
  int N;
  float eps;
  int w_period;        // > 0: row r uses the weight vector w + (r % w_period) * w_stride
  long long w_stride;
};

struct EncodeArgs {
  const __nv_bfloat16* latent;   // [rows, A]
  const __nv_bfloat16* enc_w;    // [D, A]
  const __nv_bfloat16* enc_b;    // [D]
  float* x;                      // [rows, D]
  __nv_bfloat16* h;              // [rows, D]
  ModRows mod;                   // block 0 modulation (chunks 0, 1)
  int A;
  int D;
  float eps;
};

struct HeadArgs {
  const float* x;                // [rows, D]
  const __nv_bfloat16* head_w;   // [A, D]
  const __nv_bfloat16* head_b;
  __nv_bfloat16* velocity;       // [rows, A] or null
  __nv_bfloat16* latent;         // [rows, A] (updated when apply_euler)
  float delta;
  int apply_euler;
  int rows;
  int A;
  int D;
};

// Flash attention over up to two K/V sources (cached + fresh), online softmax
// in fp32, bf16 tensor-core MMAs.  Q/K/V/out are token-major with the head
// slice at h * head_dim inside the row.
struct AttnArgs {
  const __nv_bfloat16* q;
  long long q_bs, q_ts;
  const __nv_bfloat16* k1;
  const __nv_bfloat16* v1;
  long long kv1_bs, kv1_ts;
  int S1;
  int kv1_const;                 // source 1 is not written by earlier kernels of the chain
  const __nv_bfloat16* k2;
  const __nv_bfloat16* v2;
  long long kv2_bs, kv2_ts;
  int S2;
  const uint8_t* mask2d;         // [Sq, S1+S2] shared by all batches (True = attend) or null
  long long mask_rs;
  const uint8_t* key_mask;       // [B, S1+S2] per-batch key validity or null
  long long key_mask_bs;
  int first_frame_tokens;        // > 0: queries < ff see only keys < ff
  int Sq;
  int H;
  float scale_log2;              // log2(e) / sqrt(head_dim)
  __nv_bfloat16* out;
  long long out_bs, out_ts;
  float* part;                   // split partials (nsplit > 1)
  int* counters;                 // [B*H*q_tiles] arrival counters, zero before and after
  int nsplit;
  int keys_per_split;
  int* status;
};

struct PatchArgs {
  const __nv_bfloat16* in;   // [B, Cin, F, H, W]
  __nv_bfloat16* out;        // [B * S, Cin * pt * ph * pw]
  long long B;
  int Cin, F, H, W, pt, ph, pw;
};
cudaError_t launch_patchify(const PatchArgs& a, cudaStream_t st);

cudaError_t launch_resid_norm(const ResidNormArgs& a, int rows, cudaStream_t st, bool pdl);
cudaError_t launch_qkv_post(const QkvPostArgs& a, int rows, cudaStream_t st, bool pdl);
cudaError_t launch_rms_rows(const RmsRowsArgs& a, int rows, cudaStream_t st, bool pdl);
cudaError_t launch_sinusoid(const StepTimes& t, int rows, int dim, __nv_bfloat16* out, cudaStream_t st,
                            bool pdl);
cudaError_t launch_encode_adaln(const EncodeArgs& a, int rows, cudaStream_t st, bool pdl);
cudaError_t launch_head_euler(const HeadArgs& a, cudaStream_t st, bool pdl);
// Bytes of split partials the attention launch needs (0 when nsplit == 1).
size_t attn_partial_bytes(int B, int H, int Sq, int head_dim, int nsplit);
// Query tiles per (batch, head) of an attention launch over Sq queries (the
// arrival counters hold one int per batch x head x tile).
int attn_query_tiles(int Sq);
// Key splits that fill about two waves of the GPU with >= 128 keys each.
int attn_auto_splits(int units, int skv, int* keys_per_split);
cudaError_t launch_attention(const AttnArgs& a, int B, int head_dim, cudaStream_t st, bool pdl);
// The short-query attention on tcgen05 (attention_short_tc.cu: head dim 64, at
// most 32 queries, no first-frame rule, batch x heads >= 128, TMA-compatible
// strides) when the launch qualifies, attention_kernel otherwise.
cudaError_t launch_attention_auto(const AttnArgs& a, int B, int head_dim, cudaStream_t st, bool pdl);
bool attention_short_tc_taken(const AttnArgs& a, int B, int head_dim);

}  // namespace fam
