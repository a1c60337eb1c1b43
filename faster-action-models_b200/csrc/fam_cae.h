// Kernel arguments of the compact action expert and the action decoder
// (internal).  Layer tables travel by value in the kernel parameters.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fam.h"
#include "fam_kernels.h"

namespace fam {

constexpr int kCaeMaxS = 32;      // action tokens per sample
constexpr int kCaeMaxD = 64;      // hidden width
constexpr int kCaeMaxHD = 64;     // heads x head_dim
constexpr int kCaeMaxHd = 32;     // head_dim
constexpr int kCaeMaxF = 256;     // FFN width
constexpr int kCaeMaxLayers = 32;

using CaeLayer = fam_cae_layer;

struct CaeWeightsDev {
  const float *enc_w, *enc_b, *text0_w, *text0_b, *text2_w, *text2_b, *time0_w, *time0_b,
      *time2_w, *time2_b, *tproj_w, *tproj_b, *head_w, *head_b;
  CaeLayer layers[kCaeMaxLayers];
};

// Shared-memory plan of the staged step kernel (offsets in floats from the
// dynamic shared-memory base; computed on the host by cae_staged_plan).
constexpr int kCaeStagedTensors = 18;  // per-block tensors: 0..13 attention half, 14..17 FFN half
constexpr int kCaeStagedHalfSplit = 14;
struct CaeStagePlan {
  int off[kCaeStagedTensors];      // offset inside its half (floats)
  int rows[kCaeStagedTensors], cols[kCaeStagedTensors], stride[kCaeStagedTensors];
  int a_floats, f_floats, kv_floats;
  int kc;                          // context keys per K/V chunk (16 per warp of a head)
  int units;                       // key chunks per block
  int nc;                          // CTAs per sample (a thread-block cluster): chunks dealt round-robin
  int wh;                          // warps per head in cross attention
  int tb;                          // t_mod rows per time-MLP batch
  int hdp;                         // row stride of the q/k/v/attention rows
  int o_abuf, o_fbuf, o_kv, o_x, o_h, o_q, o_k, o_v, o_att, o_qc, o_f, o_part, o_xpart, o_tm, o_tscr, o_lat,
      o_rope, o_encw, o_encb, o_headw, o_headb, o_bar;
  int total_floats;
};

struct CaeCtxArgs {
  const float* ctx_f32;            // [rows, T] (one of the two)
  const __nv_bfloat16* ctx_bf16;
  int rows, T, D, HD, L;
  const float *text0_w, *text0_b, *text2_w, *text2_b;
  CaeLayer layers[kCaeMaxLayers];
  float* ctx_k;                    // [L, rows, HD], or [L, rows, HD + 4] when kv_packed
  float* ctx_v;                    // [L, rows, HD], or [L, rows, HD + 8] when kv_packed
  float eps;
  // split path (tk > 0): slice kernel + K/V kernel, optional weight packing
  int B, C, H, hd;
  int kv_packed;
  int tk;                          // input columns per slice of text_embedding.0
  float* part;                     // [kCaeCtxSlices, rows, D] partial sums
  float* wpack;                    // [L, a_floats + f_floats] packed block weights, or null
  CaeStagePlan plan;               // tensor table of the packed layout
  int* status;                     // zeroed by the slice launch; bounded-wait failures
};

constexpr int kCaeCtxSlices = 8;    // input-column slices of text_embedding.0
constexpr int kCaeCtxRows = 16;     // context tokens per CTA on the split path
// Split context path eligibility (sets a.tk); false keeps the single-kernel path.
bool cae_ctx_split_setup(CaeCtxArgs* a);

// Action-VAE decode of the final latents in the staged step kernel's epilogue
// (ActionDecoder.forward, action_ae.py:123-166, one upsampling stage): the
// CTAs of a sample's cluster split the hidden channels in whole GroupNorm
// groups and exchange activations through distributed shared memory.
struct CaeDecode {
  int enabled;
  int hidden, latent, tokens, stride, horizon, action_dim;
  const float *in_w, *in_b, *out_w, *out_b, *suite_embed;
  const int32_t* suite_ids;        // [B] or null
  const float *convt_w, *convt_b, *gn0_w, *gn0_b, *c1_w, *c1_b, *gn1_w, *gn1_b, *c2_w, *c2_b, *gn2_w, *gn2_b;
  const float *lat_std, *lat_mean; // [tokens, latent] or null: z * std + mean is decoded
  float* out;                      // [B, horizon, action_dim]
};
// Shared-memory floats the epilogue decode needs (it uses the region before
// the step kernel's row buffers, dead after the last block).
int cae_decode_floats(const CaeDecode& d, int nc);
constexpr int kDecChunk = 8192;   // floats per weight staging buffer of the epilogue decode
constexpr int kDecStages = 3;     // staging buffers: two chunks in flight while one is used


struct CaeStepArgs {
  CaeWeightsDev w;
  CaeDecode dec;
  CaeStagePlan plan;
  const float* wpack;              // packed block weights: staged kernel when non-null
  int* status;                     // bounded-wait failures (or null)
  const float* rope;               // [positions, hd/2, 2]
  const float* ctx_k;              // [L, B*C, HD], or [L, B*C, HD + 4] with wpack
  const float* ctx_v;              // [L, B*C, HD], or [L, B*C, HD + 8] with wpack
  const uint8_t* ctx_mask;         // [B, C] or null
  float* latent;                   // [B, S, A] in/out
  float* trace;                    // [N, B, S, A] or null
  StepTimes timesteps;
  StepTimes deltas;
  int num_steps;
  int B, S, A, D, HD, hd, F, C, L, freq_dim;
  float eps;
};

cudaError_t launch_cae_context(const CaeCtxArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_cae_steps(const CaeStepArgs& a, cudaStream_t st, bool pdl);
size_t cae_smem_bytes();
// Packed per-block weight table (offsets, padded strides, half sizes) for D, H*d, F.
void cae_tensor_table(int D, int HD, int F, CaeStagePlan* p);
// Staged step kernel (packed weights and context K/V streamed through shared
// memory by bulk copies).  Returns false when the shapes do not fit it.
bool cae_staged_plan(const CaeStepArgs& a, CaeStagePlan* plan);
cudaError_t launch_cae_steps_staged(const CaeStepArgs& a, cudaStream_t st, bool pdl);

// ------------------------------------------------------------ action decoder
constexpr int kDecMaxStages = 4;

struct DecArgs {
  fam_decoder_config cfg;
  const float *in_w, *in_b, *out_w, *out_b, *suite_embed;
  fam_decoder_stage stages[kDecMaxStages];
  int num_stages;
  const float* z;                  // [B, num_tokens, latent]
  const float *lat_std, *lat_mean; // [num_tokens, latent] or null: z * std + mean is decoded
  const int32_t* suite_ids;        // [B] or null
  float* out;                      // [B, horizon, action_dim]
  float* buf0;                     // [B, hidden, max_len] scratch
  float* buf1;
  float* buf2;
  int B;
};

cudaError_t launch_action_decoder(const DecArgs& a, cudaStream_t st);
size_t decoder_scratch_floats(const fam_decoder_config& c, const fam_decoder_stage* stages, int n,
                              int B);

}  // namespace fam
