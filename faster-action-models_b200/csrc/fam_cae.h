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

struct CaeCtxArgs {
  const float* ctx_f32;            // [rows, T] (one of the two)
  const __nv_bfloat16* ctx_bf16;
  int rows, T, D, HD, L;
  const float *text0_w, *text0_b, *text2_w, *text2_b;
  CaeLayer layers[kCaeMaxLayers];
  float* ctx_k;                    // [L, rows, HD]
  float* ctx_v;
  float eps;
};

struct CaeStepArgs {
  CaeWeightsDev w;
  const float* rope;               // [positions, hd/2, 2]
  const float* ctx_k;              // [L, B*C, HD]
  const float* ctx_v;
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

// ------------------------------------------------------------ action decoder
constexpr int kDecMaxStages = 4;

struct DecArgs {
  fam_decoder_config cfg;
  const float *in_w, *in_b, *out_w, *out_b, *suite_embed;
  fam_decoder_stage stages[kDecMaxStages];
  int num_stages;
  const float* z;                  // [B, num_tokens, latent]
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
