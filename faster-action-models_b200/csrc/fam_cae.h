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

// Shared-memory plan of the staged step kernel (offsets in floats from the
// dynamic shared-memory base; computed on the host by cae_staged_plan).
constexpr int kCaeStagedTensors = 18;  // per-block tensors: 0..13 attention half, 14..17 FFN half
constexpr int kCaeStagedHalfSplit = 14;
struct CaeStagePlan {
  int off[kCaeStagedTensors];      // offset inside its half
  int rows[kCaeStagedTensors], cols[kCaeStagedTensors], stride[kCaeStagedTensors];
  int a_floats, f_floats, kv_floats;
  int kc;                          // context keys per K/V unit
  int units_per_head;
  int wpq;                         // warps per query row in cross attention
  int tb;                          // t_mod rows per time-MLP batch
  int hdp;                         // row stride of the q/k/v/attention rows
  int o_abuf, o_fbuf, o_kv, o_x, o_h, o_q, o_k, o_v, o_att, o_qc, o_f, o_part, o_tm, o_tscr, o_lat,
      o_rope, o_encw, o_encb, o_headw, o_headb;
  int total_floats;
};

struct CaeStepArgs {
  CaeWeightsDev w;
  CaeStagePlan plan;
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
// Staged step kernel (weights and context K/V streamed through shared memory).
// Returns false when the shapes or pointers do not fit it; the plan is then unset.
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
