// Arguments of the fused persistent action-chunk kernel (internal).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fam_kernels.h"

namespace fam {

constexpr int kFusedMaxLayers = 32;
constexpr int kFusedMaxD = 1024;     // hidden width bound of the fused path
constexpr int kFusedRows = 32;        // token rows of one sample (MMA N, zero padded)
constexpr int kFusedThreads = 384;    // warp 0 weight producer, warps 1..11 workers (clusters of 2 CTAs)
constexpr int kFusedWorkers = 352;
constexpr int kFusedRing = 8;         // 128 x 64 bf16 weight tiles in flight per CTA (128 KB)
constexpr int kFusedStaging = 92 * 1024;
constexpr int kFusedKeysPerSplit = 256;
constexpr int kFusedMaxSplits = 10;   // joint-attention key splits per head (partials merged in shared memory)
constexpr int kFusedMaxCtas = 256;  // barrier flag lines reserved

enum FusedGemm : int { kFQkv = 0, kFO = 1, kFCq = 2, kFCo = 3, kFFfn0 = 4, kFFfn2 = 5 };

struct FusedArgs {
  CUtensorMap tm[6];                 // stacked weights [L * N, K] per FusedGemm
  // stacked per-block vectors (bf16)
  const __nv_bfloat16 *qkv_b, *o_b, *cq_b, *co_b, *ffn0_b, *ffn2_b;
  const __nv_bfloat16 *norm_q, *norm_k, *cnorm_q, *norm3_w, *norm3_b, *modulation;
  const __nv_bfloat16 *enc_w, *enc_b, *head_w, *head_b;
  const float* tmod;                 // [N, 6D]
  const float2* rope;                // [positions, hd/2]
  const __nv_bfloat16* vk[kFusedMaxLayers];
  const __nv_bfloat16* vv[kFusedMaxLayers];
  long long v_ts;                    // cache token stride (elements)
  int Sv;
  const uint8_t* mask2d;             // [Sa, Sv + Sa] or null
  const __nv_bfloat16* ckv;          // [C, L, 2HD]: RMSNorm'd K then V per context token and block
  const uint8_t* ctx_mask;           // [C] or null
  int C;
  // workspace.  The residual stream is bf16, as the reference's: each split
  // item of a residual GEMM (o, cross-o, ffn.2) stores its fp32 partial tile
  // in its own slot, and the last split item of each 128-feature tile
  // (tile_ctr) sums them in split order (deterministic) and completes the
  // tile's residual add x = bf16(x + bf16(gate * bf16(sum + bias))).
  __nv_bfloat16* x;                  // [32, D]
  float* slots;                      // [splits][D / 128][32][128] split partials
  unsigned* tile_ctr;                // [3][kFusedMaxD / 128] split arrivals per residual GEMM tile
  __nv_bfloat16 *q, *ka, *va, *ao, *qc, *ci, *fh;
  double* ssq;                       // [N][L][3][32] q / k / cross-q sums of squares (fp64: exact, order-free)
  double* lnstat;                    // [N][L][3][32][2] per-token sum x, sum x^2 of the bf16 residual after the
                                     // o, cross-o and ffn.2 adds (fp64 sums of fp32 partials: order-free)
  float* apart;                      // [H][splits][32][hd + 2]
  unsigned* sync;                    // [0] barrier go word, [1] abort, [2..] merge counters [N][L][H]
  unsigned* flags;                   // per-CTA barrier arrival lines (32 words apart)
  int* status;
  __nv_bfloat16* latent;             // [R, A]
  __nv_bfloat16* trace;              // [N, R, A] or null
  StepTimes deltas;
  int N, L, R, Sa, D, HD, H, hd, F, A, splits;
  int kps;                           // joint-attention keys per split (<= kFusedKeysPerSplit, a multiple of 32)
  float eps, scale_log2;
};

size_t fused_smem_bytes();
cudaError_t launch_fused_chunk(const FusedArgs& a, int grid, cudaStream_t st);
cudaError_t fused_init_attributes();
// CTAs of the largest co-resident grid of 2-CTA clusters (0 if unknown).
int fused_max_ctas();

}  // namespace fam
