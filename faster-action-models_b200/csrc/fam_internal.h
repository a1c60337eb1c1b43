// Internal declarations shared by the libfam translation units (not part of
// the public C ABI; the public surface is include/fam.h).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fam {

// ----------------------------------------------------------------- errors
// Records a message for fam_last_error() and returns the non-zero status.
int set_error(const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);

// Device status word of the current device (allocated on first use, one int).
int* device_status_word();

// ------------------------------------------------------------------- TMA
// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row stride
// `row_stride` elements; box = 64 columns x box_rows rows, 128-byte swizzle,
// out-of-bounds elements read as zero.
bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                       uint64_t row_stride, uint32_t box_rows);

// 3-D bf16 tensor map over [batch, rows, cols] (row / batch strides in elements);
// box = 64 columns x box_rows rows x 1 batch, 128-byte swizzle, rows past a
// batch's end read as zero.
bool make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t batch, uint64_t rows, uint64_t cols,
                       uint64_t row_stride, uint64_t batch_stride, uint32_t box_rows);

// 2-D uint8 tensor map over [rows, cols] bytes (row stride in bytes, a multiple of
// 16); box = box_cols x box_rows, no swizzle, out-of-bounds bytes read as zero.
bool make_tmap_u8_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride,
                     uint32_t box_cols, uint32_t box_rows);

// ------------------------------------------------------------------ GEMM
enum EpiKind : int { kEpiStore = 0, kEpiPartial = 1, kEpiResidual = 2 };
enum ActKind : int { kActNone = 0, kActGeluTanh = 1, kActSilu = 2 };

struct GemmEpilogue {
  int kind;                 // EpiKind
  int act;                  // ActKind (store only)
  int out_bf16;             // store: 1 = bf16 output, 0 = fp32
  int features_on_a;        // 1: A rows index output features (weights-as-A)
  void* out;
  long long out_sa;         // output element stride per A-row index
  long long out_sb;         // output element stride per B-row index
  long long split_stride;   // partial: element stride between split-K slices
  const __nv_bfloat16* bias;   // bias[feature] (nullable)
  // residual: out += (gate_w[f] + gate_t[off(token) + f]) * (acc + bias[f])
  // with off(token) = batch * gate_bstride + (token in first frame ? 0 : gate_gstride)
  const __nv_bfloat16* gate_w;
  const float* gate_t;
  int tokens_per_batch;
  int first_frame_tokens;   // 0: a single gate row per batch
  long long gate_bstride;
  long long gate_gstride;
  int vec;                  // set by gemm_plan: 16-feature vector path of the store / residual epilogue
  // > 0: A rows are the padded positions y * conv_wp + x of a 3x3 convolution
  // (implicit GEMM); output row y * (conv_wp - 2) + x, none for x >= conv_wp - 2
  int conv_wp;
};

struct GemmArgs {
  int M, N, K;
  int kb_per_split;
  int a_is_const;           // operand constant for the launch chain (prefetched early)
  int b_is_const;
  int* status;
  GemmEpilogue epi;
  // Split last round (persistent kernel with a scratch): whole tiles go round-
  // robin for sk_full rounds; each of the remaining tiles is split into
  // sk_pieces k-ranges on consecutive CTAs.  Pieces 1.. store their fp32 partial
  // in sk_part[their CTA] and count their epilogue warps on sk_flag[piece 0's
  // CTA]; piece 0 adds the partials in piece order before the epilogue and
  // clears the flag.
  int sk_full;              // whole-tile rounds before the split round
  int sk_pieces;            // k-pieces per remaining tile (0: no split round)
  float* sk_part;           // [CTAs][128][BN] fp32
  unsigned* sk_flag;        // [CTAs], zero between launches
  // Implicit 3x3 stride-1 convolution (taps = 9): K block kb reads channel
  // block kb % tap_kpt of A row m + (t / 3) * tap_wp + t % 3, t = kb / tap_kpt,
  // from a zero-bordered channels-last activation buffer; B is [N, 9 * tap_kpt * 64].
  int taps;                 // 1: plain GEMM
  int tap_wp;
  int tap_kpt;
  // Tile raster of the persistent kernels: M-blocks fastest inside bands of
  // band_m M-blocks, the bands one after another (0 or >= the M-blocks: one
  // band).  A band's A rows stay in L2 while the weight n-blocks stream past
  // them once per band instead of once per wave.
  int band_m;
};

struct GemmPlan {
  CUtensorMap ta;
  CUtensorMap tb;
  GemmArgs args;
  int bn;
  int splits;
  int persist;              // persistent tile loop over min(tiles, SMs) CTAs
  int pair;                 // > 0: CTA-pair kernel (256 x 256 tiles) over this many pairs
};

// tcgen05 flash attention for long self attention (head_dim 128, one key source,
// no explicit / key masks; the first-frame-causal rule is supported).
struct AttnTcArgs {
  CUtensorMap tq;             // Q  [B*S, H*128]
  CUtensorMap tk;             // K  [B*Skv, H*128]
  CUtensorMap tv;             // V^T [B*H*128, Skv_pad]
  __nv_bfloat16* out;         // [B*S, out_ts]
  const uint8_t* kmask;       // [B, kmask_bs] key mask (nonzero = attend) or null
  long long out_ts, kmask_bs;
  int B, S, Skv, H, ff;
  float scale_log2;
  int* status;
};
// Self attention (Skv == Sq, optional first-frame rule) or attention over a
// second key source (Skv keys, optional per-batch key mask, ff == 0; taken
// only when the launch has at least 4 waves of CTAs: short key sources make
// each CTA a short latency chain, which pays only with many CTAs in flight).
bool attention_tc_eligible(int head_dim, int B, int H, int Sq, int S1, int S2, bool mask2d, int ff, long long q_ts,
                           long long kv_ts, long long out_ts);
size_t attention_tc_vt_bytes(int B, int H, int Skv);
// Transposes V into `vt` (attention_tc_vt_bytes) and runs the attention.
cudaError_t launch_attention_tc(const __nv_bfloat16* q, long long q_ts, const __nv_bfloat16* k, const __nv_bfloat16* v,
                                long long kv_ts, __nv_bfloat16* out, long long out_ts, int B, int S, int Skv, int H,
                                int ff, const uint8_t* kmask, long long kmask_bs, float scale_log2,
                                __nv_bfloat16* vt, int* status, cudaStream_t st, bool pdl);

int gemm_pick_bn(int n);
// sk_part / sk_flag (optional, sk_bytes of fp32 scratch and one zeroed word per
// SM): a many-tile problem may then run 256-wide tiles and split the tiles of
// the last, partial round over the idle CTAs (sk_force: whenever possible,
// else when the tile-time model predicts a gain).
int gemm_plan(GemmPlan* p, const void* A, long long lda, const void* B, long long ldb, int M, int N,
              int K, int splits, int bn, const GemmEpilogue& epi, bool a_is_const, bool b_is_const,
              int* status, float* sk_part = nullptr, unsigned* sk_flag = nullptr, size_t sk_bytes = 0,
              bool sk_force = false, bool allow_pair = false);
// Implicit-GEMM 3x3 stride-1 convolution: A is a zero-bordered channels-last
// buffer [a_rows, cin] (row stride lda) whose rows are the padded positions of
// a frame of width wp - 2; M = H * wp output rows (epi.conv_wp = wp maps them
// back); B the packed weight [N, 9 * ceil(cin / 64) * 64].
int gemm_plan_conv3(GemmPlan* p, const void* A, long long lda, long long a_rows, int cin, int wp, int M,
                    const void* B, long long ldb, int N, int splits, GemmEpilogue epi, int* status);
// Streaming-multiprocessor count of the current device, and the split-round scratch it needs.
int gemm_num_sms();
size_t gemm_sk_scratch_bytes();
cudaError_t gemm_launch(const GemmPlan& p, cudaStream_t stream, bool pdl);
// Sets the dynamic shared-memory limits of every kernel instantiation (call
// once per device before any stream capture).
cudaError_t gemm_init_attributes();
cudaError_t attn_init_attributes();

}  // namespace fam
