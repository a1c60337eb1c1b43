// tcgen05 bf16 GEMM:  D[m][n] = sum_k A[m][k] * B[n][k]   (both operands K-major)
//
// One CTA computes one 128 x BN output tile over a contiguous range of the K
// dimension (split-K when gridDim.z > 1).  Warp roles (192 threads):
//   warp 0      TMA producer: streams 128x64 A tiles and BNx64 B tiles into a
//               STAGES-deep shared-memory ring (128-byte swizzle);
//   warp 1      allocates TMEM and (lane 0) issues tcgen05.mma, 4 x K=16 per
//               stage, accumulating in fp32 in TMEM; commits free stages;
//   warps 2..5  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lane
//               quarter w%4) and apply bias / GELU / gated residual / split-K
//               partial stores.
// The persistent variant (many-tile problems) loops over tiles with two TMEM
// accumulators, so that the epilogue of one tile overlaps the main loop of the
// next, and runs sixteen epilogue warps (warps 2..17, four per lane quarter,
// 16-column chunks dealt round-robin): the epilogue is a latency-bound chain
// of TMEM loads, conversions and scattered stores per warp, and with fewer
// warps the epilogue of a K=3072 tile is longer than its main loop.
//
// The same kernel serves both operand orientations used by the models:
//   * small-M action GEMMs (8..256 tokens) run "weights as A": A = W[out,in]
//     so the 128-row MMA dimension walks output features and the token count
//     is the MMA N (16..256).  These are HBM-bound weight streams.
//   * large-M backbone GEMMs (1760 x B tokens) run "activations as A".
// The epilogue addresses the output through element strides for the A-row and
// B-row index, so either orientation writes a row-major [tokens, features]
// result.
//
// Programmatic dependent launch: the operand that is constant for the whole
// launch chain (the weights) is prefetched for the first ring stages before
// griddepcontrol.wait; the operand produced by the previous kernel is loaded
// after it.  All global writes happen after the wait.
#include "fam_common.cuh"
#include "fam_internal.h"

namespace fam {

constexpr int kGemmThreads = 192;
constexpr int kBK = 64;          // K elements per stage (128 bytes of bf16: one swizzle atom)
constexpr int kBM = 128;         // MMA M
constexpr int kSkMaxPieces = 4;  // k-pieces per tile of a split last round
// Persistent kernel: producer warp, MMA warp and four epilogue warps per TMEM
// lane quarter (16-column chunks dealt round-robin over the four).
constexpr int kPersistEpiWarps = 16;
constexpr int kEpiPerQuarter = kPersistEpiWarps / 4;
constexpr int kPersistThreads = 64 + 32 * kPersistEpiWarps;

__host__ __device__ constexpr int gemm_stage_bytes(int bn) { return kBM * kBK * 2 + bn * kBK * 2; }
__host__ __device__ constexpr int gemm_stages(int bn) {
  // Small-N tiles keep the CTA under ~113 KB so that two launches of the chain
  // can be resident on one SM (programmatic launch overlap); large-N tiles are
  // compute bound and take a deeper ring.
  return bn <= 64 ? (110 * 1024) / gemm_stage_bytes(bn) : (200 * 1024) / gemm_stage_bytes(bn);
}
__host__ __device__ constexpr int gemm_smem_bytes(int bn) {
  return gemm_stages(bn) * gemm_stage_bytes(bn) + 1024 /*align slack*/ + 256 /*barriers*/;
}
__host__ __device__ constexpr uint32_t gemm_tmem_cols(int bn) {
  return bn <= 32 ? 32u : (bn <= 64 ? 64u : (bn <= 128 ? 128u : 256u));
}

// A operand coordinates (K element, row) of K block kb for output rows from m0
// (an implicit 3x3 convolution shifts the rows per tap).
__device__ __forceinline__ void gemm_a_coord(const GemmArgs& a, int kb, int m0, int& ax, int& ay) {
  if (a.taps > 1) {
    const int t = kb / a.tap_kpt;
    ax = (kb - t * a.tap_kpt) * kBK;
    ay = m0 + (t / 3) * a.tap_wp + (t - (t / 3) * 3);
  } else {
    ax = kb * kBK;
    ay = m0;
  }
}

// Output row of A row p (-1: a padding column of an implicit convolution).
__device__ __forceinline__ int gemm_out_row(const GemmEpilogue& e, int p) {
  if (e.conv_wp <= 0) return p;
  const int y = p / e.conv_wp, x = p - y * e.conv_wp;
  return x < e.conv_wp - 2 ? y * (e.conv_wp - 2) + x : -1;
}

// Apply the epilogue to 16 accumulator values of A-row `a_row`, B-rows
// b0..b0+15.
__device__ __forceinline__ void gemm_epilogue_apply(const GemmArgs& args, const GemmEpilogue& e,
                                                    int a_row, int b0, int split, float* v) {
  if (e.vec && e.kind == kEpiStore) {
    // features contiguous in the output, N % 16 == 0: vector bias loads and stores
    if (b0 >= args.N) return;
    float bz[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) bz[j] = 0.f;
    if (e.bias != nullptr) {
      const uint4* bp = reinterpret_cast<const uint4*>(e.bias + b0);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 u = bp[h];
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[k]));
          bz[8 * h + 2 * k] = f.x;
          bz[8 * h + 2 * k + 1] = f.y;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float x = v[j] + bz[j];
      if (e.act == kActGeluTanh) x = gelu_tanh(rbf(x));
      else if (e.act == kActSilu) x = silu(rbf(x));
      v[j] = x;
    }
    if (e.out_bf16) {
      uint32_t pk[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        pk[j] = *reinterpret_cast<uint32_t*>(&h);
      }
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(e.out) +
                                            static_cast<long long>(a_row) * e.out_sa + b0);
      dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    } else {
      float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(e.out) + static_cast<long long>(a_row) * e.out_sa + b0);
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
    return;
  }
  if (e.kind == kEpiPartial) {
    float* out = reinterpret_cast<float*>(e.out) + split * e.split_stride +
                 static_cast<long long>(a_row) * e.out_sa;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (b0 + j < args.N) out[static_cast<long long>(b0 + j) * e.out_sb] = v[j];
    return;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int b = b0 + j;
    const int feat = e.features_on_a ? a_row : b;
    float x = v[j];
    if (e.bias != nullptr && b < args.N) x += bf2f(e.bias[feat]);
    if (e.act == kActGeluTanh) x = gelu_tanh(rbf(x));
    else if (e.act == kActSilu) x = silu(rbf(x));
    v[j] = x;
  }
  if (e.kind == kEpiStore) {
    if (e.out_bf16) {
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(e.out);
      const bool vec = (e.out_sb == 1) && (b0 + 16 <= args.N) && ((e.out_sa & 7) == 0) &&
                       ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
      if (vec) {
        uint32_t pk[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
          pk[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        uint4* dst = reinterpret_cast<uint4*>(out + static_cast<long long>(a_row) * e.out_sa + b0);
        dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (b0 + j < args.N)
            out[static_cast<long long>(a_row) * e.out_sa + static_cast<long long>(b0 + j) * e.out_sb] =
                f2bf(v[j]);
      }
    } else {
      float* out = reinterpret_cast<float*>(e.out);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (b0 + j < args.N)
          out[static_cast<long long>(a_row) * e.out_sa + static_cast<long long>(b0 + j) * e.out_sb] = v[j];
    }
    return;
  }
  // kEpiResidual: out_f32 += gate * x
  float* out = reinterpret_cast<float*>(e.out);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int b = b0 + j;
    if (b >= args.N) continue;
    const int feat = e.features_on_a ? a_row : b;
    const int tok = e.features_on_a ? b : a_row;
    float g = 1.0f;
    if (e.gate_t != nullptr) {
      const int bi = tok / e.tokens_per_batch;
      const int within = tok - bi * e.tokens_per_batch;
      const int grp = (e.first_frame_tokens > 0 && within >= e.first_frame_tokens) ? 1 : 0;
      g = e.gate_t[bi * e.gate_bstride + grp * e.gate_gstride + feat];
      if (e.gate_w != nullptr) g += bf2f(e.gate_w[feat]);
    }
    float* dst = out + static_cast<long long>(a_row) * e.out_sa + static_cast<long long>(b) * e.out_sb;
    *dst = *dst + g * v[j];
  }
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  constexpr int STAGES = gemm_stages(BN);
  constexpr int A_BYTES = kBM * kBK * 2;
  constexpr int B_BYTES = BN * kBK * 2;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = gemm_tmem_cols(BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM;
  const int n0 = blockIdx.y * BN;
  const int split = blockIdx.z;
  const int kb_total = (args.K + kBK - 1) / kBK;
  const int kb_begin = split * args.kb_per_split;
  const int kb_end = min(kb_total, kb_begin + args.kb_per_split);
  const int nkb = kb_end - kb_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Every CTA of this launch is resident and owns its TMEM: let the next
  // kernel of the chain start its prologue.
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0 && nkb > 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      const uint64_t polA = args.a_is_const ? pol_w : pol_x;
      const uint64_t polB = args.b_is_const ? pol_w : pol_x;
      const int pre = min(nkb, STAGES);
      // Prologue: constant operand first (may run before the previous kernel ends).
      for (int i = 0; i < pre; ++i) {
        const int kc = (kb_begin + i) * kBK;
        int ax, ay;
        gemm_a_coord(args, kb_begin + i, m0, ax, ay);
        uint8_t* sa = smem + i * STAGE_BYTES;
        mbar_arrive_expect_tx(&full[i], STAGE_BYTES);
        if (args.a_is_const) tma_load_2d(sa, &tmA, &full[i], ax, ay, polA);
        if (args.b_is_const) tma_load_2d(sa + A_BYTES, &tmB, &full[i], kc, n0, polB);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        const int kc = (kb_begin + i) * kBK;
        int ax, ay;
        gemm_a_coord(args, kb_begin + i, m0, ax, ay);
        uint8_t* sa = smem + i * STAGE_BYTES;
        if (!args.a_is_const) tma_load_2d(sa, &tmA, &full[i], ax, ay, polA);
        if (!args.b_is_const) tma_load_2d(sa + A_BYTES, &tmB, &full[i], kc, n0, polB);
      }
      int issued = pre;
      for (int i = pre; i < nkb; ++i) {
        const int s = i % STAGES;
        const uint32_t use = static_cast<uint32_t>(i / STAGES);
        if (*abort_flag) break;
        if (!mbar_wait(&empty[s], (use - 1) & 1, args.status, kErrWaitEmpty)) {
          *abort_flag = 1;
          break;
        }
        const int kc = (kb_begin + i) * kBK;
        int ax, ay;
        gemm_a_coord(args, kb_begin + i, m0, ax, ay);
        uint8_t* sa = smem + s * STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
        tma_load_2d(sa, &tmA, &full[s], ax, ay, polA);
        tma_load_2d(sa + A_BYTES, &tmB, &full[s], kc, n0, polB);
        issued = i + 1;
      }
      // Drain: every issued copy has landed before the CTA can exit (on the
      // normal path these waits return at once).
      for (int j = max(0, issued - STAGES); j < issued; ++j) {
        mbar_wait(&full[j % STAGES], static_cast<uint32_t>(j / STAGES) & 1, args.status,
                  kErrWaitFull);
      }
    } else if (lane == 0) {
      pdl_wait();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kBM, BN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        if (*abort_flag) break;
        if (!mbar_wait(&full[s], static_cast<uint32_t>(i / STAGES) & 1, args.status,
                       kErrWaitFull)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint64_t da = umma_desc_sw128(smem + s * STAGE_BYTES);
        const uint64_t db = umma_desc_sw128(smem + s * STAGE_BYTES + A_BYTES);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          // +32 bytes along K inside the swizzle atom = +2 in the 16-byte-unit address field
          umma_bf16_ss(tmem_base, da + 2 * k, db + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int sp = warp & 3;  // TMEM lane quarter accessible to this warp
    const int a_row = m0 + sp * 32 + lane;
    pdl_wait();
    const bool ok = mbar_wait(accum, 0, args.status, kErrWaitAccum);
    tc_fence_after();
    if (!ok) *abort_flag = 1;
    const GemmEpilogue& e = args.epi;
    if (ok && !*abort_flag && nkb > 0) {
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        __syncwarp();
        tmem_ld16(tmem_base + (static_cast<uint32_t>(sp * 32) << 16) + c, v);
        const int orow = gemm_out_row(e, a_row);
        if (a_row < args.M && orow >= 0) gemm_epilogue_apply(args, e, orow, n0 + c, split, v);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ------------------------------------------------------ persistent variant
// Large problems (more output tiles than SMs, no split-K): one CTA per SM loops
// over tiles (tile = blockIdx.x + i * gridDim.x, M-blocks fastest, so the CTAs
// in flight share each weight n-block through L2).  Two TMEM accumulators: the
// MMA warp fills one while the epilogue warps drain the other, so a tile's
// epilogue overlaps the next tile's main loop; the operand ring runs on across
// tile boundaries.
// A parked k-piece partial is a [BN/4][128 rows][4] fp32 block: the float4 of
// columns c..c+3 of row r sits at ((c / 4) * 128 + r) * 4, so that the 32 rows
// of a warp touch 512 contiguous bytes per access.
__device__ __forceinline__ long long gemm_part_index(int r, int c) {
  return (static_cast<long long>(c >> 2) * kBM + r) * 4;
}

// Adds columns c..c+15 of row r of the tile's later k-pieces, in piece order
// (npart partials, pstride floats apart); every load is issued before the adds.
__device__ __forceinline__ void gemm_add_partial(float* v, const float* padd, int r, int c, int npart,
                                                 long long pstride) {
  if (npart <= 0) return;
  float4 t[kSkMaxPieces - 1][4];
#pragma unroll
  for (int q = 0; q < kSkMaxPieces - 1; ++q)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      t[q][j] = q < npart ? *reinterpret_cast<const float4*>(padd + q * pstride + gemm_part_index(r, c + 4 * j))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int q = 0; q < kSkMaxPieces - 1; ++q)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[4 * j] += t[q][j].x;
      v[4 * j + 1] += t[q][j].y;
      v[4 * j + 2] += t[q][j].z;
      v[4 * j + 3] += t[q][j].w;
    }
}

// Epilogue of one epilogue warp: tile rows of its TMEM lane quarter (a row per
// lane), 16-column chunks c0, c0 + cs, ... < BN.  npart parked partials of later
// k-pieces (padd, pstride floats apart) are added in piece order first.
template <int BN>
__device__ __forceinline__ void gemm_tile_epilogue(const GemmArgs& args, uint32_t tacc, int r, int a_row, int n0,
                                                   int c0, int cs, const float* padd, int npart) {
  const GemmEpilogue& e = args.epi;
  const int out_row = gemm_out_row(e, a_row);
  const bool row_ok = a_row < args.M && out_row >= 0;
  a_row = row_ok ? out_row : 0;  // from here on, the output row
  if (e.vec && e.kind == kEpiResidual) {
    // out[row][f] += g[f] * act(acc + bias[f]); the chunk's fp32 residual and
    // gate row are loaded before its TMEM load so that the latencies overlap
    float* orow = reinterpret_cast<float*>(e.out) + static_cast<long long>(row_ok ? a_row : 0) * e.out_sa;
    const float* grow = nullptr;
    if (e.gate_t != nullptr) {
      const int tok = row_ok ? a_row : 0;
      const int bi = tok / e.tokens_per_batch, within = tok - bi * e.tokens_per_batch;
      const int grp = (e.first_frame_tokens > 0 && within >= e.first_frame_tokens) ? 1 : 0;
      grow = e.gate_t + bi * e.gate_bstride + grp * e.gate_gstride;
    }
#pragma unroll 1
    for (int c = c0; c < BN; c += cs) {
      const int b0 = n0 + c;
      const bool ok = row_ok && b0 < args.N;
      float4 rr[4], gt[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        rr[j] = ok ? *reinterpret_cast<const float4*>(orow + b0 + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
        gt[j] = (ok && grow != nullptr) ? *reinterpret_cast<const float4*>(grow + b0 + 4 * j)
                                        : make_float4(1.f, 1.f, 1.f, 1.f);
      }
      float v[16];
      __syncwarp();
      tmem_ld16(tacc + c, v);
      gemm_add_partial(v, padd, r, c, npart, static_cast<long long>(kBM) * BN);
      if (!ok) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // four columns at a time: bias and gate weight as 8-byte bf16 loads
        float bz[4] = {0.f, 0.f, 0.f, 0.f}, gw[4] = {0.f, 0.f, 0.f, 0.f};
        if (e.bias != nullptr) {
          const uint2 u = *reinterpret_cast<const uint2*>(e.bias + b0 + 4 * j);
          const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
          const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
          bz[0] = f0.x; bz[1] = f0.y; bz[2] = f1.x; bz[3] = f1.y;
        }
        if (grow != nullptr && e.gate_w != nullptr) {
          const uint2 u = *reinterpret_cast<const uint2*>(e.gate_w + b0 + 4 * j);
          const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
          const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
          gw[0] = f0.x; gw[1] = f0.y; gw[2] = f1.x; gw[3] = f1.y;
        }
        float x[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float t = v[4 * j + k] + bz[k];
          if (e.act == kActGeluTanh) t = gelu_tanh(rbf(t));
          else if (e.act == kActSilu) t = silu(rbf(t));
          x[k] = t;
        }
        const float4 g = gt[j];
        const float4 q = rr[j];
        *reinterpret_cast<float4*>(orow + b0 + 4 * j) =
            make_float4(q.x + (g.x + gw[0]) * x[0], q.y + (g.y + gw[1]) * x[1], q.z + (g.z + gw[2]) * x[2],
                        q.w + (g.w + gw[3]) * x[3]);
      }
    }
    return;
  }
#pragma unroll 1
  for (int c = c0; c < BN; c += cs) {
    float v[16];
    __syncwarp();
    tmem_ld16(tacc + c, v);
    gemm_add_partial(v, padd, r, c, npart, static_cast<long long>(kBM) * BN);
    if (row_ok) gemm_epilogue_apply(args, e, a_row, n0 + c, 0, v);
  }
}

// (M-block, N-block) of persistent tile `tile` (GemmArgs::band_m).
__device__ __forceinline__ int2 tile_mn(int tile, int tiles_m, int tiles_n, int band) {
  if (band <= 0 || band >= tiles_m) return make_int2(tile % tiles_m, tile / tiles_m);
  const int per_band = band * tiles_n;
  const int b = tile / per_band, r = tile - b * per_band;
  const int bm = min(band, tiles_m - b * band);
  return make_int2(b * band + r % bm, r / bm);
}

// Segments of a persistent CTA: whole tiles blockIdx.x + i * gridDim.x; with a
// split last round, sk_full whole rounds and then piece (blockIdx.x % P) of
// remaining tile (blockIdx.x / P) (piece = -1 for a whole tile).
struct GemmSegs {
  int i, ntiles, nkb, full, P, stage;
  __device__ __forceinline__ void init(const GemmArgs& args, int ntiles_, int nkb_) {
    ntiles = ntiles_;
    nkb = nkb_;
    P = args.sk_pieces;
    full = P > 0 ? args.sk_full : (ntiles + gridDim.x - 1) / gridDim.x;
    i = 0;
    stage = 0;
  }
  __device__ __forceinline__ bool next(int& t, int& kb0, int& kb1, int& piece) {
    if (stage == 0) {
      const int tt = blockIdx.x + i * gridDim.x;
      if (i < full && tt < ntiles) {
        ++i;
        t = tt;
        kb0 = 0;
        kb1 = nkb;
        piece = -1;
        return true;
      }
      stage = 1;
    }
    if (stage == 1) {
      stage = 2;
      if (P > 0) {
        const int j = blockIdx.x / P, p = blockIdx.x - j * P;
        const int tt = full * gridDim.x + j;
        if (tt < ntiles) {
          t = tt;
          kb0 = p * nkb / P;
          kb1 = (p + 1) * nkb / P;
          piece = p;
          return true;
        }
      }
    }
    return false;
  }
};

template <int BN>
__global__ void __launch_bounds__(kPersistThreads, 1)
    gemm_bf16_tc_persist_kernel(const __grid_constant__ CUtensorMap tmA,
                                const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  constexpr int STAGES = gemm_stages(BN);
  constexpr int A_BYTES = kBM * kBK * 2;
  constexpr int B_BYTES = BN * kBK * 2;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t ACC_COLS = gemm_tmem_cols(BN);
  constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;   // [2] accumulator ready for the epilogue
  uint64_t* tempty = tfull + 2;       // [2] accumulator drained (one arrival per epilogue warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (args.M + kBM - 1) / kBM, tiles_n = (args.N + BN - 1) / BN;
  const int ntiles = tiles_m * tiles_n;
  const int nkb = (args.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kPersistEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0 && nkb > 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      const uint64_t polA = args.a_is_const ? pol_w : pol_x;
      const uint64_t polB = args.b_is_const ? pol_w : pol_x;
      // first segment: constant operand of the first stages before the wait on the previous launch
      GemmSegs sg;
      sg.init(args, ntiles, nkb);
      int tile = 0, kb0 = 0, kb1 = 0, piece = -1;
      bool have = sg.next(tile, kb0, kb1, piece);
      int2 tmn = tile_mn(tile, tiles_m, tiles_n, args.band_m);
      int m0 = tmn.x * kBM, n0 = tmn.y * BN;
      const int pre = have ? min(kb1 - kb0, STAGES) : 0;
      for (int i = 0; i < pre; ++i) {
        int ax, ay;
        gemm_a_coord(args, kb0 + i, m0, ax, ay);
        uint8_t* sa = smem + i * STAGE_BYTES;
        mbar_arrive_expect_tx(&full[i], STAGE_BYTES);
        if (args.a_is_const) tma_load_2d(sa, &tmA, &full[i], ax, ay, polA);
        if (args.b_is_const) tma_load_2d(sa + A_BYTES, &tmB, &full[i], (kb0 + i) * kBK, n0, polB);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        int ax, ay;
        gemm_a_coord(args, kb0 + i, m0, ax, ay);
        uint8_t* sa = smem + i * STAGE_BYTES;
        if (!args.a_is_const) tma_load_2d(sa, &tmA, &full[i], ax, ay, polA);
        if (!args.b_is_const) tma_load_2d(sa + A_BYTES, &tmB, &full[i], (kb0 + i) * kBK, n0, polB);
      }
      int kb = kb0 + pre, issued = pre;
      if (have && kb == kb1) {
        have = sg.next(tile, kb0, kb1, piece);
        kb = kb0;
        tmn = tile_mn(tile, tiles_m, tiles_n, args.band_m);
        m0 = tmn.x * kBM;
        n0 = tmn.y * BN;
      }
      for (int it = pre; have; ++it) {
        const int s = it % STAGES;
        if (*abort_flag) break;
        if (!mbar_wait(&empty[s], static_cast<uint32_t>(it / STAGES - 1) & 1, args.status, kErrWaitEmpty)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* sa = smem + s * STAGE_BYTES;
        int ax, ay;
        gemm_a_coord(args, kb, m0, ax, ay);
        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
        tma_load_2d(sa, &tmA, &full[s], ax, ay, polA);
        tma_load_2d(sa + A_BYTES, &tmB, &full[s], kb * kBK, n0, polB);
        issued = it + 1;
        if (++kb == kb1) {
          have = sg.next(tile, kb0, kb1, piece);
          kb = kb0;
          tmn = tile_mn(tile, tiles_m, tiles_n, args.band_m);
          m0 = tmn.x * kBM;
          n0 = tmn.y * BN;
        }
      }
      // every issued copy has landed before the CTA can exit
      for (int j = max(0, issued - STAGES); j < issued; ++j)
        mbar_wait(&full[j % STAGES], static_cast<uint32_t>(j / STAGES) & 1, args.status, kErrWaitFull);
    } else if (lane == 0) {
      pdl_wait();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kBM, BN);
      int it = 0, lt = 0;
      GemmSegs sg;
      sg.init(args, ntiles, nkb);
      int tile, kb0, kb1, piece;
      for (; nkb > 0 && sg.next(tile, kb0, kb1, piece); ++lt) {
        const int buf = lt & 1;
        if (*abort_flag) break;
        if (lt >= 2 && !mbar_wait(&tempty[buf], static_cast<uint32_t>((lt >> 1) - 1) & 1, args.status,
                                  kErrWaitAccum)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t dacc = tmem_base + buf * ACC_COLS;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          if (*abort_flag || !mbar_wait(&full[s], static_cast<uint32_t>(it / STAGES) & 1, args.status,
                                        kErrWaitFull)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(smem + s * STAGE_BYTES);
          const uint64_t db = umma_desc_sw128(smem + s * STAGE_BYTES + A_BYTES);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16_ss(dacc, da + 2 * k, db + 2 * k, idesc, (kb > kb0 || k != 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
    }
  } else {
    static_assert(BN % 16 == 0, "epilogue chunks are whole 16-column loads");
    const int sp = warp & 3;                       // TMEM lane quarter of this warp
    const int wq = (warp - 2) >> 2;                // its rank among the quarter's warps
    const int c0 = 16 * wq, cs = 16 * kEpiPerQuarter;  // its 16-column chunks
    pdl_wait();
    int lt = 0;
    GemmSegs sg;
    sg.init(args, ntiles, nkb);
    int tile, kb0, kb1, piece;
    for (; nkb > 0 && sg.next(tile, kb0, kb1, piece); ++lt) {
      const int buf = lt & 1;
      if (args.epi.vec && args.epi.kind == kEpiResidual && piece <= 0 && wq == 0) {
        // pull this row's residual segment into L2 while the tile's main loop runs
        const int2 pmn = tile_mn(tile, tiles_m, tiles_n, args.band_m);
        const int prow = pmn.x * kBM + sp * 32 + lane, col = pmn.y * BN;
        const int row = prow < args.M ? gemm_out_row(args.epi, prow) : -1;
        const int ncols = min(BN, args.N - col);
        if (row >= 0 && ncols > 0)
          bulk_prefetch_l2(reinterpret_cast<const float*>(args.epi.out) + static_cast<long long>(row) * args.epi.out_sa + col,
                           static_cast<uint32_t>(ncols) * 4u);
      }
      const bool ok = mbar_wait(&tfull[buf], static_cast<uint32_t>(lt >> 1) & 1, args.status, kErrWaitAccum);
      tc_fence_after();
      if (!ok) *abort_flag = 1;
      if (*abort_flag) break;
      const int2 emn = tile_mn(tile, tiles_m, tiles_n, args.band_m);
      const int m0 = emn.x * kBM, n0 = emn.y * BN;
      const uint32_t tacc = tmem_base + buf * ACC_COLS + (static_cast<uint32_t>(sp * 32) << 16);
      const int r = sp * 32 + lane;  // row inside the tile
      if (piece > 0) {
        // a later k-piece of a tile that piece 0's CTA finishes: park the fp32 partial
        float* pt = args.sk_part + static_cast<long long>(blockIdx.x) * kBM * BN;
#pragma unroll 1
        for (int c = c0; c < BN; c += cs) {
          float v[16];
          __syncwarp();
          tmem_ld16(tacc + c, v);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<float4*>(pt + gemm_part_index(r, c + 4 * j)) =
                make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(args.sk_flag + blockIdx.x - piece, 1u);
      } else if (piece == 0) {
        // piece 0: wait for the other pieces' partials (every epilogue warp of each)
        unsigned* fl = args.sk_flag + blockIdx.x;
        const unsigned want = static_cast<unsigned>(kPersistEpiWarps * (args.sk_pieces - 1));
        int got = 1;
        if (lane == 0) {
          const unsigned long long t0 = globaltimer_ns();
          while (atomicAdd(fl, 0u) < want) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
              record_error(args.status, kErrWaitAccum);
              got = 0;
              break;
            }
          }
        }
        got = __shfl_sync(0xffffffffu, got, 0);
        __threadfence();
        const float* pt = args.sk_part + static_cast<long long>(blockIdx.x + 1) * kBM * BN;
        gemm_tile_epilogue<BN>(args, tacc, r, m0 + r, n0, c0, cs, pt, got ? args.sk_pieces - 1 : 0);
        // every epilogue warp is done with the partials: clear the flag
        asm volatile("bar.sync 1, %0;" ::"n"(32 * kPersistEpiWarps) : "memory");
        if (warp == 2 && lane == 0) atomicExch(fl, 0u);
      } else {
        gemm_tile_epilogue<BN>(args, tacc, r, m0 + r, n0, c0, cs, nullptr, 0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------- CTA-pair variant
// Many-tile problems with 256-wide N tiles: a cluster of two CTAs computes
// 256 x 256 output tiles with tcgen05.mma.cta_group::2.  Each CTA loads its
// own 128 rows of A and its half (128 rows) of the B tile, so a CTA streams
// 32 KB per 64-deep k-block for 128 x 256 outputs instead of 48 KB.  The even
// CTA (rank 0) issues the MMAs; its `full` barriers count both CTAs' TMA bytes,
// its commits arrive on both CTAs' `empty` and `tfull` barriers, and both CTAs'
// epilogue warps arrive on its `tempty`.  Each CTA drains its 128 TMEM lanes
// with the persistent kernel's epilogue.  Every wait is bounded.
constexpr int kPairBN = 256;
__host__ __device__ constexpr int gemm_pair_stage_bytes() { return kBM * kBK * 2 + (kPairBN / 2) * kBK * 2; }
constexpr int kPairStages = 6;
__host__ __device__ constexpr int gemm_pair_smem_bytes() {
  return kPairStages * gemm_pair_stage_bytes() + 1024 + 256;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPersistThreads, 1)
    gemm_bf16_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const GemmArgs args) {
  constexpr int BN = kPairBN;
  constexpr int STAGES = kPairStages;
  constexpr int A_BYTES = kBM * kBK * 2;
  constexpr int STAGE_BYTES = gemm_pair_stage_bytes();
  constexpr uint32_t ACC_COLS = 256;
  constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles_m = (args.M + 2 * kBM - 1) / (2 * kBM), tiles_n = (args.N + BN - 1) / BN;
  const int ntiles = tiles_m * tiles_n;
  const int nkb = (args.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kPersistEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_barrier();  // both CTAs' barriers initialised before any remote arrival or TMA
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0 && nkb > 0) {
      const uint64_t polA = args.a_is_const ? policy_evict_first() : policy_evict_last();
      const uint64_t polB = args.b_is_const ? policy_evict_first() : policy_evict_last();
      // first tile: the operand that is constant for the launch chain (the
      // weights) for the first stages before the wait on the previous launch
      int pre = 0;
      if (pair < ntiles) {
        const int2 fmn = tile_mn(pair, tiles_m, tiles_n, args.band_m);
        const int m0 = fmn.x * 2 * kBM + static_cast<int>(rank) * kBM;
        const int n0 = fmn.y * BN + static_cast<int>(rank) * (BN / 2);
        pre = min(nkb, STAGES);
        for (int i = 0; i < pre; ++i) {
          uint8_t* sa = smem + i * STAGE_BYTES;
          const uint32_t bar0 = cluster_map(&full[i], 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[i], 2 * STAGE_BYTES);
          if (args.a_is_const) tma_load_2d_pair(sa, &tmA, bar0, i * kBK, m0, polA);
          if (args.b_is_const) tma_load_2d_pair(sa + A_BYTES, &tmB, bar0, i * kBK, n0, polB);
        }
        pdl_wait();
        for (int i = 0; i < pre; ++i) {
          uint8_t* sa = smem + i * STAGE_BYTES;
          const uint32_t bar0 = cluster_map(&full[i], 0);
          if (!args.a_is_const) tma_load_2d_pair(sa, &tmA, bar0, i * kBK, m0, polA);
          if (!args.b_is_const) tma_load_2d_pair(sa + A_BYTES, &tmB, bar0, i * kBK, n0, polB);
        }
      } else {
        pdl_wait();
      }
      int it = 0;
      for (int tile = pair; tile < ntiles && !*abort_flag; tile += npairs) {
        const int2 tmn = tile_mn(tile, tiles_m, tiles_n, args.band_m);
        const int m0 = tmn.x * 2 * kBM + static_cast<int>(rank) * kBM;
        const int n0 = tmn.y * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          if (it < pre) continue;  // issued above
          const int s = it % STAGES;
          if (it >= STAGES &&
              !mbar_wait(&empty[s], static_cast<uint32_t>(it / STAGES - 1) & 1, args.status, kErrWaitEmpty)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* sa = smem + s * STAGE_BYTES;
          const uint32_t bar0 = cluster_map(&full[s], 0);  // the even CTA's barrier
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);
          tma_load_2d_pair(sa, &tmA, bar0, kb * kBK, m0, polA);
          tma_load_2d_pair(sa + A_BYTES, &tmB, bar0, kb * kBK, n0, polB);
        }
      }
      // the even CTA's full barriers count every copy of both CTAs: wait for
      // the last ones before the pair can exit
      if (rank == 0)
        for (int j = max(0, it - STAGES); j < it; ++j)
          mbar_wait(&full[j % STAGES], static_cast<uint32_t>(j / STAGES) & 1, args.status, kErrWaitFull);
    } else if (lane == 0) {
      pdl_wait();
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = umma_idesc_bf16(2 * kBM, BN);
      int it = 0, lt = 0;
      for (int tile = pair; tile < ntiles && nkb > 0; tile += npairs, ++lt) {
        const int buf = lt & 1;
        if (*abort_flag) break;
        if (lt >= 2 && !mbar_wait_cl_bounded(&tempty[buf], static_cast<uint32_t>((lt >> 1) - 1) & 1, args.status,
                                             kErrWaitAccum)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t dacc = tmem_base + buf * ACC_COLS;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % STAGES;
          if (*abort_flag || !mbar_wait(&full[s], static_cast<uint32_t>(it / STAGES) & 1, args.status, kErrWaitFull)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(smem + s * STAGE_BYTES);
          const uint64_t db = umma_desc_sw128(smem + s * STAGE_BYTES + A_BYTES);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16_ss_pair(dacc, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit_pair_both(&empty[s]);
        }
        if (!ok) break;
        umma_commit_pair_both(&tfull[buf]);
      }
    }
  } else {
    const int sp = warp & 3;
    const int wq = (warp - 2) >> 2;
    const int c0 = 16 * wq, cs = 16 * kEpiPerQuarter;
    const uint32_t tempty0 = cluster_map(&tempty[0], 0), tempty1 = cluster_map(&tempty[1], 0);
    pdl_wait();
    int lt = 0;
    for (int tile = pair; tile < ntiles && nkb > 0; tile += npairs, ++lt) {
      const int buf = lt & 1;
      const bool ok = mbar_wait_cl_bounded(&tfull[buf], static_cast<uint32_t>(lt >> 1) & 1, args.status,
                                           kErrWaitAccum);
      tc_fence_after();
      if (!ok) *abort_flag = 1;
      if (*abort_flag) break;
      const int2 emn = tile_mn(tile, tiles_m, tiles_n, args.band_m);
      const int m0 = emn.x * 2 * kBM + static_cast<int>(rank) * kBM;
      const int n0 = emn.y * BN;
      const uint32_t tacc = tmem_base + buf * ACC_COLS + (static_cast<uint32_t>(sp * 32) << 16);
      const int r = sp * 32 + lane;
      gemm_tile_epilogue<BN>(args, tacc, r, m0 + r, n0, c0, cs, nullptr, 0);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(buf ? tempty1 : tempty0);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_barrier();  // the pair is done with each other's barriers and TMEM
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
template <int BN>
static cudaError_t launch_gemm_bn(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                                  int splits, cudaStream_t stream, bool pdl) {
  static bool attr_set = false;
  constexpr int smem = gemm_smem_bytes(BN);
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tc_kernel<BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.M + kBM - 1) / kBM, (a.N + BN - 1) / BN, splits);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_bf16_tc_kernel<BN>, ta, tb, a);
}

template <int BN>
static cudaError_t launch_gemm_persist_bn(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                                          int grid, cudaStream_t stream, bool pdl) {
  static bool attr_set = false;
  constexpr int smem = gemm_smem_bytes(BN);
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tc_persist_kernel<BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPersistThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_bf16_tc_persist_kernel<BN>, ta, tb, a);
}

int gemm_num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
  }
  return n;
}

size_t gemm_sk_scratch_bytes() { return static_cast<size_t>(gemm_num_sms()) * kBM * 256 * sizeof(float); }

cudaError_t gemm_init_attributes() {
  cudaError_t e;
#define FAM_SET(BN)                                                                          \
  e = cudaFuncSetAttribute(gemm_bf16_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           gemm_smem_bytes(BN));                                             \
  if (e != cudaSuccess) return e;
  FAM_SET(16) FAM_SET(32) FAM_SET(64) FAM_SET(128) FAM_SET(160) FAM_SET(192) FAM_SET(256)
#undef FAM_SET
#define FAM_SETP(BN)                                                                              \
  e = cudaFuncSetAttribute(gemm_bf16_tc_persist_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           gemm_smem_bytes(BN));                                                  \
  if (e != cudaSuccess) return e;
  FAM_SETP(64) FAM_SETP(128) FAM_SETP(160) FAM_SETP(192) FAM_SETP(256)
#undef FAM_SETP
  return cudaSuccess;
}

int gemm_pick_bn(int n) {
  if (n <= 16) return 16;
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  if (n <= 128) return 128;
  return 256;
}

int gemm_plan_conv3(GemmPlan* p, const void* A, long long lda, long long a_rows, int cin, int wp, int M,
                    const void* B, long long ldb, int N, int splits, GemmEpilogue epi, int* status) {
  if (cin <= 0 || (cin % 8) || wp < 3 || a_rows <= 0 || M <= 0 || lda < cin)
    return set_error("gemm_plan_conv3: bad convolution geometry");
  const int kpt = (cin + kBK - 1) / kBK;
  epi.conv_wp = wp;
  // plan as a plain [M, 9 * kpt * 64] x [N, same]^T problem, then point the A
  // map at the activation buffer and switch the producer to tap addressing
  int rc = gemm_plan(p, A, 9LL * kpt * kBK, B, ldb, M, N, 9 * kpt * kBK, splits, 0, epi, false, true, status);
  if (rc) return rc;
  if (!make_tmap_bf16_2d(&p->ta, A, static_cast<uint64_t>(a_rows), static_cast<uint64_t>(cin),
                         static_cast<uint64_t>(lda), kBM))
    return set_error("gemm_plan_conv3: cuTensorMapEncodeTiled failed for A");
  p->args.taps = 9;
  p->args.tap_wp = wp;
  p->args.tap_kpt = kpt;
  p->pair = 0;
  return 0;
}

cudaError_t gemm_launch(const GemmPlan& p, cudaStream_t stream, bool pdl) {
  if (p.pair > 0) {
    static bool attr_set = false;
    if (!attr_set) {
      cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tc_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           gemm_pair_smem_bytes());
      if (e != cudaSuccess) return e;
      attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * p.pair);
    cfg.blockDim = dim3(kPersistThreads);
    cfg.dynamicSmemBytes = gemm_pair_smem_bytes();
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_bf16_tc_pair_kernel, p.ta, p.tb, p.args);
  }
  if (p.persist > 0) {
    switch (p.bn) {
      case 64: return launch_gemm_persist_bn<64>(p.ta, p.tb, p.args, p.persist, stream, pdl);
      case 128: return launch_gemm_persist_bn<128>(p.ta, p.tb, p.args, p.persist, stream, pdl);
      case 160: return launch_gemm_persist_bn<160>(p.ta, p.tb, p.args, p.persist, stream, pdl);
      case 192: return launch_gemm_persist_bn<192>(p.ta, p.tb, p.args, p.persist, stream, pdl);
      case 256: return launch_gemm_persist_bn<256>(p.ta, p.tb, p.args, p.persist, stream, pdl);
      default: break;
    }
  }
  switch (p.bn) {
    case 16: return launch_gemm_bn<16>(p.ta, p.tb, p.args, p.splits, stream, pdl);
    case 32: return launch_gemm_bn<32>(p.ta, p.tb, p.args, p.splits, stream, pdl);
    case 64: return launch_gemm_bn<64>(p.ta, p.tb, p.args, p.splits, stream, pdl);
    case 128: return launch_gemm_bn<128>(p.ta, p.tb, p.args, p.splits, stream, pdl);
    case 160: return launch_gemm_bn<160>(p.ta, p.tb, p.args, p.splits, stream, pdl);
    case 192: return launch_gemm_bn<192>(p.ta, p.tb, p.args, p.splits, stream, pdl);
    case 256: return launch_gemm_bn<256>(p.ta, p.tb, p.args, p.splits, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

// Build a launch plan.  A is [M, K] with row stride lda (elements), B is [N, K]
// with row stride ldb.  `splits` > 1 requires the partial epilogue.
int gemm_plan(GemmPlan* p, const void* A, long long lda, const void* B, long long ldb, int M,
              int N, int K, int splits, int bn, const GemmEpilogue& epi, bool a_is_const,
              bool b_is_const, int* status, float* sk_part, unsigned* sk_flag, size_t sk_bytes,
              bool sk_force, bool allow_pair) {
  if (M <= 0 || N <= 0 || K <= 0) return set_error("gemm: empty problem");
  if ((K % 8) != 0 || (lda % 8) != 0 || (ldb % 8) != 0)
    return set_error("gemm: K and row strides must be multiples of 8 elements (16 bytes)");
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15))
    return set_error("gemm: operand base addresses must be 16-byte aligned");
  // Tile width for many-tile problems: the shortest estimated makespan.  The
  // time of a 128-row tile measured on B200 grows as (BN + 340) per k-block
  // (operand rows streamed per k-block plus a fixed per-k-block cost, fitted
  // over BN = 128..256); whole rounds over the SMs cost that each.  With a
  // scratch, 256-wide tiles may instead split the last, partial round into
  // P <= 4 k-pieces, which costs 1/P of a round plus a fixed exchange
  // (measured ~25 us, about 53 k-blocks of a 256-wide tile).
  bool sk = false;
  const int sms = gemm_num_sms(), mt = (M + kBM - 1) / kBM;
  const long long nkb_all = (K + kBK - 1) / kBK;
  int sk_pieces = 0, sk_full = 0;
  if (bn == 0) {
    bn = gemm_pick_bn(N);
    if (splits <= 1 && mt * ((N + 255) / 256) > sms) {
      const int cand[4] = {256, 192, 160, 128};
      double best = -1.0;
      for (int i = 0; i < 4; ++i) {
        const long long tiles = static_cast<long long>(mt) * ((N + cand[i] - 1) / cand[i]);
        const double t = static_cast<double>((tiles + sms - 1) / sms) * (cand[i] + 340) * nkb_all;
        if (best < 0 || t < best) {
          best = t;
          bn = cand[i];
        }
      }
      if (sk_part != nullptr && sk_flag != nullptr && sk_bytes >= gemm_sk_scratch_bytes()) {
        const long long tiles = static_cast<long long>(mt) * ((N + 255) / 256);
        const int full = static_cast<int>(tiles / sms), left = static_cast<int>(tiles - static_cast<long long>(full) * sms);
        int P = left > 0 ? sms / left : 0;
        if (P > kSkMaxPieces) P = kSkMaxPieces;
        if (P > nkb_all) P = static_cast<int>(nkb_all);
        if (P >= 2) {
          const double t = (full + 1.0 / P) * (256 + 340) * nkb_all + 53.0 * (256 + 340);
          if (sk_force || t < best) {
            sk = true;
            bn = 256;
            sk_pieces = P;
            sk_full = full;
          }
        }
      }
    } else if (splits <= 1 && !epi.features_on_a && mt <= 4) {
      // few activation rows against a wide weight (context projections): halve
      // the tile width while the tiles still fit one wave, so that the weight
      // stream is spread over more SMs
      while (bn > 32 && (bn & (bn - 1)) == 0 && mt * ((N + bn / 2 - 1) / (bn / 2)) <= sms) bn /= 2;
    } else if (splits <= 1 && epi.features_on_a) {
      // weights as A with a few hundred token columns and no split-K (the
      // action expert's ffn.0 at batch 8: 32 feature tiles x one 256-token
      // tile): narrower token tiles while they fit one wave spread the weight
      // stream (re-read from L2 per token tile) over more SMs
      while (bn > 64 && (bn & (bn - 1)) == 0 && mt * ((N + bn / 2 - 1) / (bn / 2)) <= sms) bn /= 2;
    }
  }
  const int kb_total = (K + kBK - 1) / kBK;
  if (splits < 1) splits = 1;
  if (splits > kb_total) splits = kb_total;
  const int kps = (kb_total + splits - 1) / splits;
  splits = (kb_total + kps - 1) / kps;  // no empty split
  if (splits > 1 && epi.kind != kEpiPartial)
    return set_error("gemm: split-K requires the partial epilogue");
  if (epi.kind == kEpiResidual && epi.gate_t != nullptr && epi.tokens_per_batch <= 0)
    return set_error("gemm: residual gate needs tokens_per_batch > 0");
  if (!make_tmap_bf16_2d(&p->ta, A, static_cast<uint64_t>(M), static_cast<uint64_t>(K),
                         static_cast<uint64_t>(lda), kBM))
    return set_error("gemm: cuTensorMapEncodeTiled failed for A");
  if (!make_tmap_bf16_2d(&p->tb, B, static_cast<uint64_t>(N), static_cast<uint64_t>(K),
                         static_cast<uint64_t>(ldb), static_cast<uint32_t>(bn)))
    return set_error("gemm: cuTensorMapEncodeTiled failed for B");
  p->bn = bn;
  p->splits = splits;
  // persistent tile loop when the tiles outnumber the SMs (no split-K)
  const int ntiles = ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
  p->persist = (splits == 1 && bn >= 64 && ntiles > sms) ? sms : 0;
  p->args.sk_full = 0;
  p->args.sk_pieces = 0;
  p->args.sk_part = nullptr;
  p->args.sk_flag = nullptr;
  p->args.taps = 1;
  p->args.tap_wp = 0;
  p->args.tap_kpt = 0;
  // CTA pairs (256 x 256 tiles, half of B per CTA) for many-tile problems that
  // would run 256-wide tiles anyway
  p->pair = 0;
  if (allow_pair && splits == 1 && bn == 256 && !sk && !epi.features_on_a && M > kBM) {
    const int pt = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + 255) / 256);
    // each CTA of a pair loads a 128-row half of the B tile
    if (!make_tmap_bf16_2d(&p->tb, B, static_cast<uint64_t>(N), static_cast<uint64_t>(K),
                           static_cast<uint64_t>(ldb), static_cast<uint32_t>(kPairBN / 2)))
      return set_error("gemm: cuTensorMapEncodeTiled failed for the pair B half tile");
    p->pair = std::min(pt, gemm_num_sms() / 2);
  }
  // raster bands of ~24 MB of A rows (see GemmArgs::band_m)
  {
    const long long rows = p->pair > 0 ? 2 * kBM : kBM;
    const long long block_bytes = rows * static_cast<long long>(K) * 2;
    p->args.band_m = static_cast<int>(std::max(1LL, (24LL << 20) / block_bytes));
  }
  if (sk && p->persist > 0) {
    p->args.sk_full = sk_full;
    p->args.sk_pieces = sk_pieces;
    p->args.sk_part = sk_part;
    p->args.sk_flag = sk_flag;
  }
  // 16-feature vector epilogue (residual): features contiguous in the output,
  // 16-byte aligned rows, bias / gates / gate rows aligned for vector loads
  {
    GemmEpilogue& ve = p->args.epi;
    ve = epi;
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    const bool rows_ok = !epi.features_on_a && epi.out_sb == 1 && (N % 16) == 0 && al16(epi.out) &&
                         (epi.bias == nullptr || al16(epi.bias));
    if (epi.kind == kEpiResidual)
      ve.vec = (rows_ok && (epi.out_sa % 4) == 0 && (epi.gate_w == nullptr || al16(epi.gate_w)) &&
                (epi.gate_t == nullptr ||
                 (al16(epi.gate_t) && (epi.gate_bstride % 4) == 0 && (epi.gate_gstride % 4) == 0)))
                   ? 1
                   : 0;
    else if (epi.kind == kEpiStore)
      ve.vec = (rows_ok && (epi.out_sa % (epi.out_bf16 ? 8 : 4)) == 0) ? 1 : 0;
    else
      ve.vec = 0;
  }
  p->args.M = M;
  p->args.N = N;
  p->args.K = K;
  p->args.kb_per_split = kps;
  p->args.a_is_const = a_is_const ? 1 : 0;
  p->args.b_is_const = b_is_const ? 1 : 0;
  p->args.status = status;
  return 0;
}

}  // namespace fam
