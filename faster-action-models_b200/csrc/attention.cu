// Masked flash attention for the DiT blocks (SDPA with a bool mask, scale
// 1/sqrt(d): FastWAM/src/fastwam/models/wan22/wan_video_dit.py:13-22).
//
// One CTA = WARPS warps = a (16 x WARPS)-query tile of one (batch, head), over
// one split of the key range.  Keys come from up to two token-major sources:
// the cached video K/V of the layer and the fresh K/V of the current tokens
// (the joint attention of mot.py:560-566 concatenates exactly these two).
// K/V blocks of 64 keys stream through a double-buffered shared-memory ring
// with cp.async; the block's attend/ignore bits are staged next to them.
// QK^T and PV run on bf16 mma.sync tensor-core fragments with an fp32 online
// softmax in exp2 form.  With several key splits (decode-style: few queries,
// a long cache) every split writes an unnormalised partial (O, m, l) and the
// last CTA to arrive for a (batch, head, query tile) merges them in split
// order (deterministic) and resets its arrival counter.
//
// Masks: an explicit [Sq, Skv] bool mask shared by the batch (the MoT action
// rows of fastwam.py:429-451), a per-batch key mask (text context padding),
// and the first-frame-causal rule of the video self-attention
// (wan_video_dit.py:514-518) as a descriptor instead of a materialised mask.
#include "fam_common.cuh"
#include "fam_kernels.h"
#include "fam_mma.cuh"

namespace fam {

constexpr int kAttnKB = 64;  // keys per block

template <int HD, int WARPS>
struct AttnCfg {
  static constexpr int kQTile = 16 * WARPS;
  static constexpr int kRow = HD + 8;  // padded row: conflict-free fragment loads
  static constexpr int kBlockElems = kAttnKB * kRow;
  static constexpr int kKVBytes = 2 /*stages*/ * 2 /*K,V*/ * kBlockElems * 2;
  static constexpr int kMaskBytes = 2 /*stages*/ * (kQTile * kAttnKB + kAttnKB);
  static constexpr int kBytes = kKVBytes + kMaskBytes;
};

// Key j of (b, h): pointer to its K (or V) row slice.
__device__ __forceinline__ const __nv_bfloat16* kv_row(const AttnArgs& a, bool is_v, int b, int h,
                                                       int j, int hd) {
  if (j < a.S1) {
    const __nv_bfloat16* base = is_v ? a.v1 : a.k1;
    return base + b * a.kv1_bs + static_cast<long long>(j) * a.kv1_ts + h * hd;
  }
  j -= a.S1;
  const __nv_bfloat16* base = is_v ? a.v2 : a.k2;
  return base + b * a.kv2_bs + static_cast<long long>(j) * a.kv2_ts + h * hd;
}

template <int HD, int WARPS>
__device__ __forceinline__ void load_kv_block(const AttnArgs& a, __nv_bfloat16* sk,
                                              __nv_bfloat16* sv, int b, int h, int j0, int j_end) {
  using Cfg = AttnCfg<HD, WARPS>;
  constexpr int kChunks = HD / 8;  // 16-byte chunks per row
  for (int idx = threadIdx.x; idx < kAttnKB * kChunks; idx += blockDim.x) {
    const int r = idx / kChunks, c = idx % kChunks;
    const int j = j0 + r;
    const bool valid = j < j_end;
    const __nv_bfloat16* kp = valid ? kv_row(a, false, b, h, j, HD) + c * 8 : a.q;
    const __nv_bfloat16* vp = valid ? kv_row(a, true, b, h, j, HD) + c * 8 : a.q;
    cp_async16(sk + r * Cfg::kRow + c * 8, kp, valid);
    cp_async16(sv + r * Cfg::kRow + c * 8, vp, valid);
  }
}

// Raw mask bytes of the (query tile, key block) -> sm[QT][64], and the per-batch
// key-mask bytes -> sk[64].  16-byte cp.async copies with zero fill past the
// row end (or past Sq) when the strides allow; plain byte loads otherwise.
// Bytes of keys >= skv are zero (ignored by the validity test anyway).
template <int HD, int WARPS>
__device__ __forceinline__ void stage_mask(const AttnArgs& a, uint8_t* sm, uint8_t* sk, int b,
                                           int q0, int j0, int skv) {
  using Cfg = AttnCfg<HD, WARPS>;
  if (a.mask2d != nullptr) {
    const bool vec = (a.mask_rs % 16 == 0) && ((reinterpret_cast<uintptr_t>(a.mask2d) & 15) == 0);
    if (vec) {
      for (int idx = threadIdx.x; idx < Cfg::kQTile * (kAttnKB / 16); idx += blockDim.x) {
        const int qi = idx / (kAttnKB / 16), c = idx % (kAttnKB / 16);
        const int q = q0 + qi, j = j0 + 16 * c;
        int n = skv - j;
        n = n < 0 ? 0 : (n > 16 ? 16 : n);
        if (q >= a.Sq) n = 0;
        const uint8_t* src = n > 0 ? a.mask2d + static_cast<long long>(q) * a.mask_rs + j : a.mask2d;
        asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(sm + qi * kAttnKB + 16 * c)),
                     "l"(src), "r"(n)
                     : "memory");
      }
    } else {
      for (int idx = threadIdx.x; idx < Cfg::kQTile * kAttnKB; idx += blockDim.x) {
        const int qi = idx / kAttnKB, jj = idx % kAttnKB;
        const int q = q0 + qi, j = j0 + jj;
        sm[idx] = (q < a.Sq && j < skv) ? a.mask2d[static_cast<long long>(q) * a.mask_rs + j] : 0;
      }
    }
  }
  if (a.key_mask != nullptr) {
    const uint8_t* km = a.key_mask + b * a.key_mask_bs;
    for (int jj = threadIdx.x; jj < kAttnKB; jj += blockDim.x) {
      const int j = j0 + jj;
      sk[jj] = j < skv ? km[j] : 0;
    }
  }
}

template <int HD, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) attention_kernel(const AttnArgs a) {
  using Cfg = AttnCfg<HD, WARPS>;
  constexpr int QT = Cfg::kQTile;
  extern __shared__ __align__(16) uint8_t attn_smem[];
  __nv_bfloat16* smem = reinterpret_cast<__nv_bfloat16*>(attn_smem);
  uint8_t* smask = attn_smem + Cfg::kKVBytes;
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int h = blockIdx.y, b = blockIdx.z;
  const int split = blockIdx.x % a.nsplit;
  const int qt = blockIdx.x / a.nsplit;
  const int q_tiles = (a.Sq + QT - 1) / QT;
  const int skv = a.S1 + a.S2;
  const int k_begin = split * a.keys_per_split;
  const int k_end = min(skv, k_begin + a.keys_per_split);
  const int q0 = qt * QT;
  const int qr0 = q0 + warp * 16 + g, qr1 = qr0 + 8;  // the two rows this thread owns
  const bool use_m2 = a.mask2d != nullptr, use_km = a.key_mask != nullptr;
  const int ff = a.first_frame_tokens;
  const int nblocks = k_end > k_begin ? (k_end - k_begin + kAttnKB - 1) / kAttnKB : 0;
  __nv_bfloat16* sK[2] = {smem, smem + 2 * Cfg::kBlockElems};
  __nv_bfloat16* sV[2] = {smem + Cfg::kBlockElems, smem + 3 * Cfg::kBlockElems};
  uint8_t* sM[2] = {smask, smask + QT * kAttnKB};
  uint8_t* sKm[2] = {smask + 2 * QT * kAttnKB, smask + 2 * QT * kAttnKB + kAttnKB};

  // The first key block streams in before the programmatic-launch wait when it
  // lies in a source that no earlier kernel of the chain writes (the video K/V
  // cache); masks are call inputs and always qualify.
  const bool pre = a.kv1_const && nblocks > 0 && min(k_begin + kAttnKB, k_end) <= a.S1;
  if (pre) {
    load_kv_block<HD, WARPS>(a, sK[0], sV[0], b, h, k_begin, k_end);
    stage_mask<HD, WARPS>(a, sM[0], sKm[0], b, q0, k_begin, skv);
  }
  pdl_wait();
  pdl_launch_dependents();

  // Q fragments (A operand, row-major 16 x HD) straight from global.
  constexpr int KS = HD / 16;
  uint32_t qf[KS][4];
  {
    const __nv_bfloat16* qa = a.q + b * a.q_bs + static_cast<long long>(min(qr0, a.Sq - 1)) * a.q_ts + h * HD;
    const __nv_bfloat16* qb = a.q + b * a.q_bs + static_cast<long long>(min(qr1, a.Sq - 1)) * a.q_ts + h * HD;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      qf[kk][0] = *reinterpret_cast<const uint32_t*>(qa + kk * 16 + 2 * t);
      qf[kk][1] = *reinterpret_cast<const uint32_t*>(qb + kk * 16 + 2 * t);
      qf[kk][2] = *reinterpret_cast<const uint32_t*>(qa + kk * 16 + 8 + 2 * t);
      qf[kk][3] = *reinterpret_cast<const uint32_t*>(qb + kk * 16 + 8 + 2 * t);
    }
  }

  constexpr int NT = HD / 8;  // output dim tiles
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

  if (!pre && nblocks > 0) {
    load_kv_block<HD, WARPS>(a, sK[0], sV[0], b, h, k_begin, k_end);
    stage_mask<HD, WARPS>(a, sM[0], sKm[0], b, q0, k_begin, skv);
  }
  cp_async_commit();
  for (int blk = 0; blk < nblocks; ++blk) {
    const int cur = blk & 1;
    const int j0 = k_begin + blk * kAttnKB;
    if (blk + 1 < nblocks) {
      load_kv_block<HD, WARPS>(a, sK[cur ^ 1], sV[cur ^ 1], b, h, j0 + kAttnKB, k_end);
      stage_mask<HD, WARPS>(a, sM[cur ^ 1], sKm[cur ^ 1], b, q0, j0 + kAttnKB, skv);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    const __nv_bfloat16* K = sK[cur];
    const __nv_bfloat16* V = sV[cur];
    const uint8_t* M = sM[cur];
    const uint8_t* Km = sKm[cur];
    // S = Q K^T for 64 keys: 8 tiles of 8 keys; K fragments by ldmatrix (two
    // 16-dim k steps per x4 load: matrices = dims +0, +8, +16, +24 of 8 keys)
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
      const uint32_t kaddr = smem_u32(K + (n * 8 + (lane & 7)) * Cfg::kRow + (lane >> 3) * 8);
#pragma unroll
      for (int kk = 0; kk < KS; kk += 2) {
        uint32_t b4[4];
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                     : "=r"(b4[0]), "=r"(b4[1]), "=r"(b4[2]), "=r"(b4[3])
                     : "r"(kaddr + kk * 32));
        mma_bf16_16816(s[n], qf[kk], b4);
        mma_bf16_16816(s[n], qf[kk + 1], b4 + 2);
      }
    }
    // scale + mask, row max.  A block every row of the tile sees whole (no
    // explicit or key mask, inside the key range, outside the first-frame rule)
    // skips the per-element tests.
    float mx0 = -INFINITY, mx1 = -INFINITY;
    const int r0 = warp * 16 + g, r1 = r0 + 8;  // rows inside the tile
    const bool whole = !use_m2 && !use_km && j0 + kAttnKB <= k_end && (ff == 0 || q0 >= ff || j0 + kAttnKB <= ff);
    if (whole) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          s[n][e] *= a.scale_log2;
          s[n][2 + e] *= a.scale_log2;
          mx0 = fmaxf(mx0, s[n][e]);
          mx1 = fmaxf(mx1, s[n][2 + e]);
        }
      }
    } else {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int jj = n * 8 + 2 * t + e;
          const int j = j0 + jj;
          bool kv_ok = j < k_end;
          if (use_km) kv_ok = kv_ok && Km[jj] != 0;
          bool ok0 = kv_ok && qr0 < a.Sq && (ff == 0 || qr0 >= ff || j < ff);
          bool ok1 = kv_ok && qr1 < a.Sq && (ff == 0 || qr1 >= ff || j < ff);
          if (use_m2) {
            ok0 = ok0 && M[r0 * kAttnKB + jj] != 0;
            ok1 = ok1 && M[r1 * kAttnKB + jj] != 0;
          }
          s[n][e] = ok0 ? s[n][e] * a.scale_log2 : -INFINITY;
          s[n][2 + e] = ok1 ? s[n][2 + e] * a.scale_log2 : -INFINITY;
          mx0 = fmaxf(mx0, s[n][e]);
          mx1 = fmaxf(mx1, s[n][2 + e]);
        }
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.0f : mn0;
    const float base1 = mn1 == -INFINITY ? 0.0f : mn1;
    const float al0 = exp2f(m0 - base0), al1 = exp2f(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.0f, ps1 = 0.0f;
    uint32_t pf[4][4];  // P as A fragments: 4 k-steps of 16 keys
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = exp2f(s[n][0] - base0), p1 = exp2f(s[n][1] - base0);
      const float p2 = exp2f(s[n][2] - base1), p3 = exp2f(s[n][3] - base1);
      ps0 += p0 + p1;
      ps1 += p2 + p3;
      const int ks = n >> 1, hi = n & 1;
      pf[ks][hi ? 2 : 0] = pack_bf16(p0, p1);
      pf[ks][hi ? 3 : 1] = pack_bf16(p2, p3);
    }
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      o[i][0] *= al0;
      o[i][1] *= al0;
      o[i][2] *= al1;
      o[i][3] *= al1;
    }
    // O += P V : B fragments of V via ldmatrix.trans (rows = keys).
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        uint32_t bf[2];
        const int r = ks * 16 + (lane & 15);
        const uint32_t addr = smem_u32(V + r * Cfg::kRow + i * 8);
        asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
                     : "=r"(bf[0]), "=r"(bf[1])
                     : "r"(addr));
        mma_bf16_16816(o[i], pf[ks], bf);
      }
    }
    __syncthreads();
  }

  // Full row sums across the 4 threads of a quad.
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  if (a.nsplit == 1) {
    const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f;
    const float inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const int d = i * 8 + 2 * t;
      if (qr0 < a.Sq)
        *reinterpret_cast<uint32_t*>(a.out + b * a.out_bs + static_cast<long long>(qr0) * a.out_ts + h * HD + d) =
            pack_bf16(o[i][0] * inv0, o[i][1] * inv0);
      if (qr1 < a.Sq)
        *reinterpret_cast<uint32_t*>(a.out + b * a.out_bs + static_cast<long long>(qr1) * a.out_ts + h * HD + d) =
            pack_bf16(o[i][2] * inv1, o[i][3] * inv1);
    }
    return;
  }

  // ---- split partials + last-arriving-CTA merge
  const int Sq_pad = q_tiles * QT;
  const long long unit = (static_cast<long long>(b) * a.H + h) * a.nsplit;  // (b, h) base
  const long long ml_base = static_cast<long long>(gridDim.z) * a.H * a.nsplit * Sq_pad * HD;
  float* po = a.part + (unit + split) * Sq_pad * HD;
  float* pml = a.part + ml_base + (unit + split) * Sq_pad * 2;
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int d = i * 8 + 2 * t;
    *reinterpret_cast<float2*>(po + static_cast<long long>(qr0) * HD + d) = make_float2(o[i][0], o[i][1]);
    *reinterpret_cast<float2*>(po + static_cast<long long>(qr1) * HD + d) = make_float2(o[i][2], o[i][3]);
  }
  if (t == 0) {
    *reinterpret_cast<float2*>(pml + qr0 * 2) = make_float2(m0, l0);
    *reinterpret_cast<float2*>(pml + qr1 * 2) = make_float2(m1, l1);
  }
  __threadfence();
  __syncthreads();
  int* ctr = a.counters + (static_cast<long long>(b) * a.H + h) * q_tiles + qt;
  if (threadIdx.x == 0) s_last = (atomicAdd(ctr, 1) == a.nsplit - 1) ? 1 : 0;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Merge in two passes over smem (the K/V ring is free now): per query the
  // split weights exp2(m_s - M) / L, then every output element as an
  // independent weighted sum over splits.
  float* wsm = reinterpret_cast<float*>(attn_smem);  // [QT][nsplit]
  const float* po0 = a.part + unit * Sq_pad * HD;
  const float* pml0 = a.part + ml_base + unit * Sq_pad * 2;
  for (int ql = threadIdx.x; ql < QT; ql += blockDim.x) {
    const int q = q0 + ql;
    float M = -INFINITY;
    for (int s2 = 0; s2 < a.nsplit; ++s2) M = fmaxf(M, __ldcg(pml0 + (static_cast<long long>(s2) * Sq_pad + q) * 2));
    const float base = M == -INFINITY ? 0.0f : M;
    float L = 0.0f;
    for (int s2 = 0; s2 < a.nsplit; ++s2) {
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(pml0 + (static_cast<long long>(s2) * Sq_pad + q) * 2));
      const float w = exp2f(ml.x - base);
      wsm[ql * a.nsplit + s2] = w;
      L += w * ml.y;
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    for (int s2 = 0; s2 < a.nsplit; ++s2) wsm[ql * a.nsplit + s2] *= inv;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < QT * (HD / 4); idx += blockDim.x) {
    const int ql = idx / (HD / 4);
    const int d = (idx % (HD / 4)) * 4;
    const int q = q0 + ql;
    if (q >= a.Sq) continue;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* wq = wsm + ql * a.nsplit;
#pragma unroll 4
    for (int s2 = 0; s2 < a.nsplit; ++s2) {
      const float4 ov = __ldcg(reinterpret_cast<const float4*>(po0 + (static_cast<long long>(s2) * Sq_pad + q) * HD + d));
      const float w = wq[s2];
      acc.x += w * ov.x;
      acc.y += w * ov.y;
      acc.z += w * ov.z;
      acc.w += w * ov.w;
    }
    uint2 pk;
    pk.x = pack_bf16(acc.x, acc.y);
    pk.y = pack_bf16(acc.z, acc.w);
    *reinterpret_cast<uint2*>(a.out + b * a.out_bs + static_cast<long long>(q) * a.out_ts + h * HD + d) = pk;
  }
  if (threadIdx.x == 0) *ctr = 0;  // ready for the next launch
}

// Query-tile width used for a launch: 32 queries for small query counts (the
// action tokens), 64 otherwise.
static int attn_warps(int Sq) { return Sq <= 32 ? 2 : (Sq < 512 ? 4 : 8); }

size_t attn_partial_bytes(int B, int H, int Sq, int head_dim, int nsplit) {
  if (nsplit <= 1) return 0;
  const int qt = 16 * attn_warps(Sq);
  const size_t Sq_pad = static_cast<size_t>((Sq + qt - 1) / qt) * qt;
  return static_cast<size_t>(B) * H * nsplit * Sq_pad * (head_dim + 2) * sizeof(float);
}

int attn_query_tiles(int Sq) {
  const int qt = 16 * attn_warps(Sq);
  return (Sq + qt - 1) / qt;
}

int attn_auto_splits(int units, int skv, int* keys_per_split) {
  int splits = (296 + units - 1) / units;
  const int max_by_keys = (skv + 127) / 128;
  if (splits > max_by_keys) splits = max_by_keys;
  if (splits < 1) splits = 1;
  if (splits > 64) splits = 64;
  int kps = (skv + splits - 1) / splits;
  kps = (kps + kAttnKB - 1) / kAttnKB * kAttnKB;
  *keys_per_split = kps;
  return (skv + kps - 1) / kps;
}

template <int HD, int WARPS>
static cudaError_t launch_attn_cfg(const AttnArgs& a, int B, cudaStream_t st, bool pdl) {
  using Cfg = AttnCfg<HD, WARPS>;
  // The merge reuses the K/V ring for QT x nsplit weights.
  if (a.nsplit > 64 || Cfg::kQTile * a.nsplit * 4 > Cfg::kKVBytes) return cudaErrorInvalidValue;
  const int q_tiles = (a.Sq + Cfg::kQTile - 1) / Cfg::kQTile;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(q_tiles * a.nsplit, a.H, B);
  cfg.blockDim = dim3(WARPS * 32);
  cfg.dynamicSmemBytes = Cfg::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr_l[1];
  attr_l[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr_l[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr_l;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attention_kernel<HD, WARPS>, a);
}

cudaError_t attn_init_attributes() {
#define FAM_ATTN_ATTR(HD, W)                                                                  \
  {                                                                                           \
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<HD, W>,                             \
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,         \
                                         AttnCfg<HD, W>::kBytes);                             \
    if (e != cudaSuccess) return e;                                                           \
  }
  FAM_ATTN_ATTR(64, 2) FAM_ATTN_ATTR(64, 4) FAM_ATTN_ATTR(64, 8) FAM_ATTN_ATTR(128, 2) FAM_ATTN_ATTR(128, 4)
  FAM_ATTN_ATTR(128, 8)
#undef FAM_ATTN_ATTR
  return cudaSuccess;
}

cudaError_t launch_attention(const AttnArgs& a, int B, int head_dim, cudaStream_t st, bool pdl) {
  static bool attrs = false;
  if (!attrs) {
    cudaError_t e = attn_init_attributes();
    if (e != cudaSuccess) return e;
    attrs = true;
  }
  const int w = attn_warps(a.Sq);
  if (head_dim == 64)
    return w == 2 ? launch_attn_cfg<64, 2>(a, B, st, pdl)
                  : (w == 4 ? launch_attn_cfg<64, 4>(a, B, st, pdl) : launch_attn_cfg<64, 8>(a, B, st, pdl));
  if (head_dim == 128)
    return w == 2 ? launch_attn_cfg<128, 2>(a, B, st, pdl)
                  : (w == 4 ? launch_attn_cfg<128, 4>(a, B, st, pdl) : launch_attn_cfg<128, 8>(a, B, st, pdl));
  return cudaErrorInvalidValue;
}

}  // namespace fam
