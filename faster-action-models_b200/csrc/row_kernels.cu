// Row-wise HBM/L2-bound kernels of the DiT blocks.  One CTA owns one token row
// so that every full-row reduction (LayerNorm, RMSNorm over the whole H*d
// attention width) stays on chip; rows are read once with 128-bit loads and
// reduced with warp shuffles.
//
//   resid_norm   split-K reduction of the previous GEMM + bias + gated
//                residual add (fp32 residual stream, or bf16 roundings as the
//                reference's bf16 tensors) + the next LayerNorm
//                (AdaLN with (1+scale)/shift, or affine norm3) -> bf16 operand
//   qkv_post     split-K reduction of the fused QKV GEMM + bias, RMSNorm of q
//                and k over the whole H*d row, RoPE from an fp32 cos/sin table,
//                token-major bf16 q / k / v
//   rms_rows     split-K reduction + bias + RMSNorm over the row -> bf16
//   sinusoid     timestep embedding cat[cos, sin](t * 10000^(-i/half)) in fp64
//   encode_adaln action_encoder Linear(A -> D) + the first block's AdaLN
//   head_euler   head Linear(D -> A) + flow-matching Euler update
//
// Reference numerics followed (FastWAM/src/fastwam/models/wan22/...):
//   LayerNorm eps / affine: wan_video_dit.py:240-242; modulate: :26-27
//   RMSNorm: wan_video_dit.py:146-157 (fp32 statistics, cast, x weight)
//   RoPE: wan_video_dit.py:54-60 (adjacent pairs (2i, 2i+1) within a head)
//   split modulation (block.modulation + t_mod): mot.py:69-86
//   sinusoid: wan_video_dit.py:30-34; Euler: scheduler_continuous.py:82-88
#include "fam_common.cuh"
#include "fam_kernels.h"

namespace fam {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.0f;
  if (w == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[32] = t;
  __syncthreads();
  return red[32];
}

// Offset of the modulation row of `row` (see ModRows in fam_kernels.h).
__device__ __forceinline__ long long mod_row_offset(const ModRows& m, int row) {
  const int b = row / m.tokens_per_batch;
  const int within = row - b * m.tokens_per_batch;
  const int g = (m.first_frame_tokens > 0 && within >= m.first_frame_tokens) ? 1 : 0;
  return b * m.bstride + g * m.gstride;
}

// Value of modulation chunk c (0..5) at feature f for this row:
// bf16(bf16(t_mod) + modulation), the reference's bf16 (modulation + t_mod).
__device__ __forceinline__ float mod_value(const ModRows& m, long long off, int c, int f, int D) {
  float v = rbf(m.tmod[off + static_cast<long long>(c) * D + f]);
  if (m.mod_w != nullptr) v = rbf(v + bf2f(m.mod_w[c * D + f]));
  return v;
}

// Vector helpers: 4 consecutive columns per thread (128-bit fp32 loads, 64-bit
// bf16 loads), all split-K partial loads of a group issued back to back.
__device__ __forceinline__ float4 f4add(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float4 ld_bf4(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
}
__device__ __forceinline__ void st_bf4(__nv_bfloat16* p, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ float4 rbf4(float4 v) {
  return make_float4(rbf(v.x), rbf(v.y), rbf(v.z), rbf(v.w));
}
// Sum over splits of partials[s * split_stride + off .. +3] in split order.
__device__ __forceinline__ float4 sum_splits4(const float* partials, long long split_stride,
                                              int nsplit, long long off) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  int s = 0;
  for (; s + 4 <= nsplit; s += 4) {
    const float4 v0 = __ldcg(reinterpret_cast<const float4*>(partials + (s + 0) * split_stride + off));
    const float4 v1 = __ldcg(reinterpret_cast<const float4*>(partials + (s + 1) * split_stride + off));
    const float4 v2 = __ldcg(reinterpret_cast<const float4*>(partials + (s + 2) * split_stride + off));
    const float4 v3 = __ldcg(reinterpret_cast<const float4*>(partials + (s + 3) * split_stride + off));
    acc = f4add(acc, f4add(f4add(v0, v1), f4add(v2, v3)));
  }
  for (; s < nsplit; ++s)
    acc = f4add(acc, __ldcg(reinterpret_cast<const float4*>(partials + s * split_stride + off)));
  return acc;
}
// Modulation chunk c for 4 features: bf16(bf16(t_mod) + modulation).
__device__ __forceinline__ float4 mod_value4(const ModRows& m, long long off, int c, int f, int D) {
  float4 t = rbf4(*reinterpret_cast<const float4*>(m.tmod + off + static_cast<long long>(c) * D + f));
  if (m.mod_w != nullptr) {
    const float4 w = ld_bf4(m.mod_w + c * D + f);
    t = rbf4(make_float4(t.x + w.x, t.y + w.y, t.z + w.z, t.w + w.w));
  }
  return t;
}

// ---------------------------------------------------------------- resid_norm
// Each thread owns column groups g = threadIdx.x + i * blockDim.x (4 columns
// each, NG = ceil(D / 1024) of them); the updated row stays in registers.
// NG and the presence of the residual update are compile-time, so that the
// registers (and the CTAs resident per SM) follow the row width: a norm-only
// D = 3072 row keeps 3 groups of constants, not 4 groups of both sets.
constexpr int kMaxGroups = 4;  // D <= 4 * 4 * 256 = 4096
template <int NG, bool RESID>
__global__ void __launch_bounds__(kRowThreads) resid_norm_kernel(const ResidNormArgs a) {
  __shared__ float red[33];
  const int row = blockIdx.x;
  const int D = a.D;
  const int G = D / 4;
  float* x = a.x + static_cast<long long>(row) * D;
  const long long moff = (RESID && a.mod.tmod != nullptr) ? mod_row_offset(a.mod, row) : 0;
  const long long noff = a.nmod.tmod != nullptr ? mod_row_offset(a.nmod, row) : 0;
  // Constants of the chain (bias, gate, norm affine / shift / scale) load before
  // the programmatic-launch wait; only x and the partials depend on it.
  float4 cb[NG], cg[NG], c0[NG], c1[NG];
#pragma unroll
  for (int i = 0; i < NG; ++i) {
    const int g = threadIdx.x + i * blockDim.x;
    if (g >= G) break;
    const int f = 4 * g;
    if (RESID) {
      cb[i] = a.bias != nullptr ? ld_bf4(a.bias + f) : make_float4(0.f, 0.f, 0.f, 0.f);
      cg[i] = a.gate_chunk >= 0 ? mod_value4(a.mod, moff, a.gate_chunk, f, D) : make_float4(1.f, 1.f, 1.f, 1.f);
    }
    if (a.norm_mode == kNormAffine) {
      c0[i] = ld_bf4(a.norm_w + f);
      c1[i] = ld_bf4(a.norm_b + f);
    } else if (a.norm_mode == kNormAdaLN) {
      c0[i] = mod_value4(a.nmod, noff, a.shift_chunk, f, D);      // shift
      c1[i] = mod_value4(a.nmod, noff, a.shift_chunk + 1, f, D);  // scale
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  float4 v[NG];
  float lsum = 0.0f;
#pragma unroll
  for (int i = 0; i < NG; ++i) {
    const int g = threadIdx.x + i * blockDim.x;
    if (g >= G) break;
    const int f = 4 * g;
    float4 xv = *reinterpret_cast<const float4*>(x + f);
    if (RESID) {
      float4 y = sum_splits4(a.partials, a.split_stride, a.nsplit, static_cast<long long>(row) * D + f);
      y = rbf4(f4add(y, cb[i]));  // the reference's Linear output is a bf16 tensor
      const float4 gt = cg[i];
      if (a.round_residual) {
        // bf16 residual stream: bf16(x + bf16(gate * y)), as the reference's bf16 tensors
        const float4 gy = rbf4(make_float4(gt.x * y.x, gt.y * y.y, gt.z * y.z, gt.w * y.w));
        xv = rbf4(make_float4(xv.x + gy.x, xv.y + gy.y, xv.z + gy.z, xv.w + gy.w));
      } else {
        xv = make_float4(xv.x + gt.x * y.x, xv.y + gt.y * y.y, xv.z + gt.z * y.z, xv.w + gt.w * y.w);
      }
      *reinterpret_cast<float4*>(x + f) = xv;
    }
    v[i] = xv;
    lsum += xv.x + xv.y + xv.z + xv.w;
  }
  if (a.norm_mode == kNormNone) return;
  const float mean = block_sum(lsum, red) / D;
  float lvar = 0.0f;
#pragma unroll
  for (int i = 0; i < NG; ++i) {
    const int g = threadIdx.x + i * blockDim.x;
    if (g >= G) break;
    const float4 d = make_float4(v[i].x - mean, v[i].y - mean, v[i].z - mean, v[i].w - mean);
    lvar += d.x * d.x + d.y * d.y + d.z * d.z + d.w * d.w;
  }
  const float rstd = rsqrtf(block_sum(lvar, red) / D + a.eps);
  __nv_bfloat16* h = a.h + static_cast<long long>(row) * a.h_stride;
#pragma unroll
  for (int i = 0; i < NG; ++i) {
    const int g = threadIdx.x + i * blockDim.x;
    if (g >= G) break;
    const int f = 4 * g;
    float4 n = make_float4((v[i].x - mean) * rstd, (v[i].y - mean) * rstd, (v[i].z - mean) * rstd,
                           (v[i].w - mean) * rstd);
    if (a.norm_mode == kNormAffine) {
      const float4 w = c0[i], b = c1[i];
      n = make_float4(n.x * w.x + b.x, n.y * w.y + b.y, n.z * w.z + b.z, n.w * w.w + b.w);
    } else {  // AdaLN: LN(x) * (1 + scale) + shift
      const float4 sh = c0[i];
      const float4 sc = c1[i];
      // modulate on bf16 tensors: bf16(bf16(n * bf16(1 + scale)) + shift)
      n = rbf4(n);
      n = make_float4(rbf(n.x * rbf(1.f + sc.x)), rbf(n.y * rbf(1.f + sc.y)), rbf(n.z * rbf(1.f + sc.z)),
                      rbf(n.w * rbf(1.f + sc.w)));
      n = make_float4(n.x + sh.x, n.y + sh.y, n.z + sh.z, n.w + sh.w);
    }
    st_bf4(h + f, n);
  }
}

// --------------------------------------------------------- norm rows (4 per CTA)
// The norm-only form of resid_norm (the residual already updated by a GEMM
// epilogue, as in the backbone prefill).  A CTA normalises kNrRows rows, 64
// threads (two warps) per row, D / 256 float4 groups per thread in registers,
// so each thread has 4x the bytes of the CTA-per-row form in flight and the
// two CTA barriers (mean, variance) serve 4 rows.  The norm constants -- the
// affine weight and bias, or the AdaLN shift and scale of the rows' modulation
// row when the CTA's rows share it -- are built once per CTA in shared memory
// before the programmatic-launch wait (rows with different modulation rows
// read theirs directly).
constexpr int kNrRows = 4;
constexpr int kNrMaxD = 4096;
struct NormRowsArgs {
  ResidNormArgs a;
  int rows;
};
template <int NV>
__global__ void __launch_bounds__(kRowThreads) norm_rows_kernel(const NormRowsArgs na) {
  __shared__ __align__(16) float cst[2 * kNrMaxD];  // weight / shift, then bias / scale
  __shared__ float red[kNrRows][2][2];              // [row][warp][sum, sum of squares]
  const ResidNormArgs& a = na.a;
  const int D = a.D;
  const int r = threadIdx.x >> 6, t = threadIdx.x & 63, w = (threadIdx.x >> 5) & 1, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kNrRows, row = row0 + r;
  const int last = min(row0 + kNrRows, na.rows) - 1;
  const bool ada = a.norm_mode == kNormAdaLN;
  const long long off0 = ada ? mod_row_offset(a.nmod, row0) : 0;
  const bool shared_c = !ada || mod_row_offset(a.nmod, last) == off0;
  if (shared_c) {
    for (int g = threadIdx.x; g < D / 4; g += kRowThreads) {
      const int f = 4 * g;
      float4 c0, c1;
      if (ada) {
        c0 = mod_value4(a.nmod, off0, a.shift_chunk, f, D);
        c1 = mod_value4(a.nmod, off0, a.shift_chunk + 1, f, D);
      } else {
        c0 = ld_bf4(a.norm_w + f);
        c1 = ld_bf4(a.norm_b + f);
      }
      *reinterpret_cast<float4*>(cst + f) = c0;
      *reinterpret_cast<float4*>(cst + kNrMaxD + f) = c1;
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  const bool live = row < na.rows;
  float4 v[NV];
  float s = 0.f;
  const float* x = a.x + static_cast<long long>(live ? row : 0) * D;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = live ? *reinterpret_cast<const float4*>(x + 4 * (t + 64 * i)) : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  s = warp_sum(s);
  if (lane == 0) red[r][w][0] = s;
  __syncthreads();  // also publishes the constants
  const float mean = (red[r][0][0] + red[r][1][0]) / D;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float4 d = make_float4(v[i].x - mean, v[i].y - mean, v[i].z - mean, v[i].w - mean);
    q += (d.x * d.x + d.y * d.y) + (d.z * d.z + d.w * d.w);
  }
  q = warp_sum(q);
  if (lane == 0) red[r][w][1] = q;
  __syncthreads();
  if (!live) return;
  const float rstd = rsqrtf((red[r][0][1] + red[r][1][1]) / D + a.eps);
  const long long noff = ada && !shared_c ? mod_row_offset(a.nmod, row) : off0;
  __nv_bfloat16* h = a.h + static_cast<long long>(row) * a.h_stride;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int f = 4 * (t + 64 * i);
    float4 n = make_float4((v[i].x - mean) * rstd, (v[i].y - mean) * rstd, (v[i].z - mean) * rstd,
                           (v[i].w - mean) * rstd);
    if (ada) {  // bf16(bf16(LN(x) * bf16(1 + scale)) + shift), the reference's bf16 steps
      const float4 sh = shared_c ? *reinterpret_cast<const float4*>(cst + f) : mod_value4(a.nmod, noff, a.shift_chunk, f, D);
      const float4 sc = shared_c ? *reinterpret_cast<const float4*>(cst + kNrMaxD + f)
                                 : mod_value4(a.nmod, noff, a.shift_chunk + 1, f, D);
      n = rbf4(n);
      n = make_float4(rbf(n.x * rbf(1.f + sc.x)), rbf(n.y * rbf(1.f + sc.y)), rbf(n.z * rbf(1.f + sc.z)),
                      rbf(n.w * rbf(1.f + sc.w)));
      n = make_float4(n.x + sh.x, n.y + sh.y, n.z + sh.z, n.w + sh.w);
    } else {
      const float4 wt = *reinterpret_cast<const float4*>(cst + f), b = *reinterpret_cast<const float4*>(cst + kNrMaxD + f);
      n = make_float4(n.x * wt.x + b.x, n.y * wt.y + b.y, n.z * wt.z + b.z, n.w * wt.w + b.w);
    }
    st_bf4(h + f, n);
  }
}

// ------------------------------------------------------------------ qkv_post
// One CTA per token row; dynamic smem: 2*HD floats (q and k before the norm).
__global__ void __launch_bounds__(kRowThreads) qkv_post_kernel(const QkvPostArgs a) {
  extern __shared__ float sbuf[];
  __shared__ float red[33];
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int HD = a.HD;
  const int N3 = 3 * HD;
  float* sq = sbuf;  // [0, HD) q, [HD, 2HD) k
  float ssq = 0.0f, ssk = 0.0f;
  for (int g = threadIdx.x; g < N3 / 4; g += blockDim.x) {
    const int f = 4 * g;
    float4 y;
    if (a.nsplit > 0)
      y = sum_splits4(a.partials, a.split_stride, a.nsplit, static_cast<long long>(row) * N3 + f);
    else
      y = ld_bf4(a.qkv_bf16 + static_cast<long long>(row) * N3 + f);
    if (a.bias != nullptr) y = f4add(y, ld_bf4(a.bias + f));
    y = rbf4(y);
    const float s2 = y.x * y.x + y.y * y.y + y.z * y.z + y.w * y.w;
    if (f < 2 * HD) {
      *reinterpret_cast<float4*>(sq + f) = y;
      if (f < HD) ssq += s2; else ssk += s2;
    } else {
      st_bf4(a.v_out + static_cast<long long>(row) * a.out_stride + (f - 2 * HD), y);
    }
  }
  const float rq = rsqrtf(block_sum(ssq, red) / HD + a.eps);
  const float rk = rsqrtf(block_sum(ssk, red) / HD + a.eps);
  const int pos = row % a.rows_per_batch;
  const int half = a.head_dim / 2;
  const float2* tab = a.rope + static_cast<long long>(pos) * half;
  for (int g = threadIdx.x; g < HD / 2; g += blockDim.x) {  // q groups then k groups
    const bool is_k = g >= HD / 4;
    const int f = 4 * (is_k ? g - HD / 4 : g);
    const float r = is_k ? rk : rq;
    const float4 y = *reinterpret_cast<const float4*>(sq + (is_k ? HD : 0) + f);
    const float4 w = ld_bf4((is_k ? a.norm_k : a.norm_q) + f);
    const float x0 = rbf(rbf(y.x * r) * w.x), x1 = rbf(rbf(y.y * r) * w.y);
    const float x2 = rbf(rbf(y.z * r) * w.z), x3 = rbf(rbf(y.w * r) * w.w);
    const int i = (f % a.head_dim) / 2;  // first pair index inside the head (even)
    const float4 cs = *reinterpret_cast<const float4*>(tab + i);  // (cos_i, sin_i, cos_i+1, sin_i+1)
    const float4 o = make_float4(x0 * cs.x - x1 * cs.y, x0 * cs.y + x1 * cs.x,
                                 x2 * cs.z - x3 * cs.w, x2 * cs.w + x3 * cs.z);
    st_bf4((is_k ? a.k_out : a.q_out) + static_cast<long long>(row) * a.out_stride + f, o);
  }
}

// qkv_post over a bf16 [rows, 3HD] input that already holds the bias (the
// GEMM epilogue adds it), in 16-byte groups (HD and head_dim multiples of 8,
// 16-byte aligned rows).  Each thread issues every load of its
// part of the row before using any, so one memory latency covers the row; the
// RoPE table and the norm weights load before the programmatic-launch wait, and
// the q and k sums of squares share one block reduction.  Per element the
// arithmetic is the one of qkv_post_kernel.
constexpr int kQkvLoads = 5;  // 8-column groups per thread: 3HD <= 5 * 8 * kRowThreads
constexpr int kQkvNorm = 3;   // q and k groups per thread: 2HD <= 3 * 8 * kRowThreads

__device__ __forceinline__ void unpack_bf8(const uint4 u, float* o) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 t = __bfloat1622float2(h[k]);
    o[2 * k] = t.x;
    o[2 * k + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack_bf8(const float* v) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
  return u;
}

__device__ __forceinline__ float2 block_sum2(float2 v, float2* red) {
  v.x = warp_sum(v.x);
  v.y = warp_sum(v.y);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float2 t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : make_float2(0.0f, 0.0f);
  if (w == 0) {
    t.x = warp_sum(t.x);
    t.y = warp_sum(t.y);
  }
  if (threadIdx.x == 0) red[32] = t;
  __syncthreads();
  return red[32];
}

__global__ void __launch_bounds__(kRowThreads, 3) qkv_post_wide_kernel(const QkvPostArgs a) {
  extern __shared__ float sbuf[];
  __shared__ float2 red[33];
  const int row = blockIdx.x;
  const int HD = a.HD, G = 3 * HD / 8, GQ = HD / 4, GK = HD / 8;
  const int half = a.head_dim / 2;
  const float2* tab = a.rope + static_cast<long long>(row % a.rows_per_batch) * half;
  uint4 wv[kQkvNorm];
  float4 c0[kQkvNorm], c1[kQkvNorm];
#pragma unroll
  for (int j = 0; j < kQkvNorm; ++j) {
    const int g = threadIdx.x + j * kRowThreads;
    if (g < GQ) {
      const bool is_k = g >= GK;
      const int f = 8 * (is_k ? g - GK : g);
      wv[j] = *reinterpret_cast<const uint4*>((is_k ? a.norm_k : a.norm_q) + f);
      const int i = (f % a.head_dim) / 2;  // first pair index inside the head (multiple of 4)
      c0[j] = *reinterpret_cast<const float4*>(tab + i);
      c1[j] = *reinterpret_cast<const float4*>(tab + i + 2);
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  const __nv_bfloat16* in = a.qkv_bf16 + static_cast<long long>(row) * 3 * HD;
  uint4 raw[kQkvLoads];
#pragma unroll
  for (int j = 0; j < kQkvLoads; ++j) {
    const int g = threadIdx.x + j * kRowThreads;
    if (g < G) raw[j] = *reinterpret_cast<const uint4*>(in + 8 * g);
  }
  float* sq = sbuf;  // [0, HD) q, [HD, 2HD) k
  float ssq = 0.0f, ssk = 0.0f;
#pragma unroll
  for (int j = 0; j < kQkvLoads; ++j) {
    const int g = threadIdx.x + j * kRowThreads;
    if (g < G) {
      const int f = 8 * g;
      float y[8];
      unpack_bf8(raw[j], y);
      if (f < 2 * HD) {
        float s2 = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) s2 += y[e] * y[e];
        if (f < HD) ssq += s2; else ssk += s2;
        *reinterpret_cast<float4*>(sq + f) = make_float4(y[0], y[1], y[2], y[3]);
        *reinterpret_cast<float4*>(sq + f + 4) = make_float4(y[4], y[5], y[6], y[7]);
      } else {
        *reinterpret_cast<uint4*>(a.v_out + static_cast<long long>(row) * a.out_stride + (f - 2 * HD)) =
            pack_bf8(y);
      }
    }
  }
  const float2 ss = block_sum2(make_float2(ssq, ssk), red);
  const float rq = rsqrtf(ss.x / HD + a.eps);
  const float rk = rsqrtf(ss.y / HD + a.eps);
#pragma unroll
  for (int j = 0; j < kQkvNorm; ++j) {
    const int g = threadIdx.x + j * kRowThreads;
    if (g < GQ) {  // the same thread wrote these columns to shared memory above
      const bool is_k = g >= GK;
      const int f = 8 * (is_k ? g - GK : g);
      const float r = is_k ? rk : rq;
      const float* src = sq + (is_k ? HD : 0) + f;
      float w[8], x[8], o[8];
      unpack_bf8(wv[j], w);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = rbf(rbf(src[e] * r) * w[e]);
      const float cs[8] = {c0[j].x, c0[j].y, c0[j].z, c0[j].w, c1[j].x, c1[j].y, c1[j].z, c1[j].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // (cos, sin) of pair q
        o[2 * q] = x[2 * q] * cs[2 * q] - x[2 * q + 1] * cs[2 * q + 1];
        o[2 * q + 1] = x[2 * q] * cs[2 * q + 1] + x[2 * q + 1] * cs[2 * q];
      }
      *reinterpret_cast<uint4*>((is_k ? a.k_out : a.q_out) + static_cast<long long>(row) * a.out_stride + f) =
          pack_bf8(o);
    }
  }
}

// ------------------------------------------------------ qkv_post (2 rows per CTA)
// The wide form for the backbone's row counts: 2 rows per CTA, 128 threads per
// row, the row's 8-column groups g = t, t + 128, ... (9 per thread at HD =
// 3072) loaded at once into registers; V is stored on arrival, q and k stay in
// registers until their row's sums of squares are reduced (warp shuffles, one
// CTA barrier), and the q / k norm weights and the rows' RoPE tables are staged
// in shared memory before the launch wait.  Each SM keeps 4x the rows of the
// CTA-per-row form in flight.  Per element the arithmetic is qkv_post_kernel's.
constexpr int kQpRows = 2;
constexpr int kQpThreads = kRowThreads / kQpRows;
constexpr int kQpLoads = 9;      // 3 HD <= 9 * 8 * kQpThreads
constexpr int kQpMaxHD = 3072;
constexpr int kQpMaxHalf = 128;  // head_dim / 2
struct QkvRowsArgs {
  QkvPostArgs a;
  int rows;
};
__global__ void __launch_bounds__(kRowThreads) qkv_post_rows_kernel(const QkvRowsArgs na) {
  __shared__ __align__(16) __nv_bfloat16 wq[kQpMaxHD];
  __shared__ __align__(16) __nv_bfloat16 wk[kQpMaxHD];
  __shared__ __align__(16) float2 rope_s[kQpRows][kQpMaxHalf];
  __shared__ float2 red[kQpRows][kQpThreads / 32];
  const QkvPostArgs& a = na.a;
  const int rows = na.rows, HD = a.HD, G = 3 * HD / 8, GQ = HD / 8, half = a.head_dim / 2;
  const int r = threadIdx.x / kQpThreads, t = threadIdx.x % kQpThreads, wr = t >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kQpRows, row = row0 + r;
  const bool live = row < rows;
  for (int i = threadIdx.x; i < GQ; i += kRowThreads) {
    reinterpret_cast<uint4*>(wq)[i] = reinterpret_cast<const uint4*>(a.norm_q)[i];
    reinterpret_cast<uint4*>(wk)[i] = reinterpret_cast<const uint4*>(a.norm_k)[i];
  }
  for (int i = threadIdx.x; i < kQpRows * half; i += kRowThreads) {
    const int rr = i / half, p = i - rr * half, rw = min(row0 + rr, rows - 1);
    rope_s[rr][p] = a.rope[static_cast<long long>(rw % a.rows_per_batch) * half + p];
  }
  pdl_wait();
  pdl_launch_dependents();
  const __nv_bfloat16* in = a.qkv_bf16 + static_cast<long long>(live ? row : 0) * 3 * HD;
  uint4 raw[kQpLoads];
#pragma unroll
  for (int j = 0; j < kQpLoads; ++j) {
    const int g = t + j * kQpThreads;
    if (live && g < G) raw[j] = *reinterpret_cast<const uint4*>(in + 8 * g);
  }
  float ssq = 0.0f, ssk = 0.0f;
#pragma unroll
  for (int j = 0; j < kQpLoads; ++j) {
    const int g = t + j * kQpThreads;
    if (!live || g >= G) continue;
    if (g >= 2 * GQ) {
      *reinterpret_cast<uint4*>(a.v_out + static_cast<long long>(row) * a.out_stride + 8 * (g - 2 * GQ)) = raw[j];
    } else {
      float y[8];
      unpack_bf8(raw[j], y);
      float s2 = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) s2 += y[e] * y[e];
      if (g < GQ) ssq += s2; else ssk += s2;
    }
  }
  ssq = warp_sum(ssq);
  ssk = warp_sum(ssk);
  if (lane == 0) red[r][wr] = make_float2(ssq, ssk);
  __syncthreads();  // also publishes the staged constants
  if (!live) return;
  float2 tot = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kQpThreads / 32; ++i) tot = make_float2(tot.x + red[r][i].x, tot.y + red[r][i].y);
  const float rq = rsqrtf(tot.x / HD + a.eps);
  const float rk = rsqrtf(tot.y / HD + a.eps);
#pragma unroll
  for (int j = 0; j < kQpLoads; ++j) {
    const int g = t + j * kQpThreads;
    if (g >= 2 * GQ) continue;
    const bool is_k = g >= GQ;
    const int f = 8 * (is_k ? g - GQ : g);
    const float rs = is_k ? rk : rq;
    float y[8], w[8], x[8], o[8];
    unpack_bf8(raw[j], y);
    unpack_bf8(*reinterpret_cast<const uint4*>((is_k ? wk : wq) + f), w);
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = rbf(rbf(y[e] * rs) * w[e]);
    const float2* cs = &rope_s[r][(f % a.head_dim) / 2];
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // (cos, sin) of pair q
      const float2 c = cs[q];
      o[2 * q] = x[2 * q] * c.x - x[2 * q + 1] * c.y;
      o[2 * q + 1] = x[2 * q] * c.y + x[2 * q + 1] * c.x;
    }
    *reinterpret_cast<uint4*>((is_k ? a.k_out : a.q_out) + static_cast<long long>(row) * a.out_stride + f) =
        pack_bf8(o);
  }
}

// ------------------------------------------------------------------ rms_rows
// out = RMSNorm(sum partials + bias) * w, one CTA per row.  With nsplit == 0
// the input is a bf16 matrix (in place allowed).  dynamic smem: N floats.
__global__ void __launch_bounds__(kRowThreads) rms_rows_kernel(const RmsRowsArgs a) {
  extern __shared__ float sbuf[];
  __shared__ float red[33];
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  float ss = 0.0f;
  for (int g = threadIdx.x; g < a.N / 4; g += blockDim.x) {
    const int f = 4 * g;
    float4 y;
    if (a.nsplit > 0)
      y = sum_splits4(a.partials, a.split_stride, a.nsplit, static_cast<long long>(row) * a.N + f);
    else
      y = ld_bf4(a.in + static_cast<long long>(row) * a.in_stride + f);
    if (a.bias != nullptr) y = f4add(y, ld_bf4(a.bias + f));
    y = rbf4(y);
    *reinterpret_cast<float4*>(sbuf + f) = y;
    ss += y.x * y.x + y.y * y.y + y.z * y.z + y.w * y.w;
  }
  const float r = rsqrtf(block_sum(ss, red) / a.N + a.eps);
  const __nv_bfloat16* wr = a.w + (a.w_period > 0 ? static_cast<long long>(row % a.w_period) * a.w_stride : 0);
  for (int g = threadIdx.x; g < a.N / 4; g += blockDim.x) {
    const int f = 4 * g;
    const float4 y = *reinterpret_cast<const float4*>(sbuf + f);
    const float4 w = ld_bf4(wr + f);
    st_bf4(a.out + static_cast<long long>(row) * a.out_stride + f,
           make_float4(rbf(y.x * r) * w.x, rbf(y.y * r) * w.y, rbf(y.z * r) * w.z, rbf(y.w * r) * w.w));
  }
}

// rms_rows over a bias-free bf16 input in 16-byte groups: the weights load
// before the programmatic-launch wait, every load of a thread's part of the row
// is in flight at once and the row stays in registers (in place allowed: each
// thread writes only the columns it read).  Per element the arithmetic is the
// one of rms_rows_kernel.
constexpr int kRmsLoads = 2;  // 8-column groups per thread: N <= 2 * 8 * kRowThreads

__global__ void __launch_bounds__(kRowThreads) rms_rows_wide_kernel(const RmsRowsArgs a) {
  __shared__ float red[33];
  const int row = blockIdx.x;
  const int G = a.N / 8;
  const __nv_bfloat16* wr = a.w + (a.w_period > 0 ? static_cast<long long>(row % a.w_period) * a.w_stride : 0);
  uint4 wv[kRmsLoads];
#pragma unroll
  for (int j = 0; j < kRmsLoads; ++j) {
    const int g = threadIdx.x + j * kRowThreads;
    if (g < G) wv[j] = *reinterpret_cast<const uint4*>(wr + 8 * g);
  }
  pdl_wait();
  pdl_launch_dependents();
  const __nv_bfloat16* in = a.in + static_cast<long long>(row) * a.in_stride;
  uint4 raw[kRmsLoads];
#pragma unroll
  for (int j = 0; j < kRmsLoads; ++j) {
    const int g = threadIdx.x + j * kRowThreads;
    if (g < G) raw[j] = *reinterpret_cast<const uint4*>(in + 8 * g);
  }
  float y[kRmsLoads][8];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kRmsLoads; ++j) {
    const int g = threadIdx.x + j * kRowThreads;
    if (g < G) {
      unpack_bf8(raw[j], y[j]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += y[j][e] * y[j][e];
    }
  }
  const float r = rsqrtf(block_sum(ss, red) / a.N + a.eps);
  __nv_bfloat16* out = a.out + static_cast<long long>(row) * a.out_stride;
#pragma unroll
  for (int j = 0; j < kRmsLoads; ++j) {
    const int g = threadIdx.x + j * kRowThreads;
    if (g < G) {
      float w[8], o[8];
      unpack_bf8(wv[j], w);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = rbf(y[j][e] * r) * w[e];
      *reinterpret_cast<uint4*>(out + 8 * g) = pack_bf8(o);
    }
  }
}

// ------------------------------------------------------------------ sinusoid
// out[r][i] = cos(t_r * 10000^(-i/half)), out[r][half+i] = sin(...), computed
// in fp64 and rounded to bf16 (the timestep dtype of a bf16 model).
__global__ void sinusoid_kernel(const StepTimes t, int rows, int dim, __nv_bfloat16* out) {
  pdl_wait();
  pdl_launch_dependents();
  const int half = dim / 2;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < rows * half;
       idx += gridDim.x * blockDim.x) {
    const int r = idx / half, i = idx % half;
    const double freq = pow(10000.0, -static_cast<double>(i) / static_cast<double>(half));
    const double arg = static_cast<double>(t.t[r]) * freq;
    out[static_cast<long long>(r) * dim + i] = __double2bfloat16(cos(arg));
    out[static_cast<long long>(r) * dim + half + i] = __double2bfloat16(sin(arg));
  }
}

// -------------------------------------------------------------- encode_adaln
// x[row] = action_encoder(latent[row]) (bf16-rounded, as the reference's bf16
// Linear output), h[row] = AdaLN of block 0.  dynamic smem: D floats.
__global__ void __launch_bounds__(kRowThreads) encode_adaln_kernel(const EncodeArgs a) {
  extern __shared__ float srow[];
  __shared__ float red[33];
  __shared__ float lat[64];
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int D = a.D;
  if (threadIdx.x < a.A) lat[threadIdx.x] = bf2f(a.latent[static_cast<long long>(row) * a.A + threadIdx.x]);
  __syncthreads();
  float lsum = 0.0f;
  for (int f = threadIdx.x; f < D; f += blockDim.x) {
    float y = a.enc_b != nullptr ? bf2f(a.enc_b[f]) : 0.0f;
    for (int j = 0; j < a.A; ++j) y += bf2f(a.enc_w[f * a.A + j]) * lat[j];
    y = rbf(y);
    a.x[static_cast<long long>(row) * D + f] = y;
    srow[f] = y;
    lsum += y;
  }
  const float mean = block_sum(lsum, red) / D;
  float lvar = 0.0f;
  for (int f = threadIdx.x; f < D; f += blockDim.x) {
    const float d = srow[f] - mean;
    lvar += d * d;
  }
  const float rstd = rsqrtf(block_sum(lvar, red) / D + a.eps);
  const long long moff = mod_row_offset(a.mod, row);
  for (int f = threadIdx.x; f < D; f += blockDim.x) {
    const float shift = mod_value(a.mod, moff, 0, f, D);
    const float scale = mod_value(a.mod, moff, 1, f, D);
    const float n = rbf(rbf((srow[f] - mean) * rstd) * rbf(1.0f + scale)) + shift;
    a.h[static_cast<long long>(row) * D + f] = f2bf(n);
  }
}

// ---------------------------------------------------------------- head_euler
// v = head(x) (x rounded to bf16 like the reference's bf16 residual stream),
// latent <- latent + v * delta with the reference's bf16 roundings.  One warp
// per (row, action channel).
__global__ void head_euler_kernel(const HeadArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int warps = blockDim.x >> 5;
  const int gw = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= a.rows * a.A) return;
  const int row = gw / a.A, c = gw % a.A;
  const float* x = a.x + static_cast<long long>(row) * a.D;
  const __nv_bfloat16* w = a.head_w + static_cast<long long>(c) * a.D;
  float acc = 0.0f;
  for (int f = lane; f < a.D; f += 32) acc += rbf(x[f]) * bf2f(w[f]);
  acc = warp_sum(acc);
  if (lane == 0) {
    float v = rbf(acc + (a.head_b != nullptr ? bf2f(a.head_b[c]) : 0.0f));
    const long long idx = static_cast<long long>(row) * a.A + c;
    if (a.velocity != nullptr) a.velocity[idx] = f2bf(v);
    if (a.latent != nullptr && a.apply_euler) {
      const float d = rbf(a.delta);
      a.latent[idx] = f2bf(bf2f(a.latent[idx]) + rbf(v * d));
    }
  }
}

// ------------------------------------------------------------------ launches
template <typename K, typename Args>
static cudaError_t launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              bool pdl, const Args& args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args);
}

static cudaError_t ensure_smem(const void* fn, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
}

template <bool RESID>
static cudaError_t launch_resid_norm_t(const ResidNormArgs& a, int rows, cudaStream_t st, bool pdl) {
  switch ((a.D + 4 * kRowThreads - 1) / (4 * kRowThreads)) {
    case 1: return launch_pdl(resid_norm_kernel<1, RESID>, dim3(rows), dim3(kRowThreads), 0, st, pdl, a);
    case 2: return launch_pdl(resid_norm_kernel<2, RESID>, dim3(rows), dim3(kRowThreads), 0, st, pdl, a);
    case 3: return launch_pdl(resid_norm_kernel<3, RESID>, dim3(rows), dim3(kRowThreads), 0, st, pdl, a);
    default: return launch_pdl(resid_norm_kernel<4, RESID>, dim3(rows), dim3(kRowThreads), 0, st, pdl, a);
  }
}

cudaError_t launch_resid_norm(const ResidNormArgs& a, int rows, cudaStream_t st, bool pdl) {
  if (a.D % 4 != 0 || a.D > 4 * kMaxGroups * kRowThreads) return cudaErrorInvalidValue;
  if (a.partials == nullptr && (a.norm_mode == kNormAffine || a.norm_mode == kNormAdaLN) && a.D % 256 == 0 &&
      a.D <= kNrMaxD && a.h_stride % 4 == 0) {
    const dim3 grid((rows + kNrRows - 1) / kNrRows);
    const NormRowsArgs na = {a, rows};
    switch (a.D / 256) {
      case 4: return launch_pdl(norm_rows_kernel<4>, grid, dim3(kRowThreads), 0, st, pdl, na);
      case 8: return launch_pdl(norm_rows_kernel<8>, grid, dim3(kRowThreads), 0, st, pdl, na);
      case 12: return launch_pdl(norm_rows_kernel<12>, grid, dim3(kRowThreads), 0, st, pdl, na);
      case 16: return launch_pdl(norm_rows_kernel<16>, grid, dim3(kRowThreads), 0, st, pdl, na);
      default: break;
    }
  }
  return a.partials != nullptr ? launch_resid_norm_t<true>(a, rows, st, pdl)
                               : launch_resid_norm_t<false>(a, rows, st, pdl);
}

cudaError_t launch_qkv_post(const QkvPostArgs& a, int rows, cudaStream_t st, bool pdl) {
  const size_t smem = sizeof(float) * 2 * a.HD;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool wide = a.nsplit == 0 && a.qkv_bf16 != nullptr && a.bias == nullptr && a.HD % 8 == 0 &&
                    a.head_dim % 8 == 0 && 3 * a.HD <= kQkvLoads * 8 * kRowThreads &&
                    2 * a.HD <= kQkvNorm * 8 * kRowThreads && a.out_stride % 8 == 0 && al16(a.qkv_bf16) &&
                    al16(a.norm_q) && al16(a.norm_k) && al16(a.rope) && al16(a.q_out) && al16(a.k_out) &&
                    al16(a.v_out);
  if (wide && a.HD <= kQpMaxHD && 3 * a.HD <= kQpLoads * 8 * kQpThreads && a.head_dim / 2 <= kQpMaxHalf) {
    const QkvRowsArgs na = {a, rows};
    return launch_pdl(qkv_post_rows_kernel, dim3((rows + kQpRows - 1) / kQpRows), dim3(kRowThreads), 0, st, pdl,
                      na);
  }
  if (wide) {
    cudaError_t e = ensure_smem(reinterpret_cast<const void*>(qkv_post_wide_kernel), smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(qkv_post_wide_kernel, dim3(rows), dim3(kRowThreads), smem, st, pdl, a);
  }
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(qkv_post_kernel), smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(qkv_post_kernel, dim3(rows), dim3(kRowThreads), smem, st, pdl, a);
}

cudaError_t launch_rms_rows(const RmsRowsArgs& a, int rows, cudaStream_t st, bool pdl) {
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (a.nsplit == 0 && a.in != nullptr && a.bias == nullptr && a.N % 8 == 0 &&
      a.N <= kRmsLoads * 8 * kRowThreads && a.in_stride % 8 == 0 && a.out_stride % 8 == 0 &&
      (a.w_period <= 0 || a.w_stride % 8 == 0) && al16(a.in) && al16(a.out) && al16(a.w))
    return launch_pdl(rms_rows_wide_kernel, dim3(rows), dim3(kRowThreads), 0, st, pdl, a);
  const size_t smem = sizeof(float) * a.N;
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(rms_rows_kernel), smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(rms_rows_kernel, dim3(rows), dim3(kRowThreads), smem, st, pdl, a);
}

cudaError_t launch_sinusoid(const StepTimes& t, int rows, int dim, __nv_bfloat16* out, cudaStream_t st,
                            bool pdl) {
  const int total = rows * (dim / 2);
  const int blocks = (total + 255) / 256;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, sinusoid_kernel, t, rows, dim, out);
}

cudaError_t launch_encode_adaln(const EncodeArgs& a, int rows, cudaStream_t st, bool pdl) {
  const size_t smem = sizeof(float) * a.D;
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(encode_adaln_kernel), smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(encode_adaln_kernel, dim3(rows), dim3(kRowThreads), smem, st, pdl, a);
}

cudaError_t launch_head_euler(const HeadArgs& a, cudaStream_t st, bool pdl) {
  const int warps = a.rows * a.A;
  const int blocks = (warps + 7) / 8;
  return launch_pdl(head_euler_kernel, dim3(blocks), dim3(256), 0, st, pdl, a);
}

}  // namespace fam
