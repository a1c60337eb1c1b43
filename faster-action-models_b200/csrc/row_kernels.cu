// Row-wise HBM/L2-bound kernels of the DiT blocks.  One CTA owns one token row
// so that every full-row reduction (LayerNorm, RMSNorm over the whole H*d
// attention width) stays on chip; rows are read once with 128-bit loads and
// reduced with warp shuffles.
//
//   resid_norm   split-K reduction of the previous GEMM + bias + gated
//                residual add (fp32 residual stream) + the next LayerNorm
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

// ---------------------------------------------------------------- resid_norm
// Dynamic shared memory: D floats (the updated row).
__global__ void __launch_bounds__(kRowThreads) resid_norm_kernel(const ResidNormArgs a) {
  extern __shared__ float srow[];
  __shared__ float red[33];
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int D = a.D;
  float* x = a.x + static_cast<long long>(row) * D;
  const long long moff = a.mod.tmod != nullptr ? mod_row_offset(a.mod, row) : 0;
  const long long noff = a.nmod.tmod != nullptr ? mod_row_offset(a.nmod, row) : 0;
  float lsum = 0.0f;
  for (int f = threadIdx.x; f < D; f += blockDim.x) {
    float v = x[f];
    if (a.partials != nullptr) {
      float y = 0.0f;
      for (int s = 0; s < a.nsplit; ++s)
        y += __ldcg(a.partials + static_cast<long long>(s) * a.split_stride +
                    static_cast<long long>(row) * D + f);
      if (a.bias != nullptr) y += bf2f(a.bias[f]);
      y = rbf(y);  // the reference's Linear output is a bf16 tensor
      const float g = (a.gate_chunk >= 0) ? mod_value(a.mod, moff, a.gate_chunk, f, D) : 1.0f;
      v += g * y;
      if (a.round_residual) v = rbf(v);
      x[f] = v;
    }
    srow[f] = v;
    lsum += v;
  }
  if (a.norm_mode == kNormNone) return;
  const float mean = block_sum(lsum, red) / D;
  float lvar = 0.0f;
  for (int f = threadIdx.x; f < D; f += blockDim.x) {
    const float d = srow[f] - mean;
    lvar += d * d;
  }
  const float rstd = rsqrtf(block_sum(lvar, red) / D + a.eps);
  __nv_bfloat16* h = a.h + static_cast<long long>(row) * a.h_stride;
  for (int f = threadIdx.x; f < D; f += blockDim.x) {
    float n = (srow[f] - mean) * rstd;
    if (a.norm_mode == kNormAffine) {
      n = n * bf2f(a.norm_w[f]) + bf2f(a.norm_b[f]);
    } else {  // AdaLN: LN(x) * (1 + scale) + shift
      const float shift = mod_value(a.nmod, noff, a.shift_chunk, f, D);
      const float scale = mod_value(a.nmod, noff, a.shift_chunk + 1, f, D);
      n = rbf(n) * (1.0f + scale) + shift;
    }
    h[f] = f2bf(n);
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
  float* sq = sbuf;
  float* sk = sbuf + HD;
  float ssq = 0.0f, ssk = 0.0f;
  for (int f = threadIdx.x; f < N3; f += blockDim.x) {
    float y = 0.0f;
    if (a.nsplit > 0) {
      for (int s = 0; s < a.nsplit; ++s)
        y += __ldcg(a.partials + static_cast<long long>(s) * a.split_stride +
                    static_cast<long long>(row) * N3 + f);
    } else {
      y = bf2f(a.qkv_bf16[static_cast<long long>(row) * N3 + f]);
    }
    if (a.bias != nullptr) y += bf2f(a.bias[f]);
    y = rbf(y);
    if (f < HD) {
      sq[f] = y;
      ssq += y * y;
    } else if (f < 2 * HD) {
      sk[f - HD] = y;
      ssk += y * y;
    } else {
      a.v_out[static_cast<long long>(row) * a.out_stride + (f - 2 * HD)] = f2bf(y);
    }
  }
  const float rq = rsqrtf(block_sum(ssq, red) / HD + a.eps);
  const float rk = rsqrtf(block_sum(ssk, red) / HD + a.eps);
  const int pos = row % a.rows_per_batch;
  const int half = a.head_dim / 2;
  const float2* tab = a.rope + static_cast<long long>(pos) * half;
  // Each thread rotates pairs (2i, 2i+1) of q and of k.
  for (int pidx = threadIdx.x; pidx < HD / 2; pidx += blockDim.x) {
    const int f0 = 2 * pidx;
    const int i = pidx % half;  // pair index inside the head
    const float2 cs = tab[i];   // (cos, sin)
    {
      const float x0 = rbf(rbf(sq[f0] * rq) * bf2f(a.norm_q[f0]));
      const float x1 = rbf(rbf(sq[f0 + 1] * rq) * bf2f(a.norm_q[f0 + 1]));
      __nv_bfloat162 o = __floats2bfloat162_rn(x0 * cs.x - x1 * cs.y, x0 * cs.y + x1 * cs.x);
      *reinterpret_cast<__nv_bfloat162*>(a.q_out + static_cast<long long>(row) * a.out_stride + f0) = o;
    }
    {
      const float x0 = rbf(rbf(sk[f0] * rk) * bf2f(a.norm_k[f0]));
      const float x1 = rbf(rbf(sk[f0 + 1] * rk) * bf2f(a.norm_k[f0 + 1]));
      __nv_bfloat162 o = __floats2bfloat162_rn(x0 * cs.x - x1 * cs.y, x0 * cs.y + x1 * cs.x);
      *reinterpret_cast<__nv_bfloat162*>(a.k_out + static_cast<long long>(row) * a.out_stride + f0) = o;
    }
  }
}

// ------------------------------------------------------------------ rms_rows
// out = RMSNorm(sum partials + bias) * w, one CTA per row.  With nsplit == 0
// the input is a bf16 matrix (in place allowed).
__global__ void __launch_bounds__(kRowThreads) rms_rows_kernel(const RmsRowsArgs a) {
  extern __shared__ float sbuf[];
  __shared__ float red[33];
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  float ss = 0.0f;
  for (int f = threadIdx.x; f < a.N; f += blockDim.x) {
    float y = 0.0f;
    if (a.nsplit > 0) {
      for (int s = 0; s < a.nsplit; ++s)
        y += __ldcg(a.partials + static_cast<long long>(s) * a.split_stride +
                    static_cast<long long>(row) * a.N + f);
    } else {
      y = bf2f(a.in[static_cast<long long>(row) * a.in_stride + f]);
    }
    if (a.bias != nullptr) y += bf2f(a.bias[f]);
    y = rbf(y);
    sbuf[f] = y;
    ss += y * y;
  }
  const float r = rsqrtf(block_sum(ss, red) / a.N + a.eps);
  for (int f = threadIdx.x; f < a.N; f += blockDim.x)
    a.out[static_cast<long long>(row) * a.out_stride + f] = f2bf(rbf(sbuf[f] * r) * bf2f(a.w[f]));
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
    const float n = rbf((srow[f] - mean) * rstd) * (1.0f + scale) + shift;
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

cudaError_t launch_resid_norm(const ResidNormArgs& a, int rows, cudaStream_t st, bool pdl) {
  const size_t smem = sizeof(float) * a.D;
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(resid_norm_kernel), smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(resid_norm_kernel, dim3(rows), dim3(kRowThreads), smem, st, pdl, a);
}

cudaError_t launch_qkv_post(const QkvPostArgs& a, int rows, cudaStream_t st, bool pdl) {
  const size_t smem = sizeof(float) * 2 * a.HD;
  cudaError_t e = ensure_smem(reinterpret_cast<const void*>(qkv_post_kernel), smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(qkv_post_kernel, dim3(rows), dim3(kRowThreads), smem, st, pdl, a);
}

cudaError_t launch_rms_rows(const RmsRowsArgs& a, int rows, cudaStream_t st, bool pdl) {
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
