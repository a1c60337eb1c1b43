// Wan2.2 VAE encode of one observation frame (VideoVAE38_.encode with T = 1,
// FastWAM/src/fastwam/models/wan22/wan_video_vae.py:1285-1304, 619-733).
//
// Activations are channels-last [positions, channels] (one frame, batch 1);
// the residual stream is fp32, GEMM operands bf16.  A stride-1 3x3
// convolution is the tcgen05 GEMM of gemm_tc.cu in its implicit-convolution
// form (per tap the A rows of a zero-bordered buffer shift by dy * (W+2) + dx;
// RMS_norm and patchify write that layout); a stride-2 one is an im2col
// gather into [positions, 9 * C] (K order: dy, dx, c) + GEMM; 1x1
// convolutions are plain GEMMs.  With T = 1 the causal 3-D convolutions see
// two zero frames in front, so only the last temporal tap of their weights
// contributes (the host packs that slice).  The kernels here are the
// HBM-bound pieces around those GEMMs:
//   vae_patchify_kernel      patchify(2) of the [3, H, W] frame -> [P, 16] bf16
//   vae_im2col_kernel        3x3 (stride 1 or 2, asymmetric zero padding) gather
//   vae_rms_kernel           RMS_norm over channels (+ SiLU) -> bf16, and/or a
//                            plain bf16 copy of the fp32 stream
//   vae_avg_down_add_kernel  AvgDown3D shortcut added into the block output
//   vae_softmax_kernel       row softmax of the one-head attention scores
//   vae_transpose_kernel     V -> V^T for the P V product
//   vae_latent_kernel        (mu - mean) * inv_std, channel-first output
//   vae_splitk_kernel        sum of split-K GEMM partials + bias, stored or
//                            added into the fp32 stream (the few-tile
//                            low-resolution convolutions)
#include "../../include/fam.h"
#include "fam_common.cuh"
#include "fam_internal.h"

namespace fam {
namespace {

constexpr int kVaeThreads = 256;

// patchify: "b c f (h q) (w r) -> b (c r q) f h w" (wan_video_vae.py:199-212):
// output channel c * 4 + r * 2 + q of position (h, w) is image[c][2h + q][2w + r];
// channels 12..15 are zero padding for the 16-byte GEMM rows.
__global__ void vae_patchify_kernel(const __nv_bfloat16* __restrict__ img, int H, int W,
                                    __nv_bfloat16* __restrict__ out, long long out_ld, int pad) {
  const int h2 = H / 2, w2 = W / 2;
  const long long P = static_cast<long long>(h2) * w2;
  for (long long p = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; p < P;
       p += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int y = static_cast<int>(p / w2), x = static_cast<int>(p % w2);
    __nv_bfloat16 v[16];
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int q = 0; q < 2; ++q)
          v[c * 4 + r * 2 + q] = img[(static_cast<long long>(c) * H + 2 * y + q) * W + 2 * x + r];
#pragma unroll
    for (int c = 12; c < 16; ++c) v[c] = __float2bfloat16(0.f);
    const long long orow = pad ? static_cast<long long>(y + 1) * (w2 + 2) + x + 1 : p;
    uint4* o = reinterpret_cast<uint4*>(out + orow * out_ld);
    o[0] = *reinterpret_cast<const uint4*>(&v[0]);
    o[1] = *reinterpret_cast<const uint4*>(&v[8]);
  }
}

// 3x3 gather: dst[p][(dy * 3 + dx) * C + c] = src[y * s - pt + dy][x * s - pt + dx][c]
// (zero outside [0, H) x [0, W)); 8 channels (16 bytes) per thread.
__global__ void vae_im2col_kernel(const __nv_bfloat16* __restrict__ src, long long src_ld, int H, int W, int C,
                                  int stride, int pad, int Ho, int Wo, __nv_bfloat16* __restrict__ dst,
                                  long long dst_ld) {
  const int cg = C / 8;
  const long long total = static_cast<long long>(Ho) * Wo * 9 * cg;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(i % cg);
    const long long r = i / cg;
    const int tap = static_cast<int>(r % 9);
    const long long p = r / 9;
    const int y = static_cast<int>(p / Wo), x = static_cast<int>(p % Wo);
    const int iy = y * stride - pad + tap / 3, ix = x * stride - pad + tap % 3;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (iy >= 0 && iy < H && ix >= 0 && ix < W)
      v = *reinterpret_cast<const uint4*>(src + (static_cast<long long>(iy) * W + ix) * src_ld + 8 * g);
    *reinterpret_cast<uint4*>(dst + p * dst_ld + tap * C + 8 * g) = v;
  }
}

// RMS_norm over the channels of each position (wan_video_vae.py:55-70):
// x / max(||x||, 1e-12) * sqrt(C) * gamma, then SiLU when asked; one warp per
// position.  raw (nullable) receives bf16(x).  pad_w > 0: out is the
// zero-bordered buffer of a frame pad_w wide (position p at row
// (p / pad_w + 1) * (pad_w + 2) + p % pad_w + 1).
__global__ void vae_rms_kernel(const float* __restrict__ x, long long x_ld, long long P, int C,
                               const __nv_bfloat16* __restrict__ gamma, int silu_on,
                               __nv_bfloat16* __restrict__ out, long long out_ld, int pad_w,
                               __nv_bfloat16* __restrict__ raw, long long raw_ld) {
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x / 32);
  for (long long p = blockIdx.x * static_cast<long long>(blockDim.x / 32) + (threadIdx.x >> 5); p < P; p += warps) {
    const float* xr = x + p * x_ld;
    float ss = 0.f;
    for (int c = 4 * lane; c < C; c += 128) {
      const float4 v = *reinterpret_cast<const float4*>(xr + c);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      if (raw != nullptr) {
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(raw + p * raw_ld + c) = u;
      }
    }
    if (out == nullptr) continue;
    const int pi = static_cast<int>(p);  // positions < 2^31 (checked on the host)
    const long long orow = pad_w > 0 ? static_cast<long long>(pi / pad_w + 1) * (pad_w + 2) + pi % pad_w + 1 : p;
    ss = warp_sum(ss);
    const float k = sqrtf(static_cast<float>(C)) / fmaxf(sqrtf(ss), 1e-12f);
    for (int c = 4 * lane; c < C; c += 128) {
      const float4 v = *reinterpret_cast<const float4*>(xr + c);
      const float2 g0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(gamma + c));
      const float2 g1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(gamma + c + 2));
      float y[4] = {v.x * k * g0.x, v.y * k * g0.y, v.z * k * g1.x, v.w * k * g1.y};
      if (silu_on)
#pragma unroll
        for (int j = 0; j < 4; ++j) y[j] = silu(y[j]);
      __nv_bfloat162 a = __floats2bfloat162_rn(y[0], y[1]), b = __floats2bfloat162_rn(y[2], y[3]);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t*>(&a);
      u.y = *reinterpret_cast<uint32_t*>(&b);
      *reinterpret_cast<uint2*>(out + orow * out_ld + c) = u;
    }
  }
}

// AvgDown3D (wan_video_vae.py:345-395) of a one-frame input, added into out:
// the (c, t, ph, pw) flattening of the input with factor_t - 1 zero frames in
// front is averaged in groups of Cin * factor / Cout consecutive entries.
// (32-bit index arithmetic: the host checks that every index fits.)
__global__ void vae_avg_down_add_kernel(const float* __restrict__ in, int in_ld, int H, int W, int Cin,
                                        int Cout, int ft, int fs, float* __restrict__ out, int out_ld) {
  const int Ho = H / fs, Wo = W / fs;
  const int factor = ft * fs * fs, grp = Cin * factor / Cout;
  const int total = Ho * Wo * Cout;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int o = i % Cout;
    const int p = i / Cout;
    const int y = p / Wo, x = p - y * Wo;
    float acc = 0.f;
    for (int j = 0; j < grp; ++j) {
      const int f = o * grp + j;
      const int c = f / factor, rem = f % factor;
      const int t = rem / (fs * fs), ph = (rem / fs) % fs, pw = rem % fs;
      if (t < ft - 1) continue;  // a zero frame of the temporal padding
      acc += __ldg(in + ((y * fs + ph) * W + x * fs + pw) * in_ld + c);
    }
    out[p * out_ld + o] += acc / static_cast<float>(grp);
  }
}

// softmax(scale * s) over each row of the fp32 scores -> bf16 probabilities.
__global__ void vae_softmax_kernel(const float* __restrict__ s, long long s_ld, int cols, float scale,
                                   __nv_bfloat16* __restrict__ p, long long p_ld) {
  __shared__ float red[32];
  const float* row = s + blockIdx.x * s_ld;
  float m = -INFINITY;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, row[c] * scale);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = -INFINITY;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) sum += expf(row[c] * scale - m);
  sum = warp_sum(sum);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) sum += red[w];
  const float inv = 1.f / sum;
  __nv_bfloat16* pr = p + blockIdx.x * p_ld;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) pr[c] = __float2bfloat16(expf(row[c] * scale - m) * inv);
}

// dst[c][r] = src[r][c] (bf16), 32 x 32 tiles through shared memory.
__global__ void vae_transpose_kernel(const __nv_bfloat16* __restrict__ src, long long src_ld, int rows, int cols,
                                     __nv_bfloat16* __restrict__ dst, long long dst_ld) {
  __shared__ __nv_bfloat16 t[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    t[i][threadIdx.x] = (r < rows && c < cols) ? src[static_cast<long long>(r) * src_ld + c] : __float2bfloat16(0.f);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (c < cols && r < rows) dst[static_cast<long long>(c) * dst_ld + r] = t[threadIdx.x][i];
  }
}

// out[c][p] = (mu[p][c] - mean[c]) * inv_std[c] for the first z channels.
__global__ void vae_latent_kernel(const float* __restrict__ mu, long long mu_ld, long long P, int z,
                                  const float* __restrict__ mean, const float* __restrict__ inv_std,
                                  float* __restrict__ out) {
  const long long total = P * z;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i / P);
    const long long p = i % P;
    out[i] = (mu[p * mu_ld + c] - mean[c]) * inv_std[c];
  }
}

// out[m][n] (+)= bias[n] + sum_s part[s][m][n], four columns per thread.
__global__ void vae_splitk_kernel(const float* __restrict__ part, int splits, int M, int N,
                                  const __nv_bfloat16* __restrict__ bias, float* __restrict__ out, int out_ld,
                                  int accumulate) {
  const int nq = N / 4;
  const int total = M * nq;
  const long long sstride = static_cast<long long>(M) * N;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int m = i / nq;
    const int n = (i - m * nq) * 4;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (bias != nullptr) {
      const float2 b0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(bias + n));
      const float2 b1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(bias + n + 2));
      a = make_float4(b0.x, b0.y, b1.x, b1.y);
    }
    for (int sp = 0; sp < splits; ++sp) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(part + sp * sstride + static_cast<long long>(m) * N + n));
      a = make_float4(a.x + v.x, a.y + v.y, a.z + v.z, a.w + v.w);
    }
    float4* o = reinterpret_cast<float4*>(out + static_cast<long long>(m) * out_ld + n);
    if (accumulate) {
      const float4 r = *o;
      a = make_float4(a.x + r.x, a.y + r.y, a.z + r.z, a.w + r.w);
    }
    *o = a;
  }
}

int grid_for(long long work, int per_block) {
  long long g = (work + per_block - 1) / per_block;
  if (g > 148LL * 16) g = 148LL * 16;
  return static_cast<int>(g < 1 ? 1 : g);
}

int launched(const char* what) { return check_cuda(cudaGetLastError(), what); }

}  // namespace
}  // namespace fam

using namespace fam;

extern "C" {

int fam_vae_patchify(const void* image, int H, int W, void* out, int64_t out_ld, int pad, void* stream) {
  if (image == nullptr || out == nullptr || H <= 0 || W <= 0 || (H % 2) || (W % 2) || out_ld < 16)
    return set_error("fam_vae_patchify: bad arguments");
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (out_ld % 8))
    return set_error("fam_vae_patchify: output rows must be 16-byte aligned");
  const long long P = static_cast<long long>(H / 2) * (W / 2);
  vae_patchify_kernel<<<grid_for(P, kVaeThreads), kVaeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(image), H, W, static_cast<__nv_bfloat16*>(out), out_ld, pad);
  return launched("vae_patchify_kernel");
}

int fam_vae_im2col(const void* src, int64_t src_ld, int H, int W, int C, int stride, int pad, int Ho, int Wo,
                   void* dst, int64_t dst_ld, void* stream) {
  if (src == nullptr || dst == nullptr || H <= 0 || W <= 0 || C <= 0 || Ho <= 0 || Wo <= 0 || stride < 1)
    return set_error("fam_vae_im2col: bad arguments");
  if ((C % 8) || (src_ld % 8) || (dst_ld % 8) || dst_ld < 9LL * C || src_ld < C ||
      (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
    return set_error("fam_vae_im2col: channels and row strides must be 16-byte multiples");
  const long long total = static_cast<long long>(Ho) * Wo * 9 * (C / 8);
  vae_im2col_kernel<<<grid_for(total, kVaeThreads), kVaeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(src), src_ld, H, W, C, stride, pad, Ho, Wo,
      static_cast<__nv_bfloat16*>(dst), dst_ld);
  return launched("vae_im2col_kernel");
}

int fam_vae_rms(const float* x, int64_t x_ld, int64_t P, int C, const void* gamma, int silu_on, void* out,
                int64_t out_ld, int out_pad_w, void* raw, int64_t raw_ld, void* stream) {
  if (x == nullptr || P <= 0 || C <= 0 || (C % 4) || (x_ld % 4) || (out == nullptr && raw == nullptr) ||
      (out != nullptr && gamma == nullptr))
    return set_error("fam_vae_rms: bad arguments");
  if ((out != nullptr && (out_ld % 4)) || (raw != nullptr && (raw_ld % 4)))
    return set_error("fam_vae_rms: output row strides must be multiples of 4 elements");
  if (P >= (1LL << 31)) return set_error("fam_vae_rms: too many positions");
  const long long warps = P;
  vae_rms_kernel<<<grid_for(warps * 32, kVaeThreads), kVaeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, x_ld, P, C, static_cast<const __nv_bfloat16*>(gamma), silu_on, static_cast<__nv_bfloat16*>(out), out_ld,
      out_pad_w, static_cast<__nv_bfloat16*>(raw), raw_ld);
  return launched("vae_rms_kernel");
}

int fam_vae_avg_down_add(const float* in, int64_t in_ld, int H, int W, int Cin, int Cout, int factor_t,
                         int factor_s, float* out, int64_t out_ld, void* stream) {
  if (in == nullptr || out == nullptr || H <= 0 || W <= 0 || Cin <= 0 || Cout <= 0 || factor_t < 1 ||
      factor_s < 1 || (H % factor_s) || (W % factor_s) || ((Cin * factor_t * factor_s * factor_s) % Cout))
    return set_error("fam_vae_avg_down_add: bad arguments");
  const long long total = static_cast<long long>(H / factor_s) * (W / factor_s) * Cout;
  if (static_cast<long long>(H) * W * in_ld >= (1LL << 31) || total * out_ld / Cout >= (1LL << 31))
    return set_error("fam_vae_avg_down_add: frame too large for 32-bit indexing");
  vae_avg_down_add_kernel<<<grid_for(total, kVaeThreads), kVaeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      in, static_cast<int>(in_ld), H, W, Cin, Cout, factor_t, factor_s, out, static_cast<int>(out_ld));
  return launched("vae_avg_down_add_kernel");
}

int fam_vae_softmax(const float* s, int64_t s_ld, int rows, int cols, float scale, void* p, int64_t p_ld,
                    void* stream) {
  if (s == nullptr || p == nullptr || rows <= 0 || cols <= 0) return set_error("fam_vae_softmax: bad arguments");
  vae_softmax_kernel<<<rows, kVaeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      s, s_ld, cols, scale, static_cast<__nv_bfloat16*>(p), p_ld);
  return launched("vae_softmax_kernel");
}

int fam_vae_transpose(const void* src, int64_t src_ld, int rows, int cols, void* dst, int64_t dst_ld,
                      void* stream) {
  if (src == nullptr || dst == nullptr || rows <= 0 || cols <= 0) return set_error("fam_vae_transpose: bad arguments");
  dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
  vae_transpose_kernel<<<grid, block, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(src), src_ld, rows, cols, static_cast<__nv_bfloat16*>(dst), dst_ld);
  return launched("vae_transpose_kernel");
}

int fam_vae_latent(const float* mu, int64_t mu_ld, int64_t P, int z, const float* mean, const float* inv_std,
                   float* out, void* stream) {
  if (mu == nullptr || mean == nullptr || inv_std == nullptr || out == nullptr || P <= 0 || z <= 0)
    return set_error("fam_vae_latent: bad arguments");
  vae_latent_kernel<<<grid_for(P * z, kVaeThreads), kVaeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      mu, mu_ld, P, z, mean, inv_std, out);
  return launched("vae_latent_kernel");
}

int fam_vae_splitk_reduce(const float* partials, int splits, int64_t M, int N, const void* bias, float* out,
                          int64_t out_ld, int accumulate, void* stream) {
  if (partials == nullptr || out == nullptr || splits < 1 || M <= 0 || N <= 0 || (N % 4) || (out_ld % 4) ||
      (reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(partials) & 15))
    return set_error("fam_vae_splitk_reduce: bad arguments");
  if (M * N >= (1LL << 31) || M * out_ld >= (1LL << 31))
    return set_error("fam_vae_splitk_reduce: too large for 32-bit indexing");
  vae_splitk_kernel<<<grid_for(M * (N / 4), kVaeThreads), kVaeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      partials, splits, static_cast<int>(M), N, static_cast<const __nv_bfloat16*>(bias), out,
      static_cast<int>(out_ld), accumulate);
  return launched("vae_splitk_kernel");
}

}  // extern "C"
