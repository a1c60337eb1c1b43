// Action-VAE decoder (ActionDecoder.forward,
// FastWAM/src/fastwam/models/action_ae.py:123-166), fp32.
//
// Wide path (hidden % 4 == 0, the layer's input fits shared memory):
//   dec_layer_kernel   one CTA per (4 output channels, sample).  It stages its
//                      weight slice with cp.async before waiting on the
//                      previous launch (programmatic dependent launch), then
//                      builds the layer input in shared memory -- input_proj
//                      (+ suite embedding) of z, SiLU(GroupNorm(raw conv)), or
//                      skip + GroupNorm(raw conv) -- with the GroupNorm
//                      statistics recomputed by every CTA from the whole raw
//                      tensor, and writes the raw ConvTranspose1d(k=2s, stride
//                      s, pad s/2) or Conv1d(k=3, pad 1) output of its channels.
//   dec_head_kernel    skip + GroupNorm of the last stage, crop / zero-pad to
//                      the horizon, output_proj.
// Narrow fallback (kept for other shapes):
//   dec_input_kernel, dec_conv_kernel (one CTA per (sample, GroupNorm group):
//   conv + GroupNorm + SiLU / skip in shared memory), dec_output_kernel.
//
// GroupNorm(min(8, h), h, eps 1e-5, affine) and the residual block
// [Conv1d -> GN -> SiLU -> Conv1d -> GN] + skip follow action_ae.py:33-47.
#include "fam_common.cuh"
#include "fam_cae.h"
#include "fam_mma.cuh"

#include <cstring>

namespace fam {

constexpr int kDecThreads = 256;
constexpr int kDecMaxGroupElems = 8192;  // channels-per-group x length held in smem

__global__ void dec_input_kernel(const __grid_constant__ DecArgs a, float* x) {
  const int b = blockIdx.x;
  const int h = a.cfg.hidden, T = a.cfg.num_tokens, Z = a.cfg.latent_dim;
  const int sid = (a.suite_ids != nullptr && a.suite_embed != nullptr) ? a.suite_ids[b] : -1;
  for (int i = threadIdx.x; i < h * T; i += blockDim.x) {
    const int c = i / T, t = i % T;
    float acc = a.in_b[c];
    const float* zr = a.z + (static_cast<long long>(b) * T + t) * Z;
    if (a.lat_std != nullptr) {
      for (int k = 0; k < Z; ++k)
        acc += a.in_w[c * Z + k] * __fadd_rn(__fmul_rn(zr[k], a.lat_std[t * Z + k]), a.lat_mean[t * Z + k]);
    } else {
      for (int k = 0; k < Z; ++k) acc += a.in_w[c * Z + k] * zr[k];
    }
    if (sid >= 0) acc += a.suite_embed[static_cast<long long>(sid) * h + c];
    x[(static_cast<long long>(b) * h + c) * T + t] = acc;
  }
}

struct DecConvArgs {
  const float* in;       // [B, h, Lin]
  float* out;            // [B, h, Lout]
  const float* resid;    // [B, h, Lout] or null (add after GN)
  const float* w;        // convT: [h, h, 2s]; conv3: [h, h, 3]
  const float* bias;
  const float* gn_w;
  const float* gn_b;
  int h, Lin, Lout, stride, transposed, silu;
};

__global__ void __launch_bounds__(kDecThreads) dec_conv_kernel(const DecConvArgs a) {
  __shared__ float vals[kDecMaxGroupElems];
  __shared__ float red[33];
  const int b = blockIdx.x, g = blockIdx.y, G = gridDim.y;
  const int cg = a.h / G;
  const int n = cg * a.Lout;
  const float* in = a.in + static_cast<long long>(b) * a.h * a.Lin;
  const int K = a.transposed ? 2 * a.stride : 3;
  const int pad = a.transposed ? a.stride / 2 : 1;
  float lsum = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int co = g * cg + i / a.Lout, p = i % a.Lout;
    float acc = a.bias[co];
    if (a.transposed) {
      // out[co][p] += w[ci][co][k] * in[ci][j] where p = j*s - pad + k
      for (int k = 0; k < K; ++k) {
        const int num = p + pad - k;
        if (num < 0 || num % a.stride != 0) continue;
        const int j = num / a.stride;
        if (j >= a.Lin) continue;
        const float* wk = a.w + static_cast<long long>(co) * K + k;  // ci stride h*K
        for (int ci = 0; ci < a.h; ++ci) acc += wk[static_cast<long long>(ci) * a.h * K] * in[ci * a.Lin + j];
      }
    } else {
      const float* wr = a.w + static_cast<long long>(co) * a.h * K;
      for (int ci = 0; ci < a.h; ++ci) {
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          const int j = p + k - pad;
          if (j >= 0 && j < a.Lin) acc += wr[ci * K + k] * in[ci * a.Lin + j];
        }
      }
    }
    vals[i] = acc;
    lsum += acc;
  }
  // GroupNorm over the group's channels x positions
  float v = warp_sum(lsum);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (blockDim.x >> 5); ++i) t += red[i];
    red[32] = t;
  }
  __syncthreads();
  const float mean = red[32] / n;
  float lvar = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float d = vals[i] - mean;
    lvar += d * d;
  }
  v = warp_sum(lvar);
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (blockDim.x >> 5); ++i) t += red[i];
    red[32] = t;
  }
  __syncthreads();
  const float rstd = rsqrtf(red[32] / n + 1e-5f);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int co = g * cg + i / a.Lout, p = i % a.Lout;
    float y = (vals[i] - mean) * rstd * a.gn_w[co] + a.gn_b[co];
    const long long o = (static_cast<long long>(b) * a.h + co) * a.Lout + p;
    if (a.silu) y = silu(y);
    if (a.resid != nullptr) y += a.resid[o];
    a.out[o] = y;
  }
}

__global__ void dec_output_kernel(const __grid_constant__ DecArgs a, const float* x, int Lfinal) {
  const int b = blockIdx.x;
  const int h = a.cfg.hidden, Hz = a.cfg.action_horizon, A = a.cfg.action_dim;
  for (int i = threadIdx.x; i < Hz * A; i += blockDim.x) {
    const int p = i / A, c = i % A;
    float acc = a.out_b[c];
    if (p < Lfinal)
      for (int k = 0; k < h; ++k) acc += a.out_w[c * h + k] * x[(static_cast<long long>(b) * h + k) * Lfinal + p];
    a.out[(static_cast<long long>(b) * Hz + p) * A + c] = acc;
  }
}


// ------------------------------------------------------------------ wide path
constexpr int kDlThreads = 256;
constexpr int kDlCo = 4;  // output channels per CTA

struct DecLayerArgs {
  int in_mode;            // 0: input_proj(z) (+ suite); 1: SiLU(GN(src)); 2: resid + GN(src)
  const float* src;       // raw conv output [B, h, Lin] (modes 1, 2)
  const float* resid;     // [B, h, Lin] (mode 2)
  const float *gn_w, *gn_b;
  float* xsave;           // mode 1: the built input of this CTA's channels (the block's skip), or null
  const float *z, *in_w, *in_b, *suite_embed;
  const float *lat_std, *lat_mean;  // [Lin, Z] or null: z * std + mean is decoded
  const int32_t* suite_ids;
  int Z;
  const float *w, *bias;  // convT: [h, h, 2s]; conv3: [h, h, 3]
  int transposed, stride;
  float* out;             // raw [B, h, Lout]
  int h, G, Lin, Lout;
  // head only
  const float *out_w, *out_b;
  float* final_out;       // [B, horizon, A]
  int horizon, A;
};

__device__ __forceinline__ void dl_cp4(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Build the layer input x[h][Lin] in shared memory (see DecLayerArgs::in_mode).
// Ends with a barrier.
__device__ void dl_build_input(const DecLayerArgs& a, float* x, float* stat) {
  const int b = blockIdx.y, h = a.h, Lin = a.Lin, n = h * Lin;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (a.in_mode == 0) {
    // input_proj: the token rows of z first (shared), then one output per thread;
    // the weight row of each output is read with independent loads
    float* zs = stat + 16;  // [Lin][Z] (the stat area is followed by room for it)
    for (int i = threadIdx.x; i < Lin * a.Z; i += kDlThreads) {
      const float zv = a.z[static_cast<long long>(b) * Lin * a.Z + i];
      zs[i] = a.lat_std != nullptr ? __fadd_rn(__fmul_rn(zv, a.lat_std[i]), a.lat_mean[i]) : zv;
    }
    __syncthreads();
    const int sid = (a.suite_ids != nullptr && a.suite_embed != nullptr) ? a.suite_ids[b] : -1;
    for (int i = threadIdx.x; i < n; i += kDlThreads) {
      const int c = i / Lin, t = i - c * Lin;
      float acc = a.in_b[c];
      const float* zr = zs + t * a.Z;
      const float* wr = a.in_w + static_cast<long long>(c) * a.Z;
#pragma unroll 8
      for (int k = 0; k < a.Z; ++k) acc += __ldg(wr + k) * zr[k];
      if (sid >= 0) acc += a.suite_embed[static_cast<long long>(sid) * h + c];
      x[i] = acc;
    }
    __syncthreads();
    return;
  }
  const float* src = a.src + static_cast<long long>(b) * n;
  const float* res = a.in_mode == 2 ? a.resid + static_cast<long long>(b) * n : nullptr;
  // n % 4 == 0 (h % 4 == 0): independent float4 loads, all in flight at once
#pragma unroll 8
  for (int i = threadIdx.x * 4; i < n; i += kDlThreads * 4)
    *reinterpret_cast<float4*>(x + i) = __ldg(reinterpret_cast<const float4*>(src + i));
  __syncthreads();
  // GroupNorm statistics: warp per group, two passes over shared memory
  const int gsz = (h / a.G) * Lin;
  for (int g = warp; g < a.G; g += kDlThreads / 32) {
    const float* xg = x + g * gsz;
    float s = 0.f;
    for (int i = lane; i < gsz; i += 32) s += xg[i];
    const float mean = warp_sum(s) / gsz;
    float v = 0.f;
    for (int i = lane; i < gsz; i += 32) {
      const float d = xg[i] - mean;
      v += d * d;
    }
    v = warp_sum(v) / gsz;
    if (lane == 0) {
      stat[2 * g] = mean;
      stat[2 * g + 1] = rsqrtf(v + 1e-5f);
    }
  }
  __syncthreads();
  const int cg = h / a.G;
#pragma unroll 4
  for (int i = threadIdx.x * 4; i < n; i += kDlThreads * 4) {
    const int c = i / Lin, g = c / cg;  // Lin % 4 == 0: the four values share a channel
    const float m = stat[2 * g], r = stat[2 * g + 1], w = a.gn_w[c], bb = a.gn_b[c];
    float4 y = *reinterpret_cast<const float4*>(x + i);
    y = make_float4((y.x - m) * r * w + bb, (y.y - m) * r * w + bb, (y.z - m) * r * w + bb, (y.w - m) * r * w + bb);
    if (a.in_mode == 1) {
      y = make_float4(silu(y.x), silu(y.y), silu(y.z), silu(y.w));
    } else {
      const float4 q = __ldg(reinterpret_cast<const float4*>(res + i));
      y = make_float4(y.x + q.x, y.y + q.y, y.z + q.z, y.w + q.w);
    }
    *reinterpret_cast<float4*>(x + i) = y;
  }
  __syncthreads();
  if (a.xsave != nullptr) {
    const int co0 = blockIdx.x * kDlCo;
    float* dst = a.xsave + static_cast<long long>(b) * n;
    for (int i = threadIdx.x; i < kDlCo * Lin; i += kDlThreads) dst[co0 * Lin + i] = x[co0 * Lin + i];
  }
}

// dynamic smem: x[h * Lin] | w[kDlCo][h][K] | part[kDlThreads] | stat[16] | z rows
__global__ void __launch_bounds__(kDlThreads) dec_layer_kernel(const __grid_constant__ DecLayerArgs a) {
  extern __shared__ __align__(16) float dsm[];
  const int h = a.h, Lin = a.Lin, Lout = a.Lout;
  const int K = a.transposed ? 2 * a.stride : 3;
  const int pad = a.transposed ? a.stride / 2 : 1;
  float* x = dsm;
  float* w = x + ((h * Lin + 3) & ~3);
  float* part = w + kDlCo * h * K;
  float* stat = part + kDlThreads;
  const int co0 = blockIdx.x * kDlCo;
  // weight slice -> w[co_l][ci][k] (weights are never written by a launch):
  // 16-byte copies when the runs are aligned (Conv1d: one run of h*3 per output
  // channel; ConvTranspose1d: a run of K per (input, output channel))
  const bool al16 = (reinterpret_cast<uintptr_t>(a.w) & 15) == 0;
  if (al16 && !a.transposed && (h * K) % 4 == 0) {
    const int per = h * K / 4;
    for (int i = threadIdx.x; i < kDlCo * per; i += kDlThreads) {
      const int col = i / per, r = i - col * per;
      cp_async16(w + col * h * K + 4 * r, a.w + (static_cast<long long>(co0 + col) * h) * K + 4 * r, true);
    }
  } else if (al16 && a.transposed && K % 4 == 0) {
    const int per = K / 4;
    for (int i = threadIdx.x; i < kDlCo * h * per; i += kDlThreads) {
      const int q = i % per, cc = i / per, col = cc % kDlCo, ci = cc / kDlCo;
      cp_async16(w + (col * h + ci) * K + 4 * q, a.w + (static_cast<long long>(ci) * h + co0 + col) * K + 4 * q, true);
    }
  } else {
    for (int i = threadIdx.x; i < kDlCo * h * K; i += kDlThreads) {
      const int col = i / (h * K), r = i - col * h * K, ci = r / K, k = r - ci * K;
      const float* src = a.transposed ? a.w + (static_cast<long long>(ci) * h + co0 + col) * K + k
                                      : a.w + (static_cast<long long>(co0 + col) * h + ci) * K + k;
      dl_cp4(w + i, src);
    }
  }
  cp_async_commit();
  pdl_wait();
  pdl_launch_dependents();
  dl_build_input(a, x, stat);
  cp_async_wait<0>();
  __syncthreads();
  // outputs (co_l, p) x input-channel splits
  const int nout = kDlCo * Lout;
  int nsplit = 1;
  while (nsplit * 2 * nout <= kDlThreads && nsplit * 2 <= h) nsplit *= 2;
  const int chunk = (h + nsplit - 1) / nsplit;
  float* outp = a.out + static_cast<long long>(blockIdx.y) * h * Lout;
  for (int base = 0; base < nout; base += kDlThreads / nsplit) {
    const int idx = threadIdx.x;
    const int o = base + idx % (kDlThreads / nsplit), sp = idx / (kDlThreads / nsplit);
    float acc = 0.f;
    if (o < nout) {
      const int col = o / Lout, p = o - col * Lout;
      const int c0 = sp * chunk, c1 = min(h, c0 + chunk);
      const float* wc = w + col * h * K;
      if (a.transposed) {
        // out[p] += w[ci][k] * x[ci][j] where p = j * s - pad + k
        for (int k = 0; k < K; ++k) {
          const int num = p + pad - k;
          if (num < 0 || num % a.stride != 0) continue;
          const int j = num / a.stride;
          if (j >= Lin) continue;
          for (int ci = c0; ci < c1; ++ci) acc = fmaf(wc[ci * K + k], x[ci * Lin + j], acc);
        }
      } else {
        for (int ci = c0; ci < c1; ++ci) {
#pragma unroll
          for (int k = 0; k < 3; ++k) {
            const int j = p + k - pad;
            if (j >= 0 && j < Lin) acc = fmaf(wc[ci * K + k], x[ci * Lin + j], acc);
          }
        }
      }
    }
    part[idx] = acc;
    __syncthreads();
    const int per = kDlThreads / nsplit;
    if (idx < per && base + idx < nout) {
      const int oo = base + idx;
      float s = 0.f;
      for (int q = 0; q < nsplit; ++q) s += part[q * per + idx];
      const int col = oo / Lout, p = oo - col * Lout;
      outp[(co0 + col) * Lout + p] = s + a.bias[co0 + col];
    }
    __syncthreads();
  }
}

// skip + GroupNorm of the last stage, crop / zero-pad to the horizon, output_proj.
// dynamic smem: x[h * Lin] | out_w[A][h] | stat[16] | z rows
__global__ void __launch_bounds__(kDlThreads) dec_head_kernel(const __grid_constant__ DecLayerArgs a) {
  extern __shared__ __align__(16) float dsm[];
  const int h = a.h, Lin = a.Lin, A = a.A, Hz = a.horizon;
  float* x = dsm;
  float* ow = x + ((h * Lin + 3) & ~3);
  float* stat = ow + ((A * h + 3) & ~3);
  for (int i = threadIdx.x; i < A * h; i += kDlThreads) dl_cp4(ow + i, a.out_w + i);
  cp_async_commit();
  pdl_wait();
  pdl_launch_dependents();
  dl_build_input(a, x, stat);
  cp_async_wait<0>();
  __syncthreads();
  const int b = blockIdx.y;
  // warp per output feature, lanes over positions: x[k][p] reads are consecutive
  // across the lanes, the weight row is a broadcast
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = warp; c < A; c += kDlThreads / 32) {
    const float* wr = ow + c * h;
    for (int p = lane; p < Hz; p += 32) {
      float acc = a.out_b[c];
      if (p < Lin) {
#pragma unroll 8
        for (int k = 0; k < h; ++k) acc = fmaf(wr[k], x[k * Lin + p], acc);
      }
      a.final_out[(static_cast<long long>(b) * Hz + p) * A + c] = acc;
    }
  }
}

// stat[16] is followed by kDlZRows floats for the token rows of z (input_proj)
constexpr int kDlZRows = 1024;
static size_t dl_layer_smem(int h, int Lin, int K) {
  return sizeof(float) * (((h * Lin + 3) & ~3) + kDlCo * h * K + kDlThreads + 16 + kDlZRows);
}
static size_t dl_head_smem(int h, int Lin, int A) {
  return sizeof(float) * (((h * Lin + 3) & ~3) + ((A * h + 3) & ~3) + 16 + kDlZRows);
}

template <typename Kern>
static cudaError_t dl_launch(Kern k, dim3 grid, size_t smem, cudaStream_t st, const DecLayerArgs& a) {
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kDlThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, a);
}

static int stage_out_len(int Lin, int s) { return (Lin - 1) * s - 2 * (s / 2) + 2 * s; }

size_t decoder_scratch_floats(const fam_decoder_config& c, const fam_decoder_stage* stages, int n,
                              int B) {
  int L = c.num_tokens, Lmax = L;
  for (int i = 0; i < n; ++i) {
    L = stage_out_len(L, stages[i].stride);
    if (L > Lmax) Lmax = L;
  }
  return static_cast<size_t>(B) * c.hidden * Lmax;
}

// Wide path: 3 launches per stage + the head, each over h / 4 x B CTAs.
static bool decoder_wide(const DecArgs& a, cudaStream_t st, cudaError_t* err) {
  const int h = a.cfg.hidden;
  const int G = h < 8 ? h : 8;
  if (h % kDlCo != 0 || h % G != 0) return false;
  const int kSmemMax = 227 * 1024;
  int L = a.cfg.num_tokens;
  if (L % 4 != 0 || L * a.cfg.latent_dim > kDlZRows) return false;
  for (int i = 0; i < a.num_stages; ++i) {
    const int Lout = stage_out_len(L, a.stages[i].stride);
    if (Lout % 4 != 0) return false;  // float4 rows of one channel
    if (dl_layer_smem(h, L, 2 * a.stages[i].stride) > kSmemMax || dl_layer_smem(h, Lout, 3) > kSmemMax) return false;
    L = Lout;
  }
  if (dl_head_smem(h, L, a.cfg.action_dim) > kSmemMax) return false;
  float* bufs[3] = {a.buf0, a.buf1, a.buf2};
  const dim3 grid(h / kDlCo, a.B);
  DecLayerArgs c;
  memset(&c, 0, sizeof(c));
  c.h = h;
  c.G = G;
  c.z = a.z;
  c.lat_std = a.lat_std;
  c.lat_mean = a.lat_mean;
  c.in_w = a.in_w;
  c.in_b = a.in_b;
  c.suite_embed = a.suite_embed;
  c.suite_ids = a.suite_ids;
  c.Z = a.cfg.latent_dim;
  // buffer roles: r = raw output of the last conv, s = skip of the current block
  int r = -1, s = -1;
  L = a.cfg.num_tokens;
  auto free_buf = [&](int x0, int x1) {
    for (int i = 0; i < 3; ++i)
      if (i != x0 && i != x1) return i;
    return -1;
  };
  for (int i = 0; i < a.num_stages; ++i) {
    const fam_decoder_stage& sg = a.stages[i];
    const int Lout = stage_out_len(L, sg.stride);
    // up: ConvT of (input_proj(z) | skip + GN2(prev conv2))
    const int u = free_buf(r, s);
    c.in_mode = i == 0 ? 0 : 2;
    c.src = i == 0 ? nullptr : bufs[r];
    c.resid = i == 0 ? nullptr : bufs[s];
    if (i > 0) {
      c.gn_w = a.stages[i - 1].gn2_w;
      c.gn_b = a.stages[i - 1].gn2_b;
    }
    c.xsave = nullptr;
    c.w = sg.convt_w;
    c.bias = sg.convt_b;
    c.transposed = 1;
    c.stride = sg.stride;
    c.out = bufs[u];
    c.Lin = L;
    c.Lout = Lout;
    *err = dl_launch(dec_layer_kernel, grid, dl_layer_smem(h, L, 2 * sg.stride), st, c);
    if (*err != cudaSuccess) return true;
    // conv1 of x = SiLU(GN0(u)); x saved as the block's skip
    const int sk = free_buf(u, -1);
    const int t = free_buf(u, sk);
    c.in_mode = 1;
    c.src = bufs[u];
    c.resid = nullptr;
    c.gn_w = sg.gn0_w;
    c.gn_b = sg.gn0_b;
    c.xsave = bufs[sk];
    c.w = sg.c1_w;
    c.bias = sg.c1_b;
    c.transposed = 0;
    c.stride = 1;
    c.out = bufs[t];
    c.Lin = Lout;
    c.Lout = Lout;
    *err = dl_launch(dec_layer_kernel, grid, dl_layer_smem(h, Lout, 3), st, c);
    if (*err != cudaSuccess) return true;
    // conv2 of SiLU(GN1(t))
    c.src = bufs[t];
    c.gn_w = sg.gn1_w;
    c.gn_b = sg.gn1_b;
    c.xsave = nullptr;
    c.w = sg.c2_w;
    c.bias = sg.c2_b;
    c.out = bufs[u];  // the ConvT output is dead
    *err = dl_launch(dec_layer_kernel, grid, dl_layer_smem(h, Lout, 3), st, c);
    if (*err != cudaSuccess) return true;
    r = u;
    s = sk;
    L = Lout;
  }
  // head: skip + GN2 of the last stage (or input_proj(z) when there is none)
  c.in_mode = a.num_stages == 0 ? 0 : 2;
  c.src = a.num_stages == 0 ? nullptr : bufs[r];
  c.resid = a.num_stages == 0 ? nullptr : bufs[s];
  if (a.num_stages > 0) {
    c.gn_w = a.stages[a.num_stages - 1].gn2_w;
    c.gn_b = a.stages[a.num_stages - 1].gn2_b;
  }
  c.xsave = nullptr;
  c.Lin = L;
  c.out_w = a.out_w;
  c.out_b = a.out_b;
  c.final_out = a.out;
  c.horizon = a.cfg.action_horizon;
  c.A = a.cfg.action_dim;
  *err = dl_launch(dec_head_kernel, dim3(1, a.B), dl_head_smem(h, L, c.A), st, c);
  if (*err == cudaSuccess) *err = cudaGetLastError();
  return true;
}

cudaError_t launch_action_decoder(const DecArgs& a, cudaStream_t st) {
  cudaError_t wide_err = cudaSuccess;
  if (decoder_wide(a, st, &wide_err)) return wide_err;
  const int h = a.cfg.hidden;
  const int G = h < 8 ? h : 8;
  if (h % G != 0) return cudaErrorInvalidValue;
  dec_input_kernel<<<a.B, kDecThreads, 0, st>>>(a, a.buf0);
  float* cur = a.buf0;   // stage input / output
  float* t1 = a.buf1;
  float* t2 = a.buf2;
  int L = a.cfg.num_tokens;
  for (int i = 0; i < a.num_stages; ++i) {
    const fam_decoder_stage& s = a.stages[i];
    const int Lout = stage_out_len(L, s.stride);
    if ((h / G) * Lout > kDecMaxGroupElems) return cudaErrorInvalidValue;
    DecConvArgs c = {cur, t1, nullptr, s.convt_w, s.convt_b, s.gn0_w, s.gn0_b, h, L, Lout, s.stride, 1, 1};
    dec_conv_kernel<<<dim3(a.B, G), kDecThreads, 0, st>>>(c);  // up: ConvT -> GN -> SiLU
    DecConvArgs r1 = {t1, t2, nullptr, s.c1_w, s.c1_b, s.gn1_w, s.gn1_b, h, Lout, Lout, 1, 0, 1};
    dec_conv_kernel<<<dim3(a.B, G), kDecThreads, 0, st>>>(r1);  // Conv -> GN -> SiLU
    DecConvArgs r2 = {t2, cur, t1, s.c2_w, s.c2_b, s.gn2_w, s.gn2_b, h, Lout, Lout, 1, 0, 0};
    dec_conv_kernel<<<dim3(a.B, G), kDecThreads, 0, st>>>(r2);  // Conv -> GN, + skip
    L = Lout;
  }
  dec_output_kernel<<<a.B, kDecThreads, 0, st>>>(a, cur, L);
  return cudaGetLastError();
}

}  // namespace fam
