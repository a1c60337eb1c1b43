// Action-VAE decoder (ActionDecoder.forward,
// FastWAM/src/fastwam/models/action_ae.py:123-166), fp32.
//
//   dec_input_kernel   input_proj (+ suite embedding), channels-first [B, h, T]
//   dec_conv_kernel    one CTA per (sample, GroupNorm group): the group's
//                      output channels of a ConvTranspose1d(k=2s, stride s,
//                      pad s/2) or Conv1d(k=3, pad 1) over all input channels,
//                      then GroupNorm over (group channels x length) in shared
//                      memory, then SiLU or the residual add of the block
//   dec_output_kernel  crop / zero-pad to the horizon + output_proj
//
// GroupNorm(min(8, h), h, eps 1e-5, affine) and the residual block
// [Conv1d -> GN -> SiLU -> Conv1d -> GN] + skip follow action_ae.py:33-47.
#include "fam_common.cuh"
#include "fam_cae.h"

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
    for (int k = 0; k < Z; ++k) acc += a.in_w[c * Z + k] * zr[k];
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

cudaError_t launch_action_decoder(const DecArgs& a, cudaStream_t st) {
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
