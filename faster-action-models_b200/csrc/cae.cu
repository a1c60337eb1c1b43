// Compact Action Expert (hidden width <= 64): the whole Euler loop in one
// persistent launch.  BASELINE config 0 (hidden 32, 4 heads x 8, 8 blocks,
// 512-token context, 4 Euler steps) is launch-bound: every tensor of a step is
// a few KB, so one CTA per sample keeps the token states in shared memory for
// all steps x blocks and reads the (L2-resident) weights directly; the context
// side is one multi-CTA launch before it.
//
//   cae_context_kernel   text_embedding (Linear -> GELU(tanh) -> Linear) of every
//                        context token and, per block, the cross-attention K
//                        (RMSNorm over H*d) and V.  fp32, CUDA cores; each CTA
//                        owns 4 context tokens.
//   cae_steps_kernel     per sample: for every Euler step the time MLP
//                        (sinusoid -> Linear -> SiLU -> Linear -> SiLU -> Linear
//                        (6D)), action_encoder, every DiT block (AdaLN, q/k/v +
//                        RMSNorm + RoPE, self attention, gated o-proj, norm3 +
//                        cross attention, AdaLN FFN with GELU(tanh), gate), head,
//                        and the Euler update x += v * delta.
//
// Reference (FastWAM/src/fastwam/models/wan22/...): ActionDiT.prepare/forward
// (action_dit.py:312-362), DiTBlock.forward (wan_video_dit.py:248-267),
// sinusoid (:30-34), RMSNorm (:146-157), rope_apply (:54-60), the scheduler
// step (schedulers/scheduler_continuous.py:82-88).  Arithmetic in fp32 like
// the reference's fp32 CAE configuration.
#include "fam_common.cuh"
#include "fam_cae.h"

namespace fam {

constexpr int kCaeThreads = 256;
constexpr int kCaeCtxTokens = 4;  // context tokens per CTA

__device__ __forceinline__ float cae_block_sum(float v, float* red) {
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

// ------------------------------------------------------------- context side
// dynamic smem: kCaeCtxTokens * T floats (context rows) + kCaeCtxTokens * 2D.
__global__ void __launch_bounds__(kCaeThreads) cae_context_kernel(const __grid_constant__ CaeCtxArgs a) {
  extern __shared__ float sm[];
  pdl_wait();
  pdl_launch_dependents();
  const int T = a.T, D = a.D, HD = a.HD;
  float* sctx = sm;                          // [4][T]
  float* se1 = sctx + kCaeCtxTokens * T;     // [4][D] after GELU
  float* se = se1 + kCaeCtxTokens * D;       // [4][D] text embedding
  const int tok0 = blockIdx.x * kCaeCtxTokens;
  const int ntok = min(kCaeCtxTokens, a.rows - tok0);
  for (int i = threadIdx.x; i < ntok * T; i += blockDim.x) {
    const int r = i / T, c = i % T;
    const long long src = static_cast<long long>(tok0 + r) * T + c;
    sctx[i] = a.ctx_f32 != nullptr ? a.ctx_f32[src] : bf2f(a.ctx_bf16[src]);
  }
  __syncthreads();
  // e1 = GELU(W1 ctx + b1): warp w computes outputs o = w, w + 8, ... for all tokens.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int o = warp; o < D; o += nw) {
    const float* wr = a.text0_w + static_cast<long long>(o) * T;
    float acc[kCaeCtxTokens] = {0.f, 0.f, 0.f, 0.f};
    for (int c = lane; c < T; c += 32) {
      const float w = wr[c];
#pragma unroll
      for (int r = 0; r < kCaeCtxTokens; ++r) acc[r] += w * sctx[r * T + c];
    }
#pragma unroll
    for (int r = 0; r < kCaeCtxTokens; ++r) {
      const float s = warp_sum(acc[r]);
      if (lane == 0 && r < ntok) se1[r * D + o] = gelu_tanh(s + a.text0_b[o]);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < ntok * D; i += blockDim.x) {
    const int r = i / D, o = i % D;
    float s = a.text2_b[o];
    for (int c = 0; c < D; ++c) s += a.text2_w[o * D + c] * se1[r * D + c];
    se[r * D + o] = s;
  }
  __syncthreads();
  // per block: k = RMSNorm(Wk e + bk) * nk over HD, v = Wv e + bv
  for (int l = 0; l < a.L; ++l) {
    const CaeLayer& ly = a.layers[l];
    float* kout = a.ctx_k + (static_cast<long long>(l) * a.rows + tok0) * HD;
    float* vout = a.ctx_v + (static_cast<long long>(l) * a.rows + tok0) * HD;
    // one warp per token for the norm (HD <= 64: two values per lane)
    for (int r = warp; r < ntok; r += nw) {
      float kv[2], vv[2];
      float ss = 0.f;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        kv[u] = vv[u] = 0.f;
        if (o < HD) {
          float sk = ly.ckv_b[o], sv = ly.ckv_b[HD + o];
          for (int c = 0; c < D; ++c) {
            const float e = se[r * D + c];
            sk += ly.ckv_w[o * D + c] * e;
            sv += ly.ckv_w[(HD + o) * D + c] * e;
          }
          kv[u] = sk;
          vv[u] = sv;
          ss += sk * sk;
        }
      }
      const float rr = rsqrtf(warp_sum(ss) / HD + a.eps);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        if (o < HD) {
          kout[r * HD + o] = kv[u] * rr * ly.cnorm_k[o];
          vout[r * HD + o] = vv[u];
        }
      }
    }
  }
}

// ----------------------------------------------------------------- step side
struct CaeSmem {
  float x[kCaeMaxS * kCaeMaxD];      // residual stream
  float h[kCaeMaxS * kCaeMaxD];      // normalized operand
  float q[kCaeMaxS * kCaeMaxHD];
  float k[kCaeMaxS * kCaeMaxHD];
  float v[kCaeMaxS * kCaeMaxHD];
  float o[kCaeMaxS * kCaeMaxHD];     // attention output
  float f[kCaeMaxS * kCaeMaxF];      // FFN hidden
  float tm[6 * kCaeMaxD];            // t_mod of the step
  float t1[256];                     // sinusoid / time hidden
  float t2[kCaeMaxD];
  float lat[kCaeMaxS * 64];          // latent tokens (A <= 64)
  float stat[kCaeMaxS * 2];
  float red[33];
};

// y[s][o] = W[o][:] . in[s][:] + b[o] for s < S, o < O (row stride of in = K)
__device__ __forceinline__ void cae_linear(float* y, int ys, const float* in, int is, int S, int K,
                                           const float* W, const float* b, int O) {
  for (int idx = threadIdx.x; idx < S * O; idx += blockDim.x) {
    const int s = idx / O, o = idx % O;
    const float* wr = W + static_cast<long long>(o) * K;
    const float* xr = in + s * is;
    float acc = b != nullptr ? b[o] : 0.f;
    for (int c = 0; c < K; ++c) acc += wr[c] * xr[c];
    y[s * ys + o] = acc;
  }
}

// Per-row LayerNorm statistics (mean, rstd) of x[S][D] into stat.
__device__ __forceinline__ void cae_ln_stats(const float* x, int S, int D, float eps, float* stat) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int s = warp; s < S; s += nw) {
    float sum = 0.f;
    for (int c = lane; c < D; c += 32) sum += x[s * D + c];
    const float mean = warp_sum(sum) / D;
    float var = 0.f;
    for (int c = lane; c < D; c += 32) {
      const float d = x[s * D + c] - mean;
      var += d * d;
    }
    var = warp_sum(var) / D;
    if (lane == 0) {
      stat[2 * s] = mean;
      stat[2 * s + 1] = rsqrtf(var + eps);
    }
  }
}

// Row-wise RMSNorm over the first N columns of y[S][N] times w, in place.
__device__ __forceinline__ void cae_rms_rows(float* y, int S, int N, const float* w, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int s = warp; s < S; s += nw) {
    float ss = 0.f;
    for (int c = lane; c < N; c += 32) ss += y[s * N + c] * y[s * N + c];
    const float r = rsqrtf(warp_sum(ss) / N + eps);
    for (int c = lane; c < N; c += 32) y[s * N + c] = y[s * N + c] * r * w[c];
  }
}

__global__ void __launch_bounds__(kCaeThreads) cae_steps_kernel(const __grid_constant__ CaeStepArgs a) {
  extern __shared__ __align__(16) uint8_t cae_smem[];
  CaeSmem& sm = *reinterpret_cast<CaeSmem*>(cae_smem);
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const int S = a.S, D = a.D, A = a.A, HD = a.HD, hd = a.hd, H = HD / hd, F = a.F, C = a.C;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float* latent = a.latent + static_cast<long long>(b) * S * A;
  for (int i = threadIdx.x; i < S * A; i += blockDim.x) sm.lat[i] = latent[i];
  const float qk_scale = rsqrtf(static_cast<float>(hd));
  const uint8_t* kmask = a.ctx_mask != nullptr ? a.ctx_mask + static_cast<long long>(b) * C : nullptr;
  __syncthreads();

  for (int step = 0; step < a.num_steps; ++step) {
    // ---- time MLP: sinusoid (fp64, cast to fp32) -> Linear -> SiLU -> Linear -> SiLU -> Linear(6D)
    const int half = a.freq_dim / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const double fr = pow(10000.0, -static_cast<double>(i) / static_cast<double>(half));
      const double arg = static_cast<double>(a.timesteps.t[step]) * fr;
      sm.t1[i] = static_cast<float>(cos(arg));
      sm.t1[half + i] = static_cast<float>(sin(arg));
    }
    __syncthreads();
    cae_linear(sm.t2, D, sm.t1, 0, 1, a.freq_dim, a.w.time0_w, a.w.time0_b, D);
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x) sm.t2[i] = silu(sm.t2[i]);
    __syncthreads();
    cae_linear(sm.h, D, sm.t2, 0, 1, D, a.w.time2_w, a.w.time2_b, D);  // t
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x) sm.h[i] = silu(sm.h[i]);
    __syncthreads();
    cae_linear(sm.tm, 6 * D, sm.h, 0, 1, D, a.w.tproj_w, a.w.tproj_b, 6 * D);
    // ---- action_encoder
    cae_linear(sm.x, D, sm.lat, A, S, A, a.w.enc_w, a.w.enc_b, D);
    __syncthreads();

    for (int l = 0; l < a.L; ++l) {
      const CaeLayer& ly = a.w.layers[l];
      // modulation chunks: m[c][f] = modulation[c][f] + t_mod[c][f]
      const float* mw = ly.modulation;
      // AdaLN 1
      cae_ln_stats(sm.x, S, D, a.eps, sm.stat);
      __syncthreads();
      for (int i = threadIdx.x; i < S * D; i += blockDim.x) {
        const int s = i / D, f = i % D;
        const float sh = mw[0 * D + f] + sm.tm[0 * D + f], sc = mw[1 * D + f] + sm.tm[1 * D + f];
        sm.h[i] = (sm.x[i] - sm.stat[2 * s]) * sm.stat[2 * s + 1] * (1.f + sc) + sh;
      }
      __syncthreads();
      // q, k, v
      cae_linear(sm.q, HD, sm.h, D, S, D, ly.qkv_w, ly.qkv_b, HD);
      cae_linear(sm.k, HD, sm.h, D, S, D, ly.qkv_w + HD * D, ly.qkv_b + HD, HD);
      cae_linear(sm.v, HD, sm.h, D, S, D, ly.qkv_w + 2 * HD * D, ly.qkv_b + 2 * HD, HD);
      __syncthreads();
      cae_rms_rows(sm.q, S, HD, ly.norm_q, a.eps);
      cae_rms_rows(sm.k, S, HD, ly.norm_k, a.eps);
      __syncthreads();
      // RoPE on adjacent pairs, positions 0..S-1
      for (int i = threadIdx.x; i < S * (HD / 2); i += blockDim.x) {
        const int s = i / (HD / 2), p = i % (HD / 2);
        const int pi = p % (hd / 2);
        const float c = a.rope[(s * (hd / 2) + pi) * 2], sn = a.rope[(s * (hd / 2) + pi) * 2 + 1];
        float* qq = sm.q + s * HD + 2 * p;
        float* kk = sm.k + s * HD + 2 * p;
        const float q0 = qq[0], q1 = qq[1], k0 = kk[0], k1 = kk[1];
        qq[0] = q0 * c - q1 * sn;
        qq[1] = q0 * sn + q1 * c;
        kk[0] = k0 * c - k1 * sn;
        kk[1] = k0 * sn + k1 * c;
      }
      __syncthreads();
      // self attention (no mask): thread per (head, query)
      for (int i = threadIdx.x; i < H * S; i += blockDim.x) {
        const int hh = i / S, s = i % S;
        const float* qr = sm.q + s * HD + hh * hd;
        float mx = -INFINITY;
        for (int j = 0; j < S; ++j) {
          float dot = 0.f;
          for (int d = 0; d < hd; ++d) dot += qr[d] * sm.k[j * HD + hh * hd + d];
          mx = fmaxf(mx, dot * qk_scale);
        }
        float den = 0.f;
        float acc[kCaeMaxHd];
        for (int d = 0; d < hd; ++d) acc[d] = 0.f;
        for (int j = 0; j < S; ++j) {
          float dot = 0.f;
          for (int d = 0; d < hd; ++d) dot += qr[d] * sm.k[j * HD + hh * hd + d];
          const float p = expf(dot * qk_scale - mx);
          den += p;
          for (int d = 0; d < hd; ++d) acc[d] += p * sm.v[j * HD + hh * hd + d];
        }
        for (int d = 0; d < hd; ++d) sm.o[s * HD + hh * hd + d] = acc[d] / den;
      }
      __syncthreads();
      // x += gate_msa * (Wo o + bo)
      cae_linear(sm.h, D, sm.o, HD, S, HD, ly.o_w, ly.o_b, D);
      __syncthreads();
      for (int i = threadIdx.x; i < S * D; i += blockDim.x) {
        const int f = i % D;
        sm.x[i] += (mw[2 * D + f] + sm.tm[2 * D + f]) * sm.h[i];
      }
      __syncthreads();
      // norm3 (affine) -> cross q -> RMSNorm
      cae_ln_stats(sm.x, S, D, a.eps, sm.stat);
      __syncthreads();
      for (int i = threadIdx.x; i < S * D; i += blockDim.x) {
        const int s = i / D, f = i % D;
        sm.h[i] = (sm.x[i] - sm.stat[2 * s]) * sm.stat[2 * s + 1] * ly.norm3_w[f] + ly.norm3_b[f];
      }
      __syncthreads();
      cae_linear(sm.q, HD, sm.h, D, S, D, ly.cq_w, ly.cq_b, HD);
      __syncthreads();
      cae_rms_rows(sm.q, S, HD, ly.cnorm_q, a.eps);
      __syncthreads();
      // cross attention over the context: one warp per (head, query), lanes over keys
      {
        const float* ck = a.ctx_k + (static_cast<long long>(l) * a.B + b) * C * HD;
        const float* cv = a.ctx_v + (static_cast<long long>(l) * a.B + b) * C * HD;
        for (int pair = warp; pair < H * S; pair += nw) {
          const int hh = pair / S, s = pair % S;
          const float* qr = sm.q + s * HD + hh * hd;
          float mx = -INFINITY;
          for (int j = lane; j < C; j += 32) {
            if (kmask != nullptr && kmask[j] == 0) continue;
            float dot = 0.f;
            for (int d = 0; d < hd; ++d) dot += qr[d] * ck[j * HD + hh * hd + d];
            mx = fmaxf(mx, dot * qk_scale);
          }
          mx = warp_max(mx);
          float den = 0.f;
          float acc[kCaeMaxHd];
          for (int d = 0; d < hd; ++d) acc[d] = 0.f;
          if (mx != -INFINITY) {
            for (int j = lane; j < C; j += 32) {
              if (kmask != nullptr && kmask[j] == 0) continue;
              float dot = 0.f;
              for (int d = 0; d < hd; ++d) dot += qr[d] * ck[j * HD + hh * hd + d];
              const float p = expf(dot * qk_scale - mx);
              den += p;
              for (int d = 0; d < hd; ++d) acc[d] += p * cv[j * HD + hh * hd + d];
            }
          }
          den = warp_sum(den);
          for (int d = 0; d < hd; ++d) {
            const float t = warp_sum(acc[d]);
            if (lane == 0) sm.o[s * HD + hh * hd + d] = den > 0.f ? t / den : 0.f;
          }
        }
      }
      __syncthreads();
      // x += Wco o + bco  (no gate)
      cae_linear(sm.h, D, sm.o, HD, S, HD, ly.co_w, ly.co_b, D);
      __syncthreads();
      for (int i = threadIdx.x; i < S * D; i += blockDim.x) sm.x[i] += sm.h[i];
      __syncthreads();
      // AdaLN 2 + FFN + gate
      cae_ln_stats(sm.x, S, D, a.eps, sm.stat);
      __syncthreads();
      for (int i = threadIdx.x; i < S * D; i += blockDim.x) {
        const int s = i / D, f = i % D;
        const float sh = mw[3 * D + f] + sm.tm[3 * D + f], sc = mw[4 * D + f] + sm.tm[4 * D + f];
        sm.h[i] = (sm.x[i] - sm.stat[2 * s]) * sm.stat[2 * s + 1] * (1.f + sc) + sh;
      }
      __syncthreads();
      cae_linear(sm.f, F, sm.h, D, S, D, ly.ffn0_w, ly.ffn0_b, F);
      __syncthreads();
      for (int i = threadIdx.x; i < S * F; i += blockDim.x) sm.f[i] = gelu_tanh(sm.f[i]);
      __syncthreads();
      cae_linear(sm.h, D, sm.f, F, S, F, ly.ffn2_w, ly.ffn2_b, D);
      __syncthreads();
      for (int i = threadIdx.x; i < S * D; i += blockDim.x) {
        const int f = i % D;
        sm.x[i] += (mw[5 * D + f] + sm.tm[5 * D + f]) * sm.h[i];
      }
      __syncthreads();
    }
    // head + Euler
    cae_linear(sm.h, A, sm.x, D, S, D, a.w.head_w, a.w.head_b, A);
    __syncthreads();
    const float delta = a.deltas.t[step];
    for (int i = threadIdx.x; i < S * A; i += blockDim.x) {
      if (a.trace != nullptr)
        a.trace[(static_cast<long long>(step) * a.B + b) * S * A + i] = sm.h[i];
      sm.lat[i] = sm.lat[i] + sm.h[i] * delta;
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < S * A; i += blockDim.x) latent[i] = sm.lat[i];
}

cudaError_t launch_cae_context(const CaeCtxArgs& a, cudaStream_t st, bool pdl) {
  const size_t smem = sizeof(float) * kCaeCtxTokens * (a.T + 2 * a.D);
  cudaError_t e = cudaFuncSetAttribute(cae_context_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.rows + kCaeCtxTokens - 1) / kCaeCtxTokens);
  cfg.blockDim = dim3(kCaeThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, cae_context_kernel, a);
}

cudaError_t launch_cae_steps(const CaeStepArgs& a, cudaStream_t st, bool pdl) {
  CaeStepArgs staged = a;
  if (cae_staged_plan(a, &staged.plan)) return launch_cae_steps_staged(staged, st, pdl);
  const size_t smem = sizeof(CaeSmem);
  cudaError_t e = cudaFuncSetAttribute(cae_steps_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.B);
  cfg.blockDim = dim3(kCaeThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, cae_steps_kernel, a);
}

size_t cae_smem_bytes() { return sizeof(CaeSmem); }

}  // namespace fam
