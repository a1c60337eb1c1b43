// Compact Action Expert (hidden width <= 64): the context side and the
// unstaged Euler loop.  BASELINE config 0 (hidden 32, 4 heads x 8, 8 blocks,
// 512-token context, 4 Euler steps) is launch- and latency-bound.
//
//   cae_ctx_slice_kernel  text_embedding.0 partial sums: CTA per (16 context
//                         tokens, 1/8 of the text columns), both tiles brought
//                         in by bulk copies; fp32 FMA.
//   cae_ctx_kv_kernel     CTA per (16 context tokens, block): reduce the slices,
//                         GELU(tanh), text_embedding.2, the block's cross K
//                         (RMSNorm over H*d) and V, written [L, rows, H*d]
//                         (rows padded to H*d + 4 / + 8 for the staged step
//                         kernel); also packs the block's weights into the
//                         staged kernel's shared-memory layout.
//   cae_context_kernel    single-kernel context side (4 tokens per CTA) for
//                         shapes the split path does not take.
//   cae_steps_kernel      unstaged Euler loop (one CTA per sample, weights read
//                         from L2) for shapes the staged kernel does not take;
//                         the staged kernel lives in cae_staged.cu.
//
// Reference (FastWAM/src/fastwam/models/wan22/...): ActionDiT.prepare/forward
// (action_dit.py:312-362), DiTBlock.forward (wan_video_dit.py:248-267),
// sinusoid (:30-34), RMSNorm (:146-157), rope_apply (:54-60), the scheduler
// step (schedulers/scheduler_continuous.py:82-88).  Arithmetic in fp32 like
// the reference's fp32 CAE configuration.
#include "fam_common.cuh"
#include "fam_cae.h"

#include <type_traits>

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


// -------------------------------------------------------- split context path
constexpr int kCtxThreads = 256;

__device__ __forceinline__ const float* cae_layer_tensor(const CaeLayer& ly, int t) {
  switch (t) {
    case 0: return ly.modulation;
    case 1: return ly.qkv_w;
    case 2: return ly.qkv_b;
    case 3: return ly.norm_q;
    case 4: return ly.norm_k;
    case 5: return ly.o_w;
    case 6: return ly.o_b;
    case 7: return ly.norm3_w;
    case 8: return ly.norm3_b;
    case 9: return ly.cq_w;
    case 10: return ly.cq_b;
    case 11: return ly.cnorm_q;
    case 12: return ly.co_w;
    case 13: return ly.co_b;
    case 14: return ly.ffn0_w;
    case 15: return ly.ffn0_b;
    case 16: return ly.ffn2_w;
    default: return ly.ffn2_b;
  }
}

__device__ __forceinline__ void ctx_bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float4 ctx_load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ctx_load4(const __nv_bfloat16* p) {
  const uint2 raw = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
  const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
  const float2 a = __bfloat1622float2(lo), b = __bfloat1622float2(hi);
  return make_float4(a.x, a.y, b.x, b.y);
}

// part[ks][row][o] = sum over the slice's columns of text0_w[o][c] * ctx[row][c].
// smem: ctx tile [16][tk] (input type) | W slice [D][tk + 4] fp32
template <typename Tin>
__global__ void __launch_bounds__(kCtxThreads) cae_ctx_slice_kernel(const __grid_constant__ CaeCtxArgs a) {
  extern __shared__ __align__(16) float sm[];
  __shared__ uint64_t bar;
  const int r0 = blockIdx.x * kCaeCtxRows, nr = min(kCaeCtxRows, a.rows - r0);
  const int T = a.T, D = a.D, tk = a.tk, ks = blockIdx.y;
  const int k0 = ks * tk, nk = max(0, min(tk, T - k0));
  Tin* sx = reinterpret_cast<Tin*>(sm);
  float* sw = sm + (kCaeCtxRows * tk * static_cast<int>(sizeof(Tin))) / 4;
  const Tin* src = std::is_same<Tin, float>::value ? reinterpret_cast<const Tin*>(a.ctx_f32)
                                                   : reinterpret_cast<const Tin*>(a.ctx_bf16);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // the context (and the previous call's readers of the workspace)
  pdl_launch_dependents();
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && a.status != nullptr) *a.status = 0;
  if (nk > 0) {
    if (threadIdx.x == 0)
      mbar_arrive_expect_tx(&bar, static_cast<uint32_t>(nr * nk * sizeof(Tin) + D * nk * 4));
    const int t = threadIdx.x;
    if (t < nr)
      ctx_bulk(sx + t * tk, src + static_cast<long long>(r0 + t) * T + k0, static_cast<uint32_t>(nk * sizeof(Tin)),
               &bar);
    else if (t < nr + D)
      ctx_bulk(sw + (t - nr) * (tk + 4), a.text0_w + static_cast<long long>(t - nr) * T + k0,
               static_cast<uint32_t>(nk * 4), &bar);
    mbar_wait(&bar, 0, a.status, 0x4343);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  const float* w0 = sw + lane * (tk + 4);
  const float* w1 = sw + (lane + 32) * (tk + 4);
  const bool has0 = lane < D, has1 = lane + 32 < D;
  for (int c = 0; c < nk; c += 4) {
    const float4 x0 = ctx_load4(sx + warp * tk + c);
    const float4 x1 = ctx_load4(sx + (warp + 8) * tk + c);
    if (has0) {
      const float4 w = ctx_load4(w0 + c);
      acc[0][0] = fmaf(w.x, x0.x, fmaf(w.y, x0.y, fmaf(w.z, x0.z, fmaf(w.w, x0.w, acc[0][0]))));
      acc[1][0] = fmaf(w.x, x1.x, fmaf(w.y, x1.y, fmaf(w.z, x1.z, fmaf(w.w, x1.w, acc[1][0]))));
    }
    if (has1) {
      const float4 w = ctx_load4(w1 + c);
      acc[0][1] = fmaf(w.x, x0.x, fmaf(w.y, x0.y, fmaf(w.z, x0.z, fmaf(w.w, x0.w, acc[0][1]))));
      acc[1][1] = fmaf(w.x, x1.x, fmaf(w.y, x1.y, fmaf(w.z, x1.z, fmaf(w.w, x1.w, acc[1][1]))));
    }
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = warp + 8 * rr;
    if (r >= nr) continue;
    float* dst = a.part + (static_cast<long long>(ks) * a.rows + r0 + r) * D;
    if (has0) dst[lane] = acc[rr][0];
    if (has1) dst[lane + 32] = acc[rr][1];
  }
}

// smem: e1 [16][D] | e [16][D] | ckv weights [2HD][D + 4] | text_embedding.2 weight [D][D + 4]
__global__ void __launch_bounds__(kCtxThreads) cae_ctx_kv_kernel(const __grid_constant__ CaeCtxArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int r0 = blockIdx.x * kCaeCtxRows, nr = min(kCaeCtxRows, a.rows - r0);
  const int l = blockIdx.y, D = a.D, HD = a.HD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* e1 = sm;
  float* e = e1 + kCaeCtxRows * D;
  float* wkv = e + kCaeCtxRows * D;         // [2HD][D + 4]
  float* w2 = wkv + 2 * HD * (D + 4);       // text_embedding.2 weight [D][D + 4]
  const CaeLayer& ly = a.layers[l];
  // constant inputs first (they overlap the slice launch): this block's K/V
  // projection and text_embedding.2 (float4 loads when aligned, all issued
  // before use), and this CTA's share of the packed block weights
  const bool v4 = ((reinterpret_cast<uintptr_t>(ly.ckv_w) | reinterpret_cast<uintptr_t>(a.text2_w)) & 15) == 0;
  if (v4) {
    const int d4 = D / 4;
#pragma unroll 4
    for (int i = threadIdx.x; i < 2 * HD * d4; i += kCtxThreads) {
      const int o = i / d4, c = (i - o * d4) * 4;
      *reinterpret_cast<float4*>(wkv + o * (D + 4) + c) = __ldg(reinterpret_cast<const float4*>(ly.ckv_w) + i);
    }
#pragma unroll 4
    for (int i = threadIdx.x; i < D * d4; i += kCtxThreads) {
      const int o = i / d4, c = (i - o * d4) * 4;
      *reinterpret_cast<float4*>(w2 + o * (D + 4) + c) = __ldg(reinterpret_cast<const float4*>(a.text2_w) + i);
    }
  } else {
    for (int i = threadIdx.x; i < 2 * HD * D; i += kCtxThreads) wkv[(i / D) * (D + 4) + i % D] = ly.ckv_w[i];
    for (int i = threadIdx.x; i < D * D; i += kCtxThreads) w2[(i / D) * (D + 4) + i % D] = a.text2_w[i];
  }
  if (a.wpack != nullptr) {
    const CaeStagePlan& p = a.plan;
    int ntasks = 0;
    for (int t = 0; t < kCaeStagedTensors; ++t) ntasks += p.rows[t];
    float* blk = a.wpack + static_cast<long long>(l) * (p.a_floats + p.f_floats);
    for (int task = blockIdx.x * (kCtxThreads / 32) + warp; task < ntasks; task += gridDim.x * (kCtxThreads / 32)) {
      int t = 0, r = task;
      while (r >= p.rows[t]) {
        r -= p.rows[t];
        ++t;
      }
      const float* src = cae_layer_tensor(ly, t);
      float* dst = blk + (t < kCaeStagedHalfSplit ? 0 : p.a_floats) + p.off[t] + r * p.stride[t];
      const int cols = p.cols[t];
      for (int c = lane; c < cols; c += 32) dst[c] = src != nullptr ? src[static_cast<long long>(r) * cols + c] : 0.f;
    }
  }
  pdl_wait();  // slice partial sums
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < nr * D; i += kCtxThreads) {
    const int r = i / D, o = i - r * D;
    float pv[kCaeCtxSlices];
#pragma unroll
    for (int ks = 0; ks < kCaeCtxSlices; ++ks) pv[ks] = a.part[(static_cast<long long>(ks) * a.rows + r0 + r) * D + o];
    float s = a.text0_b[o];
#pragma unroll
    for (int ks = 0; ks < kCaeCtxSlices; ++ks) s += pv[ks];
    e1[r * D + o] = gelu_tanh(s);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nr * D; i += kCtxThreads) {
    const int r = i / D, o = i - r * D;
    float s = a.text2_b[o];
    const float* wr = w2 + o * (D + 4);
    for (int c = 0; c < D; ++c) s += wr[c] * e1[r * D + c];
    e[r * D + o] = s;
  }
  __syncthreads();
  // K = RMSNorm(Wk e + bk) * norm_k over H*d, V = Wv e + bv: warp per token
  for (int r = warp; r < nr; r += kCtxThreads / 32) {
    float kv[2], vv[2], ss = 0.f;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int o = lane + 32 * u;
      kv[u] = vv[u] = 0.f;
      if (o < HD) {
        float sk = ly.ckv_b[o], sv = ly.ckv_b[HD + o];
        const float* wk = wkv + o * (D + 4);
        const float* wv = wkv + (HD + o) * (D + 4);
        for (int c = 0; c < D; ++c) {
          sk = fmaf(wk[c], e[r * D + c], sk);
          sv = fmaf(wv[c], e[r * D + c], sv);
        }
        kv[u] = sk;
        vv[u] = sv;
        ss += sk * sk;
      }
    }
    const float rr = rsqrtf(warp_sum(ss) / HD + a.eps);
    const int R = r0 + r;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int o = lane + 32 * u;
      if (o >= HD) continue;
      const float kn = kv[u] * rr * ly.cnorm_k[o];
      const long long row = static_cast<long long>(l) * a.rows + R;
      if (a.kv_packed) {  // padded rows: conflict-free tensor-core fragment loads
        a.ctx_k[row * (HD + 4) + o] = kn;
        a.ctx_v[row * (HD + 8) + o] = vv[u];
      } else {
        a.ctx_k[row * HD + o] = kn;
        a.ctx_v[row * HD + o] = vv[u];
      }
    }
  }
}

static size_t ctx_slice_smem(const CaeCtxArgs& a) {
  const size_t esz = a.ctx_bf16 != nullptr ? 2 : 4;
  return kCaeCtxRows * a.tk * esz + static_cast<size_t>(a.D) * (a.tk + 4) * 4;
}

bool cae_ctx_split_setup(CaeCtxArgs* a) {
  a->tk = 0;
  const void* ctx = a->ctx_bf16 != nullptr ? static_cast<const void*>(a->ctx_bf16) : static_cast<const void*>(a->ctx_f32);
  if (a->T % 8 != 0 || a->D % 4 != 0 || a->D > 64 || a->HD > 64) return false;
  if ((reinterpret_cast<uintptr_t>(ctx) & 15) != 0 || (reinterpret_cast<uintptr_t>(a->text0_w) & 15) != 0) return false;
  int tk = (a->T + kCaeCtxSlices - 1) / kCaeCtxSlices;
  tk = (tk + 7) / 8 * 8;
  a->tk = tk;
  if (ctx_slice_smem(*a) > 227 * 1024) {
    a->tk = 0;
    return false;
  }
  return true;
}

template <typename Kern>
static cudaError_t ctx_launch(Kern k, dim3 grid, size_t smem, cudaStream_t st, bool pdl, const CaeCtxArgs& a) {
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kCtxThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, a);
}

cudaError_t launch_cae_context(const CaeCtxArgs& a, cudaStream_t st, bool pdl) {
  if (a.tk > 0) {
    const int tiles = (a.rows + kCaeCtxRows - 1) / kCaeCtxRows;
    cudaError_t e = a.ctx_bf16 != nullptr
                        ? ctx_launch(cae_ctx_slice_kernel<__nv_bfloat16>, dim3(tiles, kCaeCtxSlices), ctx_slice_smem(a), st, pdl, a)
                        : ctx_launch(cae_ctx_slice_kernel<float>, dim3(tiles, kCaeCtxSlices), ctx_slice_smem(a), st, pdl, a);
    if (e != cudaSuccess) return e;
    const size_t smem2 = sizeof(float) * (2 * kCaeCtxRows * a.D + (2 * a.HD + a.D) * (a.D + 4));
    return ctx_launch(cae_ctx_kv_kernel, dim3(tiles, a.L), smem2, st, true, a);
  }
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
  if (a.wpack != nullptr) return launch_cae_steps_staged(a, st, pdl);
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
