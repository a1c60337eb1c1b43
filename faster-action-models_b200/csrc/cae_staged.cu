// Compact Action Expert, staged Euler loop: one CTA of 1024 threads per sample
// runs every Euler step x every DiT block with all operands in shared memory.
//
// The per-block weights (~60 KB fp32 for BASELINE config 0) are staged one block
// ahead with cp.async: the attention half (modulation, qkv, o, norm3, cross q,
// cross o) double buffered, the FFN half (ffn0, ffn2) single buffered and
// reloaded once the previous block's FFN is done.  The block's context K/V
// (written by cae_context_kernel) streams through two buffers one (head, key
// chunk) unit ahead.  Every per-token chain that only needs its own row
// (projection -> residual -> LayerNorm -> next projection, the head, the Euler
// update and the next step's encoder) runs inside one warp per token row, so a
// block costs about ten CTA barriers.  Matrix rows sit in shared memory with a
// stride of K + 4 floats, which makes the lane-per-output float4 reads
// conflict-free.
//
// Reference (FastWAM/src/fastwam/models/wan22/...): ActionDiT.prepare/forward
// (action_dit.py:312-362), DiTBlock.forward (wan_video_dit.py:248-267), the
// sinusoid (:30-34), RMSNorm (:146-157), rope_apply (:54-60), flash-free
// attention (:105-124 semantics: softmax(q k^T / sqrt(d)) v), the scheduler step
// (schedulers/scheduler_continuous.py:82-88).  fp32 arithmetic like the
// reference's fp32 CAE configuration.
#include "fam_cae.h"
#include "fam_common.cuh"
#include "fam_mma.cuh"

namespace fam {

namespace {

constexpr int kCsThreads = 1024;
constexpr int kCsWarps = kCsThreads / 32;
constexpr int kCsMaxTb = 8;       // t_mod rows per time-MLP batch
constexpr int kCsMaxRows = 32;    // token rows (one warp each)
constexpr int kCsSmemLimit = 227 * 1024;

__device__ __forceinline__ void cs_cp4(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Issue the copies of one row-major tensor [rows, cols] (cols % 4 == 0) into
// shared memory with row stride `stride`; a null tensor becomes zeros.
__device__ __forceinline__ void cs_stage(float* dst, const float* src, int rows, int cols, int stride) {
  const int tid = threadIdx.x;
  if (src == nullptr) {
    for (int i = tid; i < rows * cols; i += kCsThreads) dst[(i / cols) * stride + i % cols] = 0.f;
    return;
  }
  if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const int c4 = cols >> 2;
    for (int i = tid; i < rows * c4; i += kCsThreads) {
      const int r = i / c4, c = (i - r * c4) * 4;
      cp_async16(dst + r * stride + c, src + static_cast<long long>(r) * cols + c, true);
    }
  } else {
    for (int i = tid; i < rows * cols; i += kCsThreads) {
      const int r = i / cols, c = i - r * cols;
      cs_cp4(dst + r * stride + c, src + static_cast<long long>(r) * cols + c);
    }
  }
}

__device__ __forceinline__ const float* cs_src(const CaeLayer& ly, int t) {
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

__device__ __forceinline__ void cs_stage_half(float* base, const CaeLayer& ly, const CaeStagePlan& p, int t0,
                                              int t1) {
  for (int t = t0; t < t1; ++t) cs_stage(base + p.off[t], cs_src(ly, t), p.rows[t], p.cols[t], p.stride[t]);
}

// W[0:K] . v[0:K], both 16-byte aligned in shared memory, K % 4 == 0.
__device__ __forceinline__ float cs_dot(const float* w, const float* v, int K) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 4
  for (int c = 0; c < K; c += 4) {
    const float4 x = *reinterpret_cast<const float4*>(w + c);
    const float4 y = *reinterpret_cast<const float4*>(v + c);
    a0 = fmaf(x.x, y.x, a0);
    a1 = fmaf(x.y, y.y, a1);
    a2 = fmaf(x.z, y.z, a2);
    a3 = fmaf(x.w, y.w, a3);
  }
  return (a0 + a1) + (a2 + a3);
}

// Row statistics of a D-wide row held two values per lane (o = lane, lane + 32).
__device__ __forceinline__ void cs_row_stats(const float (&xv)[2], int D, float eps, float& mean, float& rstd) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
#pragma unroll
  for (int u = 0; u < 2; ++u)
    if (lane + 32 * u < D) s += xv[u];
  mean = warp_sum(s) / D;
  float v = 0.f;
#pragma unroll
  for (int u = 0; u < 2; ++u)
    if (lane + 32 * u < D) {
      const float d = xv[u] - mean;
      v += d * d;
    }
  rstd = rsqrtf(warp_sum(v) / D + eps);
}

// AdaLN of a row held in registers: h = LN(x) * (1 + scale) + shift, where
// shift/scale = modulation chunk + t_mod chunk.
__device__ __forceinline__ void cs_adaln_row(const float (&xv)[2], float* hrow, const float* mod, const float* tmr,
                                             int D, float eps, int c_shift, int c_scale) {
  const int lane = threadIdx.x & 31;
  float mean, rstd;
  cs_row_stats(xv, D, eps, mean, rstd);
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int o = lane + 32 * u;
    if (o < D) {
      const float sh = mod[c_shift * D + o] + tmr[c_shift * D + o];
      const float sc = mod[c_scale * D + o] + tmr[c_scale * D + o];
      hrow[o] = (xv[u] - mean) * rstd * (1.f + sc) + sh;
    }
  }
}

struct CsPtrs {
  float *abuf0, *abuf1, *fbuf, *kv0, *kv1, *x, *h, *q, *k, *v, *att, *qc, *f, *part, *tm, *tscr, *lat, *rope, *encw,
      *encb, *headw, *headb;
};

// t_mod rows of steps [step0, step0 + nb): sinusoid (fp64 then fp32) -> Linear ->
// SiLU -> Linear -> SiLU -> Linear(6D).  Block-wide; ends with a barrier.
__device__ void cs_time_batch(const CaeStepArgs& a, const CsPtrs& P, int step0, int nb) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = a.D, fd = a.freq_dim, half = fd / 2;
  float* t1 = P.tscr;                    // [tb][fd]
  float* t2 = t1 + a.plan.tb * fd;       // [tb][D]
  float* t3 = t2 + a.plan.tb * D;        // [tb][D]
  for (int i = threadIdx.x; i < nb * half; i += kCsThreads) {
    const int r = i / half, j = i - r * half;
    const double fr = pow(10000.0, -static_cast<double>(j) / static_cast<double>(half));
    const double arg = static_cast<double>(a.timesteps.t[step0 + r]) * fr;
    t1[r * fd + j] = static_cast<float>(cos(arg));
    t1[r * fd + half + j] = static_cast<float>(sin(arg));
  }
  __syncthreads();
  // warp per output, lanes over the input (coalesced global weight rows)
  auto mlp = [&](const float* W, const float* bias, const float* in, int K, float* out, int O, bool act) {
    for (int o = warp; o < O; o += kCsWarps) {
      const float* wr = W + static_cast<long long>(o) * K;
      float acc[kCsMaxTb];
#pragma unroll
      for (int r = 0; r < kCsMaxTb; ++r) acc[r] = 0.f;
      for (int c = lane; c < K; c += 32) {
        const float w = __ldg(wr + c);
#pragma unroll
        for (int r = 0; r < kCsMaxTb; ++r)
          if (r < nb) acc[r] = fmaf(w, in[r * K + c], acc[r]);
      }
#pragma unroll
      for (int r = 0; r < kCsMaxTb; ++r) {
        if (r >= nb) break;
        const float s = warp_sum(acc[r]) + (bias != nullptr ? __ldg(bias + o) : 0.f);
        if (lane == 0) out[r * O + o] = act ? silu(s) : s;
      }
    }
    __syncthreads();
  };
  mlp(a.w.time0_w, a.w.time0_b, t1, fd, t2, D, true);
  mlp(a.w.time2_w, a.w.time2_b, t2, D, t3, D, true);
  mlp(a.w.tproj_w, a.w.tproj_b, t3, D, P.tm, 6 * D, false);
}

// Cross attention of one (head, key chunk) unit for the warp's query row and key
// slice; running softmax state (m, l, acc) persists across the head's chunks.
template <int HDIM>
__device__ __forceinline__ void cs_cross_unit(const float* kb, const float* vb, int nk, const float (&qv)[HDIM],
                                              const uint8_t* kmask, int wpq, int qw, float scale, float& m, float& l,
                                              float (&acc)[HDIM]) {
  const int lane = threadIdx.x & 31;
  const int per = (nk + wpq - 1) / wpq;
  const int k_lo = qw * per, k_hi = min(nk, k_lo + per);
  for (int j0 = k_lo; j0 < k_hi; j0 += 128) {
    float sc[4];
    float bm = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = j0 + lane + 32 * i;
      sc[i] = -INFINITY;
      if (j < k_hi && (kmask == nullptr || kmask[j] != 0)) {
        const float* kr = kb + j * (HDIM + 4);
        float d = 0.f;
#pragma unroll
        for (int c = 0; c < HDIM; c += 4) {
          const float4 kk = *reinterpret_cast<const float4*>(kr + c);
          d = fmaf(qv[c], kk.x, d);
          d = fmaf(qv[c + 1], kk.y, d);
          d = fmaf(qv[c + 2], kk.z, d);
          d = fmaf(qv[c + 3], kk.w, d);
        }
        sc[i] = d * scale;
        bm = fmaxf(bm, sc[i]);
      }
    }
    bm = warp_max(bm);
    const float mn = fmaxf(m, bm);
    if (mn == -INFINITY) continue;  // every key so far masked (warp-uniform)
    const float alpha = expf(m - mn);
    l *= alpha;
#pragma unroll
    for (int d = 0; d < HDIM; ++d) acc[d] *= alpha;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (sc[i] == -INFINITY) continue;
      const int j = j0 + lane + 32 * i;
      const float pj = expf(sc[i] - mn);
      l += pj;
      const float* vr = vb + j * HDIM;
#pragma unroll
      for (int c = 0; c < HDIM; c += 4) {
        const float4 vv = *reinterpret_cast<const float4*>(vr + c);
        acc[c] = fmaf(pj, vv.x, acc[c]);
        acc[c + 1] = fmaf(pj, vv.y, acc[c + 1]);
        acc[c + 2] = fmaf(pj, vv.z, acc[c + 2]);
        acc[c + 3] = fmaf(pj, vv.w, acc[c + 3]);
      }
    }
    m = mn;
  }
}

// Issue the K/V copies of unit u of block l (head u / uph, key chunk u % uph).
__device__ __forceinline__ void cs_stage_kv(const CaeStepArgs& a, float* buf, int l, int u) {
  const CaeStagePlan& p = a.plan;
  const int hd = a.hd, HD = a.HD;
  const int hh = u / p.units_per_head, ch = u - hh * p.units_per_head;
  const int j0 = ch * p.kc, nk = min(p.kc, a.C - j0);
  const long long row0 = (static_cast<long long>(l) * a.B + blockIdx.x) * a.C + j0;
  const float* ck = a.ctx_k + row0 * HD + hh * hd;
  const float* cv = a.ctx_v + row0 * HD + hh * hd;
  float* kb = buf;
  float* vb = buf + p.kc * (hd + 4);
  const int c4 = hd >> 2;
  for (int i = threadIdx.x; i < nk * c4; i += kCsThreads) {
    const int r = i / c4, c = (i - r * c4) * 4;
    cp_async16(kb + r * (hd + 4) + c, ck + static_cast<long long>(r) * HD + c, true);
    cp_async16(vb + r * hd + c, cv + static_cast<long long>(r) * HD + c, true);
  }
}

template <int HDIM>
__global__ void __launch_bounds__(kCsThreads, 1) cae_steps_staged_kernel(const __grid_constant__ CaeStepArgs a) {
  extern __shared__ __align__(16) float csm[];
  const CaeStagePlan& p = a.plan;
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.S, D = a.D, A = a.A, HD = a.HD, H = HD / HDIM, F = a.F, L = a.L, N = a.num_steps;
  const int hdp = p.hdp;
  CsPtrs P;
  P.abuf0 = csm + p.o_abuf;
  P.abuf1 = P.abuf0 + p.a_floats;
  P.fbuf = csm + p.o_fbuf;
  P.kv0 = csm + p.o_kv;
  P.kv1 = P.kv0 + p.kv_floats;
  P.x = csm + p.o_x;
  P.h = csm + p.o_h;
  P.q = csm + p.o_q;
  P.k = csm + p.o_k;
  P.v = csm + p.o_v;
  P.att = csm + p.o_att;
  P.qc = csm + p.o_qc;
  P.f = csm + p.o_f;
  P.part = csm + p.o_part;
  P.tm = csm + p.o_tm;
  P.tscr = csm + p.o_tscr;
  P.lat = csm + p.o_lat;
  P.rope = csm + p.o_rope;
  P.encw = csm + p.o_encw;
  P.encb = csm + p.o_encb;
  P.headw = csm + p.o_headw;
  P.headb = csm + p.o_headb;
  const float scale = rsqrtf(static_cast<float>(HDIM));
  const uint8_t* kmask = a.ctx_mask != nullptr ? a.ctx_mask + static_cast<long long>(b) * a.C : nullptr;
  float* latent = a.latent + static_cast<long long>(b) * S * A;

  // ---- prologue: constant tensors, block 0 weights, the latent; first t_mod batch
  cs_stage(P.encw, a.w.enc_w, D, A, A + 4);
  cs_stage(P.encb, a.w.enc_b, 1, D, D);
  cs_stage(P.headw, a.w.head_w, A, D, D + 4);
  cs_stage(P.headb, a.w.head_b, 1, A, A);
  cs_stage(P.rope, a.rope, 1, S * HDIM, S * HDIM);
  cs_stage(P.lat, latent, 1, S * A, S * A);
  cs_stage_half(P.abuf0, a.w.layers[0], p, 0, kCaeStagedHalfSplit);
  cs_stage_half(P.fbuf, a.w.layers[0], p, kCaeStagedHalfSplit, kCaeStagedTensors);
  cp_async_commit();
  cs_time_batch(a, P, 0, min(p.tb, N));
  pdl_wait();  // the context K/V come from the preceding launch
  pdl_launch_dependents();
  cp_async_wait<0>();
  __syncthreads();

  // standalone block-0 AdaLN of a step: encoder from the latent, then AdaLN 1
  auto step_entry_row = [&](int s, int step, const float* abuf) {
    const float* tmr = P.tm + (step % p.tb) * 6 * D;
    float xv[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int o = lane + 32 * u;
      xv[u] = 0.f;
      if (o < D) {
        xv[u] = P.encb[o] + cs_dot(P.encw + o * (A + 4), P.lat + s * A, A);
        P.x[s * D + o] = xv[u];
      }
    }
    cs_adaln_row(xv, P.h + s * D, abuf + p.off[0], tmr, D, a.eps, 0, 1);
  };
  for (int s = warp; s < S; s += kCsWarps) step_entry_row(s, 0, P.abuf0);

  const int uph = p.units_per_head, U = H * uph;
  const int total = N * L;
  for (int e = 0; e < total; ++e) {
    const int step = e / L, l = e - step * L;
    const CaeLayer& ly = a.w.layers[l];
    float* ab = (e & 1) ? P.abuf1 : P.abuf0;
    const float* mod = ab + p.off[0];
    const float* tmr = P.tm + (step % p.tb) * 6 * D;
    __syncthreads();  // AdaLN-1 rows of this block written; previous block's FFN done
    // prefetch: K/V unit 0 of this block, then the next block's attention half
    // and this block's FFN half (block 0's FFN half came with the prologue)
    cs_stage_kv(a, P.kv0, l, 0);
    cp_async_commit();
    if (e + 1 < total) {
      const int ln = (e + 1) % L;
      cs_stage_half((e & 1) ? P.abuf0 : P.abuf1, a.w.layers[ln], p, 0, kCaeStagedHalfSplit);
    }
    if (e > 0) cs_stage_half(P.fbuf, ly, p, kCaeStagedHalfSplit, kCaeStagedTensors);
    cp_async_commit();

    // ---- q, k, v (+ RMSNorm over H*d, RoPE on q and k): warp per (row, part)
    for (int item = warp; item < 3 * S; item += kCsWarps) {
      const int s = item / 3, part = item - 3 * s;
      const float* w = ab + p.off[1] + part * HD * (D + 4);
      const float* bias = ab + p.off[2] + part * HD;
      float y[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        y[u] = o < HD ? bias[o] + cs_dot(w + o * (D + 4), P.h + s * D, D) : 0.f;
      }
      float* dst = part == 0 ? P.q : (part == 1 ? P.k : P.v);
      if (part < 2) {
        const float* nw = ab + p.off[part == 0 ? 3 : 4];
        const float r = rsqrtf(warp_sum(y[0] * y[0] + y[1] * y[1]) / HD + a.eps);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int o = lane + 32 * u;
          const float yn = o < HD ? y[u] * r * nw[o] : 0.f;
          const float other = __shfl_xor_sync(0xffffffffu, yn, 1);
          if (o < HD) {
            const int pi = (o % HDIM) >> 1;
            const float c = P.rope[(s * (HDIM / 2) + pi) * 2], sn = P.rope[(s * (HDIM / 2) + pi) * 2 + 1];
            dst[s * hdp + o] = (o & 1) == 0 ? yn * c - other * sn : other * sn + yn * c;
          }
        }
      } else {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int o = lane + 32 * u;
          if (o < HD) dst[s * hdp + o] = y[u];
        }
      }
    }
    __syncthreads();

    // ---- self attention over the S action tokens: warp per (row, head), lanes over keys
    for (int item = warp; item < S * H; item += kCsWarps) {
      const int s = item / H, hh = item - s * H;
      float sc = -INFINITY;
      if (lane < S) {
        const float* qr = P.q + s * hdp + hh * HDIM;
        const float* kr = P.k + lane * hdp + hh * HDIM;
        float d = 0.f;
#pragma unroll
        for (int c = 0; c < HDIM; c += 4) {
          const float4 qq = *reinterpret_cast<const float4*>(qr + c);
          const float4 kk = *reinterpret_cast<const float4*>(kr + c);
          d = fmaf(qq.x, kk.x, d);
          d = fmaf(qq.y, kk.y, d);
          d = fmaf(qq.z, kk.z, d);
          d = fmaf(qq.w, kk.w, d);
        }
        sc = d * scale;
      }
      const float mx = warp_max(sc);
      const float pj = lane < S ? expf(sc - mx) : 0.f;
      const float den = warp_sum(pj);
      float acc = 0.f;
      const int d = lane % HDIM;
      for (int j = 0; j < S; ++j) {
        const float pp = __shfl_sync(0xffffffffu, pj, j);
        acc = fmaf(pp, P.v[j * hdp + hh * HDIM + d], acc);
      }
      if (lane < HDIM) P.att[s * hdp + hh * HDIM + lane] = acc / den;
    }
    __syncthreads();

    // ---- row chain: x += gate_msa * o_proj(attn); h = norm3(x); qc = RMSNorm(cross_q(h))
    for (int s = warp; s < S; s += kCsWarps) {
      const float* ow = ab + p.off[5];
      const float* ob = ab + p.off[6];
      float xv[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        xv[u] = 0.f;
        if (o < D) {
          const float y = ob[o] + cs_dot(ow + o * (HD + 4), P.att + s * hdp, HD);
          xv[u] = P.x[s * D + o] + (mod[2 * D + o] + tmr[2 * D + o]) * y;
          P.x[s * D + o] = xv[u];
        }
      }
      float mean, rstd;
      cs_row_stats(xv, D, a.eps, mean, rstd);
      const float* n3w = ab + p.off[7];
      const float* n3b = ab + p.off[8];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        if (o < D) P.h[s * D + o] = (xv[u] - mean) * rstd * n3w[o] + n3b[o];
      }
      __syncwarp();
      const float* cw = ab + p.off[9];
      const float* cb = ab + p.off[10];
      const float* cn = ab + p.off[11];
      float y[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        y[u] = o < HD ? cb[o] + cs_dot(cw + o * (D + 4), P.h + s * D, D) : 0.f;
      }
      const float r = rsqrtf(warp_sum(y[0] * y[0] + y[1] * y[1]) / HD + a.eps);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        if (o < HD) P.qc[s * hdp + o] = y[u] * r * cn[o];
      }
    }

    // ---- cross attention: (head, key chunk) units stream through two buffers
    {
      const int s = warp / p.wpq, qw = warp - s * p.wpq;
      const bool active = s < S;
      float m = -INFINITY, lsum = 0.f;
      float acc[HDIM];
      float qv[HDIM];
#pragma unroll
      for (int d = 0; d < HDIM; ++d) acc[d] = qv[d] = 0.f;
      for (int u = 0; u < U; ++u) {
        if (u == 0)
          cp_async_wait<1>();
        else
          cp_async_wait<0>();
        __syncthreads();
        if (u + 1 < U) cs_stage_kv(a, ((u + 1) & 1) ? P.kv1 : P.kv0, l, u + 1);
        cp_async_commit();
        const int hh = u / uph, ch = u - hh * uph;
        if (!active) continue;
        if (ch == 0) {
          m = -INFINITY;
          lsum = 0.f;
#pragma unroll
          for (int d = 0; d < HDIM; ++d) {
            acc[d] = 0.f;
            qv[d] = P.qc[s * hdp + hh * HDIM + d];
          }
        }
        const float* buf = (u & 1) ? P.kv1 : P.kv0;
        const int j0 = ch * p.kc, nk = min(p.kc, a.C - j0);
        cs_cross_unit<HDIM>(buf, buf + p.kc * (HDIM + 4), nk, qv, kmask != nullptr ? kmask + j0 : nullptr, p.wpq,
                            qw, scale, m, lsum, acc);
        if (ch == uph - 1) {
          const float lt = warp_sum(lsum);
#pragma unroll
          for (int d = 0; d < HDIM; ++d) acc[d] = warp_sum(acc[d]);
          if (lane == 0) {
            float* pp = P.part + ((s * H + hh) * p.wpq + qw) * (HDIM + 2);
            pp[0] = m;
            pp[1] = lt;
#pragma unroll
            for (int d = 0; d < HDIM; ++d) pp[2 + d] = acc[d];
          }
        }
      }
    }
    __syncthreads();

    // ---- row chain: merge the key slices; x += cross_o(attn); h = AdaLN 2(x)
    for (int s = warp; s < S; s += kCsWarps) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        if (o < HD) {
          const int hh = o / HDIM, d = o - hh * HDIM;
          const float* pp = P.part + (s * H + hh) * p.wpq * (HDIM + 2);
          float mx = -INFINITY;
          for (int q = 0; q < p.wpq; ++q) mx = fmaxf(mx, pp[q * (HDIM + 2)]);
          float num = 0.f, den = 0.f;
          if (mx != -INFINITY) {
            for (int q = 0; q < p.wpq; ++q) {
              const float mq = pp[q * (HDIM + 2)];
              if (mq == -INFINITY) continue;
              const float f = expf(mq - mx);
              den = fmaf(f, pp[q * (HDIM + 2) + 1], den);
              num = fmaf(f, pp[q * (HDIM + 2) + 2 + d], num);
            }
          }
          P.att[s * hdp + o] = den > 0.f ? num / den : 0.f;
        }
      }
      __syncwarp();
      const float* cw = ab + p.off[12];
      const float* cb = ab + p.off[13];
      float xv[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        xv[u] = 0.f;
        if (o < D) {
          xv[u] = P.x[s * D + o] + (cb[o] + cs_dot(cw + o * (HD + 4), P.att + s * hdp, HD));
          P.x[s * D + o] = xv[u];
        }
      }
      cs_adaln_row(xv, P.h + s * D, mod, tmr, D, a.eps, 3, 4);
    }
    cp_async_wait<0>();  // the FFN half of this block and the next block's attention half
    __syncthreads();

    // ---- FFN 0 + GELU(tanh): warp per (row, 32 outputs)
    {
      const int ng = (F + 31) / 32;
      const float* w = P.fbuf + p.off[14];
      const float* bias = P.fbuf + p.off[15];
      for (int item = warp; item < S * ng; item += kCsWarps) {
        const int s = item / ng, o = (item - s * ng) * 32 + lane;
        if (o < F) P.f[s * F + o] = gelu_tanh(bias[o] + cs_dot(w + o * (D + 4), P.h + s * D, D));
      }
    }
    __syncthreads();

    // ---- row chain: x += gate_mlp * ffn2(f); then the next block's AdaLN 1, or
    // (last block) head, Euler update, the next step's encoder and AdaLN 1
    const bool last = l == L - 1;
    const bool more = e + 1 < total;
    const bool new_batch = last && more && ((step + 1) % p.tb) == 0;
    const float* mod_next = (e & 1) ? P.abuf0 + p.off[0] : P.abuf1 + p.off[0];
    for (int s = warp; s < S; s += kCsWarps) {
      const float* w = P.fbuf + p.off[16];
      const float* bias = P.fbuf + p.off[17];
      float xv[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        xv[u] = 0.f;
        if (o < D) {
          const float y = bias[o] + cs_dot(w + o * (F + 4), P.f + s * F, F);
          xv[u] = P.x[s * D + o] + (mod[5 * D + o] + tmr[5 * D + o]) * y;
          P.x[s * D + o] = xv[u];
        }
      }
      if (!last) {
        cs_adaln_row(xv, P.h + s * D, mod_next, tmr, D, a.eps, 0, 1);
        continue;
      }
      __syncwarp();
      const float delta = a.deltas.t[step];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        if (o < A) {
          const float vel = P.headb[o] + cs_dot(P.headw + o * (D + 4), P.x + s * D, D);
          if (a.trace != nullptr) a.trace[(static_cast<long long>(step) * a.B + b) * S * A + s * A + o] = vel;
          const float nl = P.lat[s * A + o] + vel * delta;
          P.lat[s * A + o] = nl;
          if (!more) latent[s * A + o] = nl;
        }
      }
      __syncwarp();
      if (more && !new_batch) step_entry_row(s, step + 1, (e & 1) ? P.abuf0 : P.abuf1);
    }
    if (new_batch) {
      __syncthreads();
      cs_time_batch(a, P, step + 1, min(p.tb, N - step - 1));
      for (int s = warp; s < S; s += kCsWarps) step_entry_row(s, step + 1, (e & 1) ? P.abuf0 : P.abuf1);
    }
  }
}

template <int HDIM>
cudaError_t launch_staged(const CaeStepArgs& a, cudaStream_t st, bool pdl) {
  const size_t smem = static_cast<size_t>(a.plan.total_floats) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(cae_steps_staged_kernel<HDIM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.B);
  cfg.blockDim = dim3(kCsThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, cae_steps_staged_kernel<HDIM>, a);
}

int round4(int v) { return (v + 3) & ~3; }

}  // namespace

bool cae_staged_plan(const CaeStepArgs& a, CaeStagePlan* out) {
  const int S = a.S, D = a.D, A = a.A, HD = a.HD, hd = a.hd, F = a.F, C = a.C;
  if (S < 1 || S > kCsMaxRows || D > 64 || HD > 64 || A > 64 || A < 1 || C < 1) return false;
  if (hd != 4 && hd != 8 && hd != 16) return false;
  if (HD % hd != 0 || D % 4 != 0 || HD % 4 != 0 || F % 4 != 0 || A % 4 != 0 || F < 4) return false;
  if (a.freq_dim < 2 || a.freq_dim % 2 != 0 || a.num_steps < 1 || a.L < 1) return false;
  // RoPE table rows for S positions, the latent rows, and the encoder/head
  // weights are staged with 16-byte copies when aligned, 4-byte otherwise.
  CaeStagePlan p;
  memset(&p, 0, sizeof(p));
  const int H = HD / hd;
  auto tensor = [&](int t, int rows, int cols, int stride, int& cursor) {
    p.off[t] = cursor;
    p.rows[t] = rows;
    p.cols[t] = cols;
    p.stride[t] = stride;
    cursor += round4(rows * stride);
  };
  int ca = 0;
  tensor(0, 1, 6 * D, 6 * D, ca);
  tensor(1, 3 * HD, D, D + 4, ca);
  tensor(2, 1, 3 * HD, 3 * HD, ca);
  tensor(3, 1, HD, HD, ca);
  tensor(4, 1, HD, HD, ca);
  tensor(5, D, HD, HD + 4, ca);
  tensor(6, 1, D, D, ca);
  tensor(7, 1, D, D, ca);
  tensor(8, 1, D, D, ca);
  tensor(9, HD, D, D + 4, ca);
  tensor(10, 1, HD, HD, ca);
  tensor(11, 1, HD, HD, ca);
  tensor(12, D, HD, HD + 4, ca);
  tensor(13, 1, D, D, ca);
  int cf = 0;
  tensor(14, F, D, D + 4, cf);
  tensor(15, 1, F, F, cf);
  tensor(16, D, F, F + 4, cf);
  tensor(17, 1, D, D, cf);
  p.a_floats = ca;
  p.f_floats = cf;
  p.hdp = HD + 4;
  p.wpq = kCsWarps / S;
  p.tb = a.num_steps < kCsMaxTb ? a.num_steps : kCsMaxTb;
  auto layout = [&](int kc) {
    int c = 0;
    auto take = [&](int n) {
      const int o = c;
      c += round4(n);
      return o;
    };
    p.kc = kc;
    p.units_per_head = (C + kc - 1) / kc;
    p.kv_floats = round4(kc * (hd + 4) + kc * hd);
    p.o_abuf = take(2 * p.a_floats);
    p.o_fbuf = take(p.f_floats);
    p.o_kv = take(2 * p.kv_floats);
    p.o_x = take(S * D);
    p.o_h = take(S * D);
    p.o_q = take(S * p.hdp);
    p.o_k = take(S * p.hdp);
    p.o_v = take(S * p.hdp);
    p.o_att = take(S * p.hdp);
    p.o_qc = take(S * p.hdp);
    p.o_f = take(S * F);
    p.o_part = take(S * H * p.wpq * (hd + 2));
    p.o_tm = take(p.tb * 6 * D);
    p.o_tscr = take(p.tb * (a.freq_dim + 2 * D));
    p.o_lat = take(S * A);
    p.o_rope = take(S * hd);
    p.o_encw = take(D * (A + 4));
    p.o_encb = take(D);
    p.o_headw = take(A * (D + 4));
    p.o_headb = take(A);
    p.total_floats = c;
    return static_cast<size_t>(c) * sizeof(float) <= static_cast<size_t>(kCsSmemLimit);
  };
  // context keys per K/V unit: the largest of 512, 256, ..., 32 that fits
  // (the whole context when it is shorter)
  bool ok = false;
  for (int kc0 = 512; kc0 >= 32 && !ok; kc0 >>= 1) ok = layout(kc0 < round4(C) ? kc0 : round4(C));
  if (!ok) return false;
  *out = p;
  return true;
}

cudaError_t launch_cae_steps_staged(const CaeStepArgs& a, cudaStream_t st, bool pdl) {
  switch (a.hd) {
    case 4: return launch_staged<4>(a, st, pdl);
    case 8: return launch_staged<8>(a, st, pdl);
    default: return launch_staged<16>(a, st, pdl);
  }
}

}  // namespace fam
