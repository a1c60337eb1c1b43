// Compact Action Expert, staged Euler loop: one CTA of 1024 threads per sample
// runs every Euler step x every DiT block with all operands in shared memory.
//
// Weights: the context launch packs every block's tensors into one global blob
// in exactly the shared-memory layout (matrix rows padded to K + 4 floats, so
// the lane-per-output float4 reads are conflict-free).  Each block's attention
// half (modulation, qkv, o, norm3, cross q, cross o) is double buffered and
// arrives one block ahead by a single bulk copy; the FFN half (ffn0, ffn2) is
// single buffered and reloaded once the previous block's FFN is done.
// Context K/V ([L, B*C, H*d] with rows padded to H*d + 4 / + 8, also written by
// the context launch) streams through two buffers one key chunk ahead, two bulk
// copies per chunk.  Every copy completes on an mbarrier with a bounded wait.
//
// Per block: warp-per-row chains for everything that only needs its own token
// row (projection -> residual -> LayerNorm -> next projection, the head, the
// Euler update, the next step's encoder).  Cross attention: each warp owns one
// head and 16 keys of every chunk and keeps a running softmax over the chunks;
// scores and P.V run on the tensor cores (mma.sync TF32, split into high and
// low parts for fp32 accuracy); the key slices merge in the next row chain.
//
// Reference (FastWAM/src/fastwam/models/wan22/...): ActionDiT.prepare/forward
// (action_dit.py:312-362), DiTBlock.forward (wan_video_dit.py:248-267), the
// sinusoid (:30-34), RMSNorm (:146-157), rope_apply (:54-60), attention
// softmax(q k^T / sqrt(d)) v, the scheduler step
// (schedulers/scheduler_continuous.py:82-88).  fp32 arithmetic like the
// reference's fp32 CAE configuration.
#include "fam_cae.h"
#include "fam_common.cuh"
#include "fam_mma.cuh"

#include <cstring>

namespace fam {

namespace {

constexpr int kCsThreads = 1024;
constexpr int kCsWarps = kCsThreads / 32;
constexpr int kCsMaxTb = 8;       // t_mod rows per time-MLP batch
constexpr int kCsMaxRows = 16;    // token rows (one 16-row tensor-core tile)
constexpr int kCsSmemLimit = 227 * 1024;
constexpr int kCsErrWait = 0x4341;  // a bulk copy did not complete within the wait limit
constexpr int kCsMaxCluster = 4;    // CTAs per sample sharing the cross-attention key chunks

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

// One bulk copy global -> shared completing on `bar` (16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void cs_bulk(float* dst, const float* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
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

// Shared-memory regions: base + plan offset, evaluated at each use (the plan
// lives in the kernel parameters, so no pointer stays live in registers).
#define CS_SM(name) (csm + a.plan.o_##name)
#define CS_ABUF(e) (csm + a.plan.o_abuf + (((e) & 1) ? a.plan.a_floats : 0))
#define CS_KV(g) (csm + a.plan.o_kv + (((g) & 1) ? a.plan.kv_floats : 0))
#define CS_BAR(i) (reinterpret_cast<uint64_t*>(csm + a.plan.o_bar) + (i))

// t_mod rows of steps [step0, step0 + nb): sinusoid (fp64 then fp32) -> Linear ->
// SiLU -> Linear -> SiLU -> Linear(6D).  Block-wide; ends with a barrier.
__device__ __noinline__ void cs_time_batch(const CaeStepArgs& a, float* csm, int step0, int nb) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = a.D, fd = a.freq_dim, half = fd / 2;
  float* t1 = CS_SM(tscr);               // [tb][fd]
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
      const float bo = bias != nullptr ? __ldg(bias + o) : 0.f;
#pragma unroll
      for (int r = 0; r < kCsMaxTb; ++r) {
        const float s = warp_sum(acc[r]) + bo;
        if (lane == 0 && r < nb) out[r * O + o] = act ? silu(s) : s;
      }
    }
    __syncthreads();
  };
  mlp(a.w.time0_w, a.w.time0_b, t1, fd, t2, D, true);
  mlp(a.w.time2_w, a.w.time2_b, t2, D, t3, D, true);
  mlp(a.w.tproj_w, a.w.tproj_b, t3, D, CS_SM(tm), 6 * D, false);
}

// ------------------------------------------------ tensor-core cross attention
// mma.sync m16n8k8 TF32 with each operand split into a high part (the fp32
// value with its low 13 mantissa bits cleared: exactly a TF32 number) and the
// exact remainder, which the tensor core reads to TF32 precision again:
// a*b ~ al*bh + ah*bl + ah*bh keeps ~21 significant bits, fp32-level accuracy
// for the fp32 reference.  The split is one AND and one subtraction.
__device__ __forceinline__ uint32_t cs_tf32(float x) { return __float_as_uint(x) & 0xffffe000u; }
__device__ __forceinline__ void cs_mma_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cs_mma_3xtf32(float (&c)[4], const float (&a)[4], float b0, float b1) {
  uint32_t ah[4], al[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    ah[i] = cs_tf32(a[i]);
    al[i] = cs_tf32(a[i] - __uint_as_float(ah[i]));
  }
  const uint32_t bh0 = cs_tf32(b0), bh1 = cs_tf32(b1);
  const uint32_t bl0 = cs_tf32(b0 - __uint_as_float(bh0)), bl1 = cs_tf32(b1 - __uint_as_float(bh1));
  cs_mma_tf32(c, al, bh0, bh1);
  cs_mma_tf32(c, ah, bl0, bl1);
  cs_mma_tf32(c, ah, bh0, bh1);
}

// One warp's running softmax over its 16-key slice of every chunk of one head,
// for the 16-row query tile (rows >= S are zero).  Fragment rows: g = lane / 4
// (r0) and g + 8 (r1); score columns 2t, 2t+1 of each 8-key tile (t = lane % 4).
template <int HDIM>
struct CsFlash {
  static constexpr int KS = (HDIM + 7) / 8;  // 8-wide k steps over the head dims / 8-wide dim tiles
  float m0, m1, l0, l1;
  float o[KS][4];
  __device__ __forceinline__ void init() {
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
#pragma unroll
    for (int i = 0; i < KS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  }
  // buf: K [kc][HD + 4] then V [kc][HD + 8]; keys [k0, k0 + 16) of the chunk (nk valid)
  __device__ __forceinline__ void chunk(const float* buf, int kc, int HD, int nk, int k0, int hh, const float* qc,
                                        int hdp, int S, const uint8_t* kmask, float scale) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const float* kb = buf;
    const float* vb = buf + kc * (HD + 4);
    float qa[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int d0 = ks * 8 + t;
      const float* q0 = qc + g * hdp + hh * HDIM;
      const float* q1 = qc + (g + 8) * hdp + hh * HDIM;
      qa[ks][0] = (g < S && d0 < HDIM) ? q0[d0] : 0.f;
      qa[ks][1] = (g + 8 < S && d0 < HDIM) ? q1[d0] : 0.f;
      qa[ks][2] = (g < S && d0 + 4 < HDIM) ? q0[d0 + 4] : 0.f;
      qa[ks][3] = (g + 8 < S && d0 + 4 < HDIM) ? q1[d0 + 4] : 0.f;
    }
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int n0 = k0 + nt * 8;
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
      const float* kr = kb + (n0 + g) * (HD + 4) + hh * HDIM;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int d0 = ks * 8 + t;
        const float b0 = d0 < HDIM ? kr[d0] : 0.f;
        const float b1 = d0 + 4 < HDIM ? kr[d0 + 4] : 0.f;
        cs_mma_3xtf32(sc[nt], qa[ks], b0, b1);
      }
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) {
        const int j = n0 + 2 * t + e2;
        const bool valid = j < nk && (kmask == nullptr || kmask[j] != 0);
        sc[nt][e2] = valid ? sc[nt][e2] * scale : -INFINITY;  // scale includes log2(e): exp2 form
        sc[nt][2 + e2] = valid ? sc[nt][2 + e2] * scale : -INFINITY;
      }
    }
    float mx0 = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
    float mx1 = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float al0 = mn0 == -INFINITY ? 1.f : exp2f(m0 - mn0);
    const float al1 = mn1 == -INFINITY ? 1.f : exp2f(m1 - mn1);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) {
        sc[nt][e2] = sc[nt][e2] == -INFINITY ? 0.f : exp2f(sc[nt][e2] - mn0);
        sc[nt][2 + e2] = sc[nt][2 + e2] == -INFINITY ? 0.f : exp2f(sc[nt][2 + e2] - mn1);
      }
    }
    l0 = l0 * al0 + ((sc[0][0] + sc[0][1]) + (sc[1][0] + sc[1][1]));
    l1 = l1 * al1 + ((sc[0][2] + sc[0][3]) + (sc[1][2] + sc[1][3]));
#pragma unroll
    for (int nd = 0; nd < KS; ++nd) {
      o[nd][0] *= al0;
      o[nd][1] *= al0;
      o[nd][2] *= al1;
      o[nd][3] *= al1;
    }
    m0 = mn0;
    m1 = mn1;
    // P.V: the score fragment of each 8-key tile becomes the A fragment
    const int srcA = (lane & ~3) | (t >> 1), srcB = srcA + 2;
    const bool odd = (t & 1) != 0;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float pa[4];
      {
        const float x0 = __shfl_sync(0xffffffffu, sc[nt][0], srcA), x1 = __shfl_sync(0xffffffffu, sc[nt][1], srcA);
        const float y0 = __shfl_sync(0xffffffffu, sc[nt][0], srcB), y1 = __shfl_sync(0xffffffffu, sc[nt][1], srcB);
        const float z0 = __shfl_sync(0xffffffffu, sc[nt][2], srcA), z1 = __shfl_sync(0xffffffffu, sc[nt][3], srcA);
        const float w0 = __shfl_sync(0xffffffffu, sc[nt][2], srcB), w1 = __shfl_sync(0xffffffffu, sc[nt][3], srcB);
        pa[0] = odd ? x1 : x0;
        pa[2] = odd ? y1 : y0;
        pa[1] = odd ? z1 : z0;
        pa[3] = odd ? w1 : w0;
      }
      const int n0 = k0 + nt * 8;
      const float* vr0 = vb + (n0 + t) * (HD + 8) + hh * HDIM + g;
      const float* vr1 = vr0 + 4 * (HD + 8);
#pragma unroll
      for (int nd = 0; nd < KS; ++nd) {
        const bool dv = nd * 8 + g < HDIM;
        cs_mma_3xtf32(o[nd], pa, dv ? vr0[nd * 8] : 0.f, dv ? vr1[nd * 8] : 0.f);
      }
    }
  }
  // Partial of this warp: rows < S of [m, l, O[HDIM]] with row stride HDIM + 2.
  __device__ __forceinline__ void store(float* part, int S) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    float lt0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
    lt0 += __shfl_xor_sync(0xffffffffu, lt0, 2);
    float lt1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
    lt1 += __shfl_xor_sync(0xffffffffu, lt1, 2);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = g + 8 * half;
      if (r >= S) continue;
      float* pr = part + r * (HDIM + 2);
      if (t == 0) {
        pr[0] = half ? m1 : m0;
        pr[1] = half ? lt1 : lt0;
      }
#pragma unroll
      for (int nd = 0; nd < KS; ++nd)
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2) {
          const int d = nd * 8 + 2 * t + e2;
          if (d < HDIM) pr[2 + d] = o[nd][2 * half + e2];
        }
    }
  }
};

// Bulk-copy issue (one thread) and waits (every thread).
__device__ __forceinline__ void cs_issue_a(const CaeStepArgs& a, float* csm, int e) {
  uint64_t* bar = CS_BAR(e & 1);
  const int blk = a.plan.a_floats + a.plan.f_floats;
  mbar_arrive_expect_tx(bar, a.plan.a_floats * 4);
  cs_bulk(CS_ABUF(e), a.wpack + static_cast<long long>(e % a.L) * blk, a.plan.a_floats * 4, bar);
}
__device__ __forceinline__ void cs_issue_f(const CaeStepArgs& a, float* csm, int e) {
  uint64_t* bar = CS_BAR(2);
  const int blk = a.plan.a_floats + a.plan.f_floats;
  mbar_arrive_expect_tx(bar, a.plan.f_floats * 4);
  cs_bulk(CS_SM(fbuf), a.wpack + static_cast<long long>(e % a.L) * blk + a.plan.a_floats, a.plan.f_floats * 4, bar);
}
// K/V chunk g of this CTA's sequence: block g / ur, its (g % ur)-th chunk, i.e.
// key chunk rank + (g % ur) * nc of the block (chunks are dealt round-robin over
// the nc CTAs of the sample's cluster).
template <int HDIM>
__device__ __forceinline__ void cs_issue_kv(const CaeStepArgs& a, float* csm, int g, int b, int rank, int ur) {
  const int nc = a.plan.nc, kc = a.plan.kc, HD = a.HD;
  const int e = g / ur, i = g - e * ur, l = e % a.L;
  const int u = rank + i * nc;
  const int j0 = u * kc, nk = min(kc, a.C - j0);
  const long long row = (static_cast<long long>(l) * a.B + b) * a.C + j0;
  const uint32_t kbytes = static_cast<uint32_t>(nk * (HD + 4) * 4), vbytes = static_cast<uint32_t>(nk * (HD + 8) * 4);
  uint64_t* bar = CS_BAR(3 + (g & 1));
  float* buf = CS_KV(g);
  mbar_arrive_expect_tx(bar, kbytes + vbytes);
  cs_bulk(buf, a.ctx_k + row * (HD + 4), kbytes, bar);
  cs_bulk(buf + kc * (HD + 4), a.ctx_v + row * (HD + 8), vbytes, bar);
}
__device__ __forceinline__ void cs_wait(const CaeStepArgs& a, float* csm, int i, int parity) {
  mbar_wait(CS_BAR(i), static_cast<uint32_t>(parity), a.status, kCsErrWait);
}

// Block-0 entry of a step for token row s (one warp): encoder from the latent,
// then AdaLN 1 with the attention half `abuf`.
__device__ __forceinline__ void cs_step_entry_row(const CaeStepArgs& a, float* csm, int s, int step,
                                                  const float* abuf, int D, int A) {
  const int lane = threadIdx.x & 31;
  const float* tmr = CS_SM(tm) + (step % a.plan.tb) * 6 * D;
  float xv[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int o = lane + 32 * u;
    xv[u] = 0.f;
    if (o < D) {
      xv[u] = CS_SM(encb)[o] + cs_dot(CS_SM(encw) + o * (A + 4), CS_SM(lat) + s * A, A);
      CS_SM(x)[s * D + o] = xv[u];
    }
  }
  cs_adaln_row(xv, CS_SM(h) + s * D, abuf + a.plan.off[0], tmr, D, a.eps, 0, 1);
}

// FD, FHD, FF, FA, FS: compile-time hidden width, H*d, FFN width, latent width and
// token count of a specialised instance (0 = read from the arguments): with
// constant widths every dot product and row reduction unrolls completely.
// ------------------------------------------------- epilogue: Action-VAE decode
// The sample's final latents [T, Z] (every CTA of the cluster holds them) ->
// the action chunk: input_proj (+ suite embedding), ConvTranspose1d(h, h, 2s,
// s, s/2) -> GroupNorm -> SiLU, residual [Conv1d k3 -> GN -> SiLU -> Conv1d k3
// -> GN] + skip, crop / zero-pad to the horizon, output_proj; fp32 like the
// reference's Action-VAE.  CTA `rank` of the nc-CTA cluster owns the channels
// [rank h / nc, (rank + 1) h / nc) -- whole GroupNorm groups -- and writes each
// stage's activations of its channels into every CTA's copy of the full
// activation (st.shared::cluster), one cluster barrier per exchange.  Weights
// stream from global (L2) through a ring of kDecStages cp.async staging
// buffers, two chunks in flight while the third is used.  Every stage call
// commits one group (empty past the last chunk), so "wait_group 2" always
// means "chunk k has landed".  The decode's buffers end below the step
// kernel's latent rows, which the input projection reads first.
//
// Both convolutions are register-tiled (DecTask): each weight value a lane
// loads serves 16 positions; the input-channel splits are summed in a fixed
// order, so the result does not depend on timing.
constexpr float kDecGnEps = 1e-5f;

// Row strides of the input_proj output h0 [h][ht] and of the stage activations
// xa / xb [h][xs]: the rows of 8 consecutive input channels (the 8 lane phases)
// start in distinct shared-memory banks (ht odd; xs / 4 odd).
__host__ __device__ inline int dec_ht(int T) { return T | 1; }
__host__ __device__ inline int dec_xs(int Lo) { return (((Lo + 4) >> 2) & 1) ? Lo + 4 : Lo + 8; }

__host__ __device__ int dec_layout(const CaeDecode& d, int nc, int* o_xa, int* o_xb, int* o_loc, int* o_w,
                                   int* o_st) {
  const int h = d.hidden, Lo = d.tokens * d.stride, ch = h / nc, xs = dec_xs(Lo);
  int c = (h * dec_ht(d.tokens) + 3) & ~3;  // h0
  *o_xa = c;
  c += h * xs;
  *o_xb = c;
  c += h * xs;
  *o_loc = c;
  c += (ch * Lo + 3) & ~3;
  *o_w = c;
  c += kDecStages * kDecChunk;
  *o_st = c;                        // GroupNorm (mean, rstd) per local group
  c += 16;
  return c;
}

// Copy `n` contiguous floats (n % 4 == 0, both ends 16-byte aligned) into
// shared memory with cp.async, as one commit group.
__device__ __forceinline__ void dec_copy(float* dst, const float* src, int n) {
  for (int i = threadIdx.x * 4; i < n; i += kCsThreads * 4) cp_async16(dst + i, src + i, true);
  cp_async_commit();
}

// GroupNorm statistics of this CTA's groups of loc [ch][Lo] (warp g: group g),
// then y = GN(loc) (* SiLU) written to rows [c0, c0 + ch) of `full` [h][xs] in
// every CTA of the cluster (skip: add skip[c][p] after the norm), 4 positions
// per store.
__device__ void dec_norm_exchange(float* loc, float* full, const float* skip, const float* gw, const float* gb,
                                  int ch, int c0, int Lo, int xs, int cg, bool act, float* st, int nc) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, ng = ch / cg, n = cg * Lo;
  if (warp < ng) {
    const float* v = loc + warp * n;
    float s = 0.f;
    for (int i = lane; i < n; i += 32) s += v[i];
    const float mean = warp_sum(s) / n;
    float q = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float d = v[i] - mean;
      q += d * d;
    }
    const float var = warp_sum(q) / n;
    if (lane == 0) {
      st[2 * warp] = mean;
      st[2 * warp + 1] = rsqrtf(var + kDecGnEps);
    }
  }
  __syncthreads();
  const int me = nc > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  for (int i = threadIdx.x * 4; i < ch * Lo; i += kCsThreads * 4) {
    const int cl = i / Lo, pp = i - cl * Lo, c = c0 + cl, g = cl / cg;  // Lo % 4 == 0: one channel
    const float m = st[2 * g], r = st[2 * g + 1], w = gw[c], bb = gb[c];
    const float4 x = *reinterpret_cast<const float4*>(loc + i);
    float4 y = make_float4((x.x - m) * r * w + bb, (x.y - m) * r * w + bb, (x.z - m) * r * w + bb,
                           (x.w - m) * r * w + bb);
    if (act) y = make_float4(silu(y.x), silu(y.y), silu(y.z), silu(y.w));
    if (skip != nullptr) {
      const float4 k = *reinterpret_cast<const float4*>(skip + c * xs + pp);
      y = make_float4(y.x + k.x, y.y + k.y, y.z + k.z, y.w + k.w);
    }
    float* dst = full + c * xs + pp;
    *reinterpret_cast<float4*>(dst) = y;
    for (int r2 = 0; r2 < nc; ++r2)
      if (r2 != me) st_cluster_v4(cluster_map(dst, r2), y);
  }
  if (nc > 1) cluster_barrier(); else __syncthreads();
}

// A conv task: lane = one output channel, 16 positions; warp w = task t = w mod
// nt (a block of 32 channels x a tile of 16 positions) x input-channel split
// s = w / nt (ns = 32 / nt splits).  Weight loads are then one row per lane
// (128-bit, conflict-free) and activation loads broadcasts; the splits'
// partials meet in `part` and are summed in split order.
struct DecTask {
  int nt, ns, t, s, cl, p0;
};
__device__ __forceinline__ DecTask dec_task(int ch, int Lo) {
  DecTask k;
  const int nb = ch / 32, warp = threadIdx.x >> 5;
  k.nt = nb * (Lo / 16);
  k.ns = kCsWarps / k.nt;
  k.t = warp % k.nt;
  k.s = warp / k.nt;
  k.cl = (k.t % nb) * 32 + (threadIdx.x & 31);
  k.p0 = (k.t / nb) * 16;
  return k;
}

// The splits' partials -> loc [ch][Lo] (+ bias).  part [ns][nt][16][33] (rows of
// 32 lanes padded to 33) is the staging ring, free once the last chunk is used.
__device__ void dec_split_sum(const float (&acc)[16], const DecTask& k, float* part, float* loc, const float* bias,
                              int c0, int ch, int Lo) {
  float* my = part + (k.s * k.nt + k.t) * 16 * 33 + (threadIdx.x & 31);
#pragma unroll
  for (int i = 0; i < 16; ++i) my[i * 33] = acc[i];
  __syncthreads();
  const int nb = ch / 32;
  for (int j = threadIdx.x; j < ch * Lo; j += kCsThreads) {
    const int cl = j / Lo, p = j - cl * Lo, t = (cl >> 5) + (p >> 4) * nb;
    const float* src = part + (t * 16 + (p & 15)) * 33 + (cl & 31);
    float v = 0.f;
    for (int s = 0; s < k.ns; ++s) v += src[s * k.nt * 16 * 33];
    loc[j] = v + bias[c0 + cl];
  }
  __syncthreads();
}

// Row stride of a staged Conv1d chunk [ch][n * 3] (n % 4 == 0): a multiple of 4
// floats whose quarter is odd, so 8 consecutive lanes' rows are conflict-free.
__device__ __forceinline__ int dec_r3(int n) { return ((n * 3 / 4) & 1) ? n * 3 : n * 3 + 4; }

// Conv1d(h, h, 3, padding 1) of the full activation `in` [h][xs] for this CTA's
// output channels -> loc [ch][Lo] (+ bias); weight [h][h][3], staged per chunk
// of cc input channels as [ch][n * 3] rows.  A split takes groups of 4 input
// channels (one lane loads 12 weights as three 128-bit loads).
__device__ void dec_conv3(const float* in, float* loc, float* wbuf, const float* w, const float* bias, int h, int c0,
                          int ch, int Lo, int xs) {
  const DecTask k = dec_task(ch, Lo);
  int cmax = 4;
  while (ch * dec_r3(cmax + 4) <= kDecChunk && cmax + 4 <= h) cmax += 4;
  const int cc = cmax >= 4 * k.ns ? cmax / (4 * k.ns) * (4 * k.ns) : cmax;  // equal groups per split
  const int nchunk = (h + cc - 1) / cc;
  float acc[16] = {};
  auto stage = [&](int kk) {
    if (kk < nchunk) {
      const int ci0 = kk * cc, n = min(cc, h - ci0), r3 = dec_r3(n), l4 = n * 3 / 4;
      float* dst = wbuf + (kk % kDecStages) * kDecChunk;
      for (int i = threadIdx.x; i < ch * l4; i += kCsThreads) {
        const int r = i / l4, c = (i - r * l4) * 4;
        cp_async16(dst + r * r3 + c, w + (static_cast<long long>(c0 + r) * h + ci0) * 3 + c, true);
      }
    }
    cp_async_commit();
  };
  stage(0);
  stage(1);
  for (int kk = 0; kk < nchunk; ++kk) {
    stage(kk + 2);
    cp_async_wait<2>();
    __syncthreads();
    const int ci0 = kk * cc, n = min(cc, h - ci0);
    const float* wr = wbuf + (kk % kDecStages) * kDecChunk + k.cl * dec_r3(n);
    for (int g = k.s; g < n / 4; g += k.ns) {
      float wv[12];
#pragma unroll
      for (int f = 0; f < 3; ++f) {
        const float4 t4 = *reinterpret_cast<const float4*>(wr + g * 12 + 4 * f);
        wv[4 * f] = t4.x;
        wv[4 * f + 1] = t4.y;
        wv[4 * f + 2] = t4.z;
        wv[4 * f + 3] = t4.w;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float* xr = in + (ci0 + 4 * g + c) * xs + k.p0;
        float xv[18];
        xv[0] = k.p0 > 0 ? xr[-1] : 0.f;
#pragma unroll
        for (int f = 0; f < 4; ++f) {
          const float4 t4 = *reinterpret_cast<const float4*>(xr + 4 * f);
          xv[1 + 4 * f] = t4.x;
          xv[2 + 4 * f] = t4.y;
          xv[3 + 4 * f] = t4.z;
          xv[4 + 4 * f] = t4.w;
        }
        xv[17] = k.p0 + 16 < Lo ? xr[16] : 0.f;
        const float w0 = wv[3 * c], w1 = wv[3 * c + 1], w2 = wv[3 * c + 2];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = fmaf(w2, xv[i + 2], fmaf(w1, xv[i + 1], fmaf(w0, xv[i], acc[i])));
      }
    }
    __syncthreads();  // the buffer is refilled three chunks on
  }
  dec_split_sum(acc, k, wbuf, loc, bias, c0, ch, Lo);
}

// Stage ConvTranspose1d chunk kk (input channels [kk cc, kk cc + n)) as rows
// [ci][ch * K] into ring buffer kk mod kDecStages; channel c's taps are K / 4
// 16-byte units at 4-float unit c K / 4 (+ half ^ bit 2 of c when K = 8, so 8
// consecutive lanes' loads are conflict-free).  One commit group, empty past
// the last chunk.
__device__ __forceinline__ int dec_tunit(int c, int half, int K) {
  return K == 8 ? 2 * c + (half ^ ((c >> 2) & 1)) : c * (K / 4) + half;
}
__device__ __forceinline__ int dec_convt_cc(int h, int ch, int K) {
  return kDecChunk / (ch * K) >= h ? h : kDecChunk / (ch * K);
}
__device__ __forceinline__ void dec_convt_stage(float* wbuf, const float* w, int h, int c0, int ch, int K, int kk) {
  const int cc = dec_convt_cc(h, ch, K);
  if (kk * cc < h) {
    const int ci0 = kk * cc, n = min(cc, h - ci0), u = ch * K / 4;
    float* dst = wbuf + (kk % kDecStages) * kDecChunk;
    for (int i = threadIdx.x; i < n * u; i += kCsThreads) {
      const int r = i / u, e = i - r * u, c = e / (K / 4), half = e - c * (K / 4);
      cp_async16(dst + r * ch * K + 4 * dec_tunit(c, half, K),
                 w + (static_cast<long long>(ci0 + r) * h + c0 + c) * K + 4 * half, true);
    }
  }
  cp_async_commit();
}

// ConvTranspose1d(h, h, 2S, S, S/2) of h0 [h][ht] (T positions) for this CTA's
// output channels -> loc [ch][Lo = T S] (+ bias); weight [h][h][2S].  Output p
// takes tap k1 = (p + S/2) mod S at input j1 = (p + S/2) div S and tap k1 + S
// at j1 - 1; a lane's 16 positions start at a multiple of 16 (S divides 16), so
// its taps and input offsets are compile-time constants.  The caller has issued
// the staging of chunks 0 and 1 (dec_convt_stage).
template <int S>
__device__ void dec_convt(const float* h0, float* loc, float* wbuf, const float* w, const float* bias, int h, int c0,
                          int ch, int T, int ht) {
  constexpr int K = 2 * S, pad = S / 2, NJ = 16 / S + 2;  // input positions a lane reads
  const int Lo = T * S, cc = dec_convt_cc(h, ch, K);
  const int nchunk = (h + cc - 1) / cc;
  const DecTask k = dec_task(ch, Lo);
  const int jb = k.p0 / S - 1;  // first input position the lane reads
  float acc[16] = {};
  for (int kk = 0; kk < nchunk; ++kk) {
    dec_convt_stage(wbuf, w, h, c0, ch, K, kk + 2);
    cp_async_wait<2>();
    __syncthreads();
    const int ci0 = kk * cc, n = min(cc, h - ci0);
    const float* wk = wbuf + (kk % kDecStages) * kDecChunk;
    for (int cil = k.s; cil < n; cil += k.ns) {
      const float* hr = h0 + (ci0 + cil) * ht;
      float hv[NJ];
#pragma unroll
      for (int m = 0; m < NJ; ++m) hv[m] = (jb + m >= 0 && jb + m < T) ? hr[jb + m] : 0.f;
      float tv[K];
#pragma unroll
      for (int f = 0; f < K / 4; ++f) {
        const float4 t4 = *reinterpret_cast<const float4*>(wk + cil * ch * K + 4 * dec_tunit(k.cl, f, K));
        tv[4 * f] = t4.x;
        tv[4 * f + 1] = t4.y;
        tv[4 * f + 2] = t4.z;
        tv[4 * f + 3] = t4.w;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int k1 = (pad + i) % S, jo = (pad + i) / S;  // constants after unrolling
        acc[i] = fmaf(tv[k1 + S], hv[jo], fmaf(tv[k1], hv[jo + 1], acc[i]));
      }
    }
    __syncthreads();  // the buffer is refilled three chunks on
  }
  dec_split_sum(acc, k, wbuf, loc, bias, c0, ch, Lo);
}

__device__ void cs_decode_epilogue(const CaeStepArgs& a, float* csm, int b, int nc) {
  const CaeDecode& d = a.dec;
  const int h = d.hidden, T = d.tokens, Z = d.latent, sdn = d.stride, K = 2 * sdn, Lo = T * sdn;
  const int G = h < 8 ? h : 8, cg = h / G, ch = h / nc, ht = dec_ht(T), xs = dec_xs(Lo);
  const int rank = nc > 1 ? static_cast<int>(cluster_ctarank()) : 0, c0 = rank * ch;
  int o_xa, o_xb, o_loc, o_w, o_st;
  dec_layout(d, nc, &o_xa, &o_xb, &o_loc, &o_w, &o_st);
  float* h0 = csm;
  float* xa = csm + o_xa;
  float* xb = csm + o_xb;
  float* loc = csm + o_loc;
  float* wbuf = csm + o_w;
  float* st = csm + o_st;
  const float* lat = CS_SM(lat);  // [T][Z]: the final latents of the sample
  // 1. stage input_proj's weight (buffer 2) and the first two ConvTranspose1d
  //    chunks (buffers 0, 1); the latents (DiT4DiT-un-normalised when statistics
  //    are given) go to loc while they land
  dec_copy(wbuf + 2 * kDecChunk, d.in_w, h * Z);
  dec_convt_stage(wbuf, d.convt_w, h, c0, ch, K, 0);
  dec_convt_stage(wbuf, d.convt_w, h, c0, ch, K, 1);
  for (int i = threadIdx.x; i < T * Z; i += kCsThreads)
    loc[i] = d.lat_std != nullptr ? __fadd_rn(__fmul_rn(lat[i], d.lat_std[i]), d.lat_mean[i]) : lat[i];
  cp_async_wait<2>();
  __syncthreads();
  // input_proj (+ suite embedding), every channel on every CTA: h0 [h][ht]
  const float* win = wbuf + 2 * kDecChunk;
  const int sid = (d.suite_ids != nullptr && d.suite_embed != nullptr) ? d.suite_ids[b] : -1;
  for (int i = threadIdx.x; i < h * T; i += kCsThreads) {
    const int c = i / T, t = i - c * T;
    float acc = d.in_b[c];
    for (int k = 0; k < Z; ++k) acc = fmaf(win[c * Z + k], loc[t * Z + k], acc);
    if (sid >= 0) acc += d.suite_embed[static_cast<long long>(sid) * h + c];
    h0[c * ht + t] = acc;
  }
  __syncthreads();  // h0 complete; buffer 2 free for chunk 2
  // 2. ConvTranspose1d for this CTA's channels, then GroupNorm + SiLU -> xa
  //    (the skip of the residual block), all CTAs
  if (sdn == 2)
    dec_convt<2>(h0, loc, wbuf, d.convt_w, d.convt_b, h, c0, ch, T, ht);
  else
    dec_convt<4>(h0, loc, wbuf, d.convt_w, d.convt_b, h, c0, ch, T, ht);
  dec_norm_exchange(loc, xa, nullptr, d.gn0_w, d.gn0_b, ch, c0, Lo, xs, cg, true, st, nc);
  // 3. residual block: Conv1d -> GN -> SiLU -> xb; Conv1d -> GN, + skip -> xb
  dec_conv3(xa, loc, wbuf, d.c1_w, d.c1_b, h, c0, ch, Lo, xs);
  dec_norm_exchange(loc, xb, nullptr, d.gn1_w, d.gn1_b, ch, c0, Lo, xs, cg, true, st, nc);
  dec_conv3(xb, loc, wbuf, d.c2_w, d.c2_b, h, c0, ch, Lo, xs);
  // output_proj's weight streams in while the last exchange runs; the block
  // output overwrites xb (no CTA reads xb any more once conv2 is done:
  // dec_conv3 ends with a CTA barrier and the exchange below with a cluster one)
  dec_copy(wbuf, d.out_w, d.action_dim * h);
  if (nc > 1) cluster_barrier();
  dec_norm_exchange(loc, xb, xa, d.gn2_w, d.gn2_b, ch, c0, Lo, xs, cg, false, st, nc);
  cp_async_wait<0>();
  __syncthreads();
  // 4. crop / zero-pad to the horizon, output_proj: CTA `rank` writes the rows
  //    [rank, rank + nc, ...) of the chunk, 4 threads per output
  const float* wo = wbuf;
  float* out = d.out + static_cast<long long>(b) * d.horizon * d.action_dim;
  const int A = d.action_dim, nout = ((d.horizon - rank + nc - 1) / nc) * A;
  for (int i0 = 0; i0 < nout * 4; i0 += kCsThreads) {
    const int i = i0 + threadIdx.x, e = i >> 2, part = i & 3;
    const bool live = i < nout * 4;
    const int pp = rank + (e / A) * nc, o = e - (e / A) * A;
    float acc = 0.f;
    if (live && pp < Lo)
      for (int c = part; c < h; c += 4) acc = fmaf(wo[o * h + c], xb[c * xs + pp], acc);
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (live && part == 0) out[pp * A + o] = acc + d.out_b[o];
  }
}

template <int HDIM, int FD, int FHD, int FF, int FA, int FS>
__global__ void __launch_bounds__(kCsThreads, 1) cae_steps_staged_kernel(const __grid_constant__ CaeStepArgs a) {
  extern __shared__ __align__(16) float csm[];
  const CaeStagePlan& p = a.plan;
  const int nc = p.nc;                                     // CTAs of the sample's cluster
  const int b = blockIdx.x / nc;
  const int rank = nc > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = FS ? FS : a.S, D = FD ? FD : a.D, A = FA ? FA : a.A, HD = FHD ? FHD : a.HD, H = HD / HDIM;
  const int F = FF ? FF : a.F, L = a.L, N = a.num_steps, C = a.C;
  const int hdp = FHD ? FHD + 4 : p.hdp, kc = p.kc;
  const float scale = rsqrtf(static_cast<float>(HDIM));
  const float scale_log2 = scale * 1.4426950408889634f;  // softmax in exp2 form
  const uint8_t* kmask = a.ctx_mask != nullptr ? a.ctx_mask + static_cast<long long>(b) * C : nullptr;
  float* latent = a.latent + static_cast<long long>(b) * S * A;
  const int U = p.units;
  const int ur = (U - rank + nc - 1) / nc;  // key chunks of each block handled by this CTA
  const int total = N * L;

  // ---- prologue: barriers, constant tensors, first t_mod batch, block 0 weights
  if (tid == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(CS_BAR(i), 1);
    for (int i = 5; i < 7; ++i) mbar_init(CS_BAR(i), nc);  // slice exchange, one arrival per CTA
    fence_mbar_init();
  }
  cs_stage(CS_SM(encw), a.w.enc_w, D, A, A + 4);
  cs_stage(CS_SM(encb), a.w.enc_b, 1, D, D);
  cs_stage(CS_SM(headw), a.w.head_w, A, D, D + 4);
  cs_stage(CS_SM(headb), a.w.head_b, 1, A, A);
  cs_stage(CS_SM(rope), a.rope, 1, S * HDIM, S * HDIM);
  cs_stage(CS_SM(lat), latent, 1, S * A, S * A);
  cp_async_commit();
  __syncthreads();
  if (nc > 1) cluster_barrier();  // every CTA's exchange barriers are initialised before any peer arrives
  cs_time_batch(a, csm, 0, min(p.tb, N));
  // K/V buffers start at zero: rows past a short last chunk are read by the
  // tensor-core tiles (their scores are masked, and 0 * finite stays 0)
  for (int i = tid; i < 2 * p.kv_floats; i += kCsThreads) CS_SM(kv)[i] = 0.f;
  fence_async_smem();
  __syncthreads();
  pdl_wait();  // packed weights and context K/V come from the preceding launch
  if (tid == 0) {
    cs_issue_a(a, csm, 0);
    cs_issue_f(a, csm, 0);
    cs_issue_kv<HDIM>(a, csm, 0, b, rank, ur);
  }
  pdl_launch_dependents();
  cp_async_wait<0>();
  cs_wait(a, csm, 0, 0);
  __syncthreads();

  for (int s = warp; s < S; s += kCsWarps) cs_step_entry_row(a, csm, s, 0, CS_ABUF(0), D, A);

  for (int e = 0; e < total; ++e) {
    const int step = e / L, l = e - step * L;
    float* ab = CS_ABUF(e);
    const float* mod = ab + p.off[0];
    const float* tmr = CS_SM(tm) + (step % p.tb) * 6 * D;
    __syncthreads();  // AdaLN-1 rows of this block written; previous block's FFN done
    if (tid == 0) {
      if (e + 1 < total) cs_issue_a(a, csm, e + 1);
      if (e > 0) cs_issue_f(a, csm, e);
    }

    // ---- q, k, v (+ RMSNorm over H*d, RoPE on q and k): warp per (row, part)
    for (int item = warp; item < 3 * S; item += kCsWarps) {
      const int s = item / 3, part = item - 3 * s;
      const float* w = ab + p.off[1] + part * HD * (D + 4);
      const float* bias = ab + p.off[2] + part * HD;
      float y[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        y[u] = o < HD ? bias[o] + cs_dot(w + o * (D + 4), CS_SM(h) + s * D, D) : 0.f;
      }
      float* dst = part == 0 ? CS_SM(q) : (part == 1 ? CS_SM(k) : CS_SM(v));
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
            const float c = CS_SM(rope)[(s * (HDIM / 2) + pi) * 2], sn = CS_SM(rope)[(s * (HDIM / 2) + pi) * 2 + 1];
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
      float scv = -INFINITY;
      if (lane < S) {
        const float* qr = CS_SM(q) + s * hdp + hh * HDIM;
        const float* kr = CS_SM(k) + lane * hdp + hh * HDIM;
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
        scv = d * scale_log2;
      }
      const float mx = warp_max(scv);
      const float pj = lane < S ? exp2f(scv - mx) : 0.f;
      const float den = warp_sum(pj);
      float acc = 0.f;
      const int d = lane % HDIM;
      for (int j = 0; j < S; ++j) {
        const float pp = __shfl_sync(0xffffffffu, pj, j);
        acc = fmaf(pp, CS_SM(v)[j * hdp + hh * HDIM + d], acc);
      }
      if (lane < HDIM) CS_SM(att)[s * hdp + hh * HDIM + lane] = acc / den;
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
          const float y = ob[o] + cs_dot(ow + o * (HD + 4), CS_SM(att) + s * hdp, HD);
          xv[u] = CS_SM(x)[s * D + o] + (mod[2 * D + o] + tmr[2 * D + o]) * y;
          CS_SM(x)[s * D + o] = xv[u];
        }
      }
      float mean, rstd;
      cs_row_stats(xv, D, a.eps, mean, rstd);
      const float* n3w = ab + p.off[7];
      const float* n3b = ab + p.off[8];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        if (o < D) CS_SM(h)[s * D + o] = (xv[u] - mean) * rstd * n3w[o] + n3b[o];
      }
      __syncwarp();
      const float* cw = ab + p.off[9];
      const float* cb = ab + p.off[10];
      const float* cn = ab + p.off[11];
      float y[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        y[u] = o < HD ? cb[o] + cs_dot(cw + o * (D + 4), CS_SM(h) + s * D, D) : 0.f;
      }
      const float r = rsqrtf(warp_sum(y[0] * y[0] + y[1] * y[1]) / HD + a.eps);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int o = lane + 32 * u;
        if (o < HD) CS_SM(qc)[s * hdp + o] = y[u] * r * cn[o];
      }
    }

    // ---- cross attention: key chunks of all heads; warp = (head, 16 keys of the
    // chunk), tensor-core scores and P.V with a running softmax across chunks.
    // The chunks of a block are dealt over the nc CTAs of the sample's cluster.
    {
      const int wh = p.wh, hh = warp / wh, slot = warp - hh * wh;
      const bool act = hh < H;
      CsFlash<HDIM> fl;
      fl.init();
      for (int i = 0; i < ur; ++i) {
        const int g = e * ur + i;
        cs_wait(a, csm, 3 + (g & 1), (g >> 1) & 1);
        __syncthreads();  // chunk g landed; every warp is done with chunk g - 1 (the other buffer)
        if (tid == 0 && g + 1 < total * ur) cs_issue_kv<HDIM>(a, csm, g + 1, b, rank, ur);
        if (act) {
          const int j0 = (rank + i * nc) * kc;
          fl.chunk(CS_KV(g), kc, HD, min(kc, C - j0), slot * 16, hh, CS_SM(qc), hdp, S,
                   kmask != nullptr ? kmask + j0 : nullptr, scale_log2);
        }
      }
      if (act) fl.store(CS_SM(part) + (hh * wh + slot) * S * (HDIM + 2), S);
    }
    __syncthreads();
    // merge the wh key slices of each (head, row) into one partial (m, l, o) and
    // publish it to slot `rank` of every cluster CTA's exchange buffer
    {
      const int par = e & 1, row_f = HDIM + 2;
      float* xp = CS_SM(xpart) + (par * nc + rank) * H * S * row_f;
      for (int t = tid; t < H * S * row_f; t += kCsThreads) {
        const int j = t % row_f, hs = t / row_f, hh = hs / S, s2 = hs - hh * S;
        const float* pp = CS_SM(part) + (hh * p.wh * S + s2) * row_f;
        const int pst = S * row_f;
        float mx = -INFINITY;
        for (int sl = 0; sl < p.wh; ++sl) mx = fmaxf(mx, pp[sl * pst]);
        float v = mx;
        if (j > 0) {
          v = 0.f;
          if (mx != -INFINITY)
            for (int sl = 0; sl < p.wh; ++sl) {
              const float* q = pp + sl * pst;
              if (q[0] != -INFINITY) v = fmaf(exp2f(q[0] - mx), q[j], v);  // slice maxima: log2 domain
            }
        }
        if (nc == 1) {
          xp[t] = v;
        } else {
          for (int r2 = 0; r2 < nc; ++r2) st_cluster_f32(cluster_map(xp + t, r2), v);
        }
      }
      if (nc > 1) {
        asm volatile("fence.acq_rel.cluster;" ::: "memory");
        __syncthreads();
        if (tid == 0)
          for (int r2 = 0; r2 < nc; ++r2) mbar_arrive_cluster(cluster_map(CS_BAR(5 + par), r2));
        // every CTA's slices of this block have landed (bounded wait)
        const uint32_t want = static_cast<uint32_t>(e >> 1) & 1;
        if (!mbar_try_wait_cluster(CS_BAR(5 + par), want)) {
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait_cluster(CS_BAR(5 + par), want)) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
              record_error(a.status, kCsErrWait);
              break;
            }
          }
        }
      }
    }
    __syncthreads();

    // ---- row chain: merge the key chunks; x += cross_o(attn); h = AdaLN 2(x)
    for (int s = warp; s < S; s += kCsWarps) {
#pragma unroll
      for (int u2 = 0; u2 < 2; ++u2) {
        const int o = lane + 32 * u2;
        if (o < HD) {
          const int hh = o / HDIM, d = o - hh * HDIM;
          const int row_f = HDIM + 2;
          const float* pp = CS_SM(xpart) + ((e & 1) * nc * H * S + hh * S + s) * row_f;
          const int pst = H * S * row_f;  // next cluster rank
          float mx = -INFINITY;
          for (int r2 = 0; r2 < nc; ++r2) mx = fmaxf(mx, pp[r2 * pst]);
          float num = 0.f, den = 0.f;
          if (mx != -INFINITY) {
            for (int r2 = 0; r2 < nc; ++r2) {
              const float* q = pp + r2 * pst;
              if (q[0] == -INFINITY) continue;
              const float fct = exp2f(q[0] - mx);  // maxima in the log2 domain
              den = fmaf(fct, q[1], den);
              num = fmaf(fct, q[2 + d], num);
            }
          }
          CS_SM(att)[s * hdp + o] = den > 0.f ? num / den : 0.f;
        }
      }
      __syncwarp();
      const float* cw = ab + p.off[12];
      const float* cb = ab + p.off[13];
      float xv[2];
#pragma unroll
      for (int u2 = 0; u2 < 2; ++u2) {
        const int o = lane + 32 * u2;
        xv[u2] = 0.f;
        if (o < D) {
          xv[u2] = CS_SM(x)[s * D + o] + (cb[o] + cs_dot(cw + o * (HD + 4), CS_SM(att) + s * hdp, HD));
          CS_SM(x)[s * D + o] = xv[u2];
        }
      }
      cs_adaln_row(xv, CS_SM(h) + s * D, mod, tmr, D, a.eps, 3, 4);
    }
    cs_wait(a, csm, 2, e & 1);                                      // this block's FFN half
    if (e + 1 < total) cs_wait(a, csm, (e + 1) & 1, ((e + 1) >> 1) & 1);  // next block's attention half
    __syncthreads();

    // ---- FFN 0 + GELU(tanh): warp per (row, 32 outputs)
    {
      const int ng = (F + 31) / 32;
      const float* w = CS_SM(fbuf) + p.off[14];
      const float* bias = CS_SM(fbuf) + p.off[15];
      for (int item = warp; item < S * ng; item += kCsWarps) {
        const int s = item / ng, o = (item - s * ng) * 32 + lane;
        if (o < F) CS_SM(f)[s * F + o] = gelu_tanh(bias[o] + cs_dot(w + o * (D + 4), CS_SM(h) + s * D, D));
      }
    }
    __syncthreads();

    // ---- row chain: x += gate_mlp * ffn2(f); then the next block's AdaLN 1, or
    // (last block) head, Euler update, the next step's encoder and AdaLN 1
    const bool last = l == L - 1;
    const bool more = e + 1 < total;
    const bool new_batch = last && more && ((step + 1) % p.tb) == 0;
    const float* abn = CS_ABUF(e + 1);
    for (int s = warp; s < S; s += kCsWarps) {
      const float* w = CS_SM(fbuf) + p.off[16];
      const float* bias = CS_SM(fbuf) + p.off[17];
      float xv[2];
#pragma unroll
      for (int u2 = 0; u2 < 2; ++u2) {
        const int o = lane + 32 * u2;
        xv[u2] = 0.f;
        if (o < D) {
          const float y = bias[o] + cs_dot(w + o * (F + 4), CS_SM(f) + s * F, F);
          xv[u2] = CS_SM(x)[s * D + o] + (mod[5 * D + o] + tmr[5 * D + o]) * y;
          CS_SM(x)[s * D + o] = xv[u2];
        }
      }
      if (!last) {
        cs_adaln_row(xv, CS_SM(h) + s * D, abn + p.off[0], tmr, D, a.eps, 0, 1);
        continue;
      }
      __syncwarp();
      const float delta = a.deltas.t[step];
#pragma unroll
      for (int u2 = 0; u2 < 2; ++u2) {
        const int o = lane + 32 * u2;
        if (o < A) {
          const float vel = CS_SM(headb)[o] + cs_dot(CS_SM(headw) + o * (D + 4), CS_SM(x) + s * D, D);
          if (a.trace != nullptr && rank == 0) a.trace[(static_cast<long long>(step) * a.B + b) * S * A + s * A + o] = vel;
          const float nl = CS_SM(lat)[s * A + o] + vel * delta;
          CS_SM(lat)[s * A + o] = nl;
          if (!more && rank == 0) latent[s * A + o] = nl;
        }
      }
      __syncwarp();
      if (more && !new_batch) cs_step_entry_row(a, csm, s, step + 1, abn, D, A);
    }
    if (new_batch) {
      __syncthreads();
      cs_time_batch(a, csm, step + 1, min(p.tb, N - step - 1));
      for (int s = warp; s < S; s += kCsWarps) cs_step_entry_row(a, csm, s, step + 1, abn, D, A);
    }
  }
  if (a.dec.enabled) {
    // every CTA of the cluster is past its last block before any peer writes
    // decode activations into the (now dead) weight buffers
    if (nc > 1) cluster_barrier(); else __syncthreads();
    cs_decode_epilogue(a, csm, b, nc);
  }
  if (nc > 1) cluster_barrier();  // no CTA leaves while a peer could still address its shared memory
}

template <int HDIM, int FD, int FHD, int FF, int FA, int FS>
cudaError_t launch_staged(const CaeStepArgs& a, cudaStream_t st, bool pdl) {
  auto kern = cae_steps_staged_kernel<HDIM, FD, FHD, FF, FA, FS>;
  const size_t smem = static_cast<size_t>(a.plan.total_floats) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.B * a.plan.nc);
  cfg.blockDim = dim3(kCsThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = a.plan.nc;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

int round4(int v) { return (v + 3) & ~3; }

}  // namespace

void cae_tensor_table(int D, int HD, int F, CaeStagePlan* p) {
  auto tensor = [&](int t, int rows, int cols, int stride, int& cursor) {
    p->off[t] = cursor;
    p->rows[t] = rows;
    p->cols[t] = cols;
    p->stride[t] = stride;
    cursor += round4(rows * stride);
  };
  int ca = 0;
  tensor(0, 1, 6 * D, 6 * D, ca);        // modulation
  tensor(1, 3 * HD, D, D + 4, ca);       // qkv
  tensor(2, 1, 3 * HD, 3 * HD, ca);
  tensor(3, 1, HD, HD, ca);              // norm_q
  tensor(4, 1, HD, HD, ca);              // norm_k
  tensor(5, D, HD, HD + 4, ca);          // o
  tensor(6, 1, D, D, ca);
  tensor(7, 1, D, D, ca);                // norm3
  tensor(8, 1, D, D, ca);
  tensor(9, HD, D, D + 4, ca);           // cross q
  tensor(10, 1, HD, HD, ca);
  tensor(11, 1, HD, HD, ca);             // cross norm_q
  tensor(12, D, HD, HD + 4, ca);         // cross o
  tensor(13, 1, D, D, ca);
  int cf = 0;
  tensor(14, F, D, D + 4, cf);           // ffn.0
  tensor(15, 1, F, F, cf);
  tensor(16, D, F, F + 4, cf);           // ffn.2
  tensor(17, 1, D, D, cf);
  p->a_floats = ca;
  p->f_floats = cf;
}

int cae_decode_floats(const CaeDecode& d, int nc) {
  int a, b, l, w, st;
  return dec_layout(d, nc, &a, &b, &l, &w, &st);
}

bool cae_staged_plan(const CaeStepArgs& a, CaeStagePlan* out) {
  const int S = a.S, D = a.D, A = a.A, HD = a.HD, hd = a.hd, F = a.F, C = a.C;
  if (S < 1 || S > kCsMaxRows || D > 64 || HD > 64 || A > 64 || A < 1 || C < 1) return false;
  if (HD / hd > kCsWarps) return false;
  if (hd != 4 && hd != 8 && hd != 16) return false;
  if (HD % hd != 0 || D % 4 != 0 || HD % 4 != 0 || F % 4 != 0 || A % 4 != 0 || F < 4) return false;
  if (a.freq_dim < 2 || a.freq_dim % 2 != 0 || a.num_steps < 1 || a.L < 1) return false;
  CaeStagePlan p;
  memset(&p, 0, sizeof(p));
  const int H = HD / hd;
  cae_tensor_table(D, HD, F, &p);
  p.hdp = HD + 4;
  p.tb = a.num_steps < kCsMaxTb ? a.num_steps : kCsMaxTb;
  p.wh = kCsWarps / H;
  p.kc = 16 * p.wh;
  p.units = (C + p.kc - 1) / p.kc;
  p.nc = p.units < kCsMaxCluster ? p.units : kCsMaxCluster;
  int c = 0;
  auto take = [&](int n) {
    const int o = c;
    c += round4(n);
    return o;
  };
  p.kv_floats = round4(p.kc * (2 * HD + 12));
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
  p.o_part = take(H * p.wh * S * (hd + 2));
  p.o_xpart = take(2 * p.nc * H * S * (hd + 2));  // [block parity][cluster rank][H][S][m, l, o]
  p.o_tm = take(p.tb * 6 * D);
  p.o_tscr = take(p.tb * (a.freq_dim + 2 * D));
  p.o_lat = take(S * A);
  p.o_rope = take(S * hd);
  p.o_encw = take(D * (A + 4));
  p.o_encb = take(D);
  p.o_headw = take(A * (D + 4));
  p.o_headb = take(A);
  p.o_bar = take(14);  // 7 mbarriers (8-byte aligned: every offset is a multiple of 4 floats)
  p.total_floats = c;
  const bool ok = static_cast<size_t>(c) * sizeof(float) <= static_cast<size_t>(kCsSmemLimit);
  if (!ok) return false;
  *out = p;
  return true;
}

cudaError_t launch_cae_steps_staged(const CaeStepArgs& a, cudaStream_t st, bool pdl) {
  // BASELINE config 0 shape (hidden 32, 4 x 8 heads, FFN 128, 16 latent dims, 8 tokens)
  if (a.hd == 8 && a.D == 32 && a.HD == 32 && a.F == 128 && a.A == 16 && a.S == 8)
    return launch_staged<8, 32, 32, 128, 16, 8>(a, st, pdl);
  switch (a.hd) {
    case 4: return launch_staged<4, 0, 0, 0, 0, 0>(a, st, pdl);
    case 8: return launch_staged<8, 0, 0, 0, 0, 0>(a, st, pdl);
    default: return launch_staged<16, 0, 0, 0, 0, 0>(a, st, pdl);
  }
}

}  // namespace fam
