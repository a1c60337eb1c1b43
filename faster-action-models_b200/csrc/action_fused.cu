// Fused persistent action chunk: every Euler step x every block of the action
// expert in ONE cooperative launch, one CTA per SM.
//
// At batch 1 the action path is latency bound (32 token rows against 0.8 GB
// of weights per model evaluation): a chain of small kernels pays a launch /
// grid-drain latency per op.  Here the weight stream is decoupled from the
// activation dependency chain:
//
//   warp 0 (producer)   walks this CTA's static list of GEMM work items for the
//                       whole chunk and TMA-loads their 128 x 64 weight tiles
//                       into an 8-stage shared-memory ring as fast as the ring
//                       drains — weights never depend on activations, so the
//                       stream runs ahead across phase and step boundaries;
//   warps 1..11         run the phases: stage the MMA B operand (the token
//   (workers)           rows) straight from the bf16 residual stream with the
//                       block's LayerNorm / AdaLN folded in, issue tcgen05.mma
//                       into 128 x 32 fp32 TMEM accumulators, and apply the
//                       epilogue in warps 2..9 (bias, RMSNorm statistics,
//                       RoPE, GELU; the residual GEMMs store split partials
//                       and the last split of a tile completes the gated
//                       residual add with the reference's bf16 roundings).
//                       Attention phases stage K / V with cp.async in the
//                       128-byte-swizzled layout and run S = Q K^T and P.V on
//                       tcgen05 (S, P and O in TMEM; the 32 queries replicated
//                       over the four TMEM lane quarters, each softmax warp
//                       owning a quarter of the item's keys).
// Every cross-CTA sum is order-independent (fp64 sums of squares, split
// partials summed in split order), so a launch is deterministic.
//
// Per block the phases are separated by grid barriers:
//   qkv GEMM (AdaLN1 prologue; q/k RMSNorm sums + weight + RoPE epilogue)
//   -> joint attention over [video cache ; action] (RMSNorm scales applied to
//      the logits; split-KV merged by the last CTA per head)
//   -> o GEMM (+= gate_msa, split by head)  -> cross-q GEMM (norm3 prologue)
//   -> cross attention -> cross-o GEMM (+=) -> ffn.0 GEMM (AdaLN2 prologue,
//      GELU epilogue) -> ffn.2 GEMM (+= gate_mlp, split by ffn.0 tile)
// and each step starts with action_encoder and ends with head + Euler update.
//
// RMSNorm over the whole H*d row (wan_video_dit.py:146-157) is applied as a
// per-token scale: RMSNorm(y)*w then RoPE equals s(y) * RoPE(y*w) because the
// rotation is linear, so the GEMM epilogue stores RoPE(y*w) and accumulates
// sum(y^2) per token; the attention multiplies q by s_q and the logits of the
// fresh keys by s_k.  Reference numerics otherwise as the separate kernels:
// DiTBlock.forward (wan_video_dit.py:248-267), MoT joint attention
// (mot.py:528-578), scheduler step (scheduler_continuous.py:82-88).
#include <cstddef>

#include "action_fused.h"
#include "fam_common.cuh"
#include "fam_internal.h"
#include "fam_mma.cuh"

namespace fam {

constexpr int kATile = 128 * 64 * 2;          // one weight tile (16 KB)
constexpr int kBBlock = kFusedRows * 128;     // one B k-block: 32 rows x 128 B (4 KB)
constexpr int kFusedIssuers = 4;               // MMA-issuing threads per GEMM item
constexpr int kFusedIssuer1 = 6;               // warps kFusedIssuer1.. host issuers 1..
static_assert(kFusedIssuer1 + kFusedIssuers - 1 <= kFusedThreads / 32 && kFusedIssuers % 2 == 0, "issuer warps");
constexpr int kSplitStride = kFusedRows * 64 + kFusedRows * 2;  // floats per split partial
// Staging layout for the GEMM phases: the B operand (<= 16 K blocks = 64 KB,
// D <= 1024), then the RoPE (cos, sin) slices of the q/k epilogue warps
// (4 x 32 tokens x 16 pairs), then the LayerNorm constants (2 x D fp32).
constexpr int kStgRope = 16 * kBBlock;
constexpr int kStgLnConst = kStgRope + 4 * kFusedRows * 16 * 8;
// pair items: the peer's partial accumulators of this CTA's output rows,
// [32 tokens][64 rows] fp32, behind the half-width B operand (<= 8 K blocks)
constexpr int kStgXacc = 8 * kBBlock;
constexpr int kStgXsend = kStgXacc + kFusedRows * 64 * 4;  // this CTA's outgoing partials
constexpr uint32_t kXaccBytes = kFusedRows * 64 * 4;
static_assert(kStgXsend + kXaccBytes <= kStgRope, "pair exchange buffers");
static_assert(kStgLnConst + 2 * 1024 * 4 <= kFusedStaging, "staging layout");

struct FusedSmemTail {
  uint64_t full[kFusedRing];
  uint64_t empty[kFusedRing];
  uint64_t accum;
  uint32_t tmem;
  volatile int abort;
  float stat[kFusedRows][2];
  int last;
  int fin;                                    // this residual item completes its tile
  // pair items: the peer CTA writes its half-row LayerNorm sums here and
  // arrives on xstat_bar (one arrival per worker warp); its partial
  // accumulators arrive in the staging (kStgXacc) by one bulk copy that
  // completes on xacc_bar (armed here with the expected bytes); xsend_bar
  // gathers this CTA's four sending warps before it issues its own copy
  alignas(16) float xstat[kFusedRows][2];  // 8-byte (v2) remote stores and loads
  uint64_t xstat_bar;
  uint64_t xacc_bar;
  uint64_t xsend_bar;
  uint64_t attn_s;     // S = Q K^T of the attention item complete
  uint64_t attn_o[4];  // softmax warp w's P.V complete
};

static_assert(offsetof(FusedSmemTail, xstat) % 8 == 0, "xstat rows are accessed as float2");

__host__ __device__ constexpr size_t fused_tail_offset() {
  return static_cast<size_t>(kFusedRing) * kATile + kFusedStaging;
}
size_t fused_smem_bytes() { return fused_tail_offset() + sizeof(FusedSmemTail) + 1024; }

__device__ __forceinline__ void bar_workers() {
  asm volatile("barrier.sync 1, %0;" ::"r"(kFusedWorkers) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---------------------------------------------------------------- schedule
// GEMM work items.  The LayerNorm GEMMs (qkv, cross-q, ffn.0: full K = D) run
// as pair items on the two CTAs of a cluster: each CTA LayerNorms and stages
// half of the K columns, runs half of the K blocks, and the pair exchanges the
// row statistics and the partial accumulators through distributed shared
// memory (each CTA then finishes half of the 128 output rows).  The residual
// GEMMs (o, cross-o, ffn.2) are split-K items of one CTA.
struct FItem {
  int n;       // 128-row tile of the output features
  int sub;     // head group (o, co), ffn.0 tile group (ffn2), 0 otherwise
  int kb0;     // first 64-wide K block
  int nkb;     // K blocks
};

__device__ __forceinline__ bool f_pair(int p) { return p == kFQkv || p == kFCq || p == kFFfn0; }
__device__ __forceinline__ int f_rows(const FusedArgs& a, int p) {
  switch (p) {
    case kFQkv: return 3 * a.HD;
    case kFO: return a.D;
    case kFCq: return a.HD;
    case kFCo: return a.D;
    case kFFfn0: return a.F;
    default: return a.D;
  }
}
// Split-K items of the residual GEMMs take a group of heads (o, cross-o) or of
// ffn.0 tiles (ffn.2): fewer fp32 atomic contributions per output element.
__device__ __forceinline__ int f_head_group(const FusedArgs& a) {
  return (a.H % 4 == 0) ? 4 : ((a.H % 2 == 0) ? 2 : 1);
}
__device__ __forceinline__ int f_ffn_group(const FusedArgs& a) {
  const int js = a.F / 128;
  return (js % 4 == 0) ? 4 : ((js % 2 == 0) ? 2 : 1);
}
__device__ __forceinline__ int f_count(const FusedArgs& a, int p) {
  const int nt = f_rows(a, p) / 128;
  if (p == kFO || p == kFCo) return nt * (a.H / f_head_group(a));
  if (p == kFFfn2) return nt * (a.F / 128 / f_ffn_group(a));
  return nt;
}
// Placement: pair items on pairs 0.. (qkv, then cross-q, then ffn.0); ffn.2 on
// CTAs 0.. (the qkv / cross-q CTAs: their next LayerNorm GEMM is phases away,
// so both items' tiles fit the ring in time); o and cross-o after the pair
// CTAs (idle in the phase before the ffn.0 pairs take theirs).
__device__ __forceinline__ int f_offset(const FusedArgs& a, int p) {
  const int pq = 3 * a.HD / 128, pc = a.HD / 128, pf = a.F / 128;
  switch (p) {
    case kFQkv: return 0;
    case kFCq: return pq;
    case kFFfn0: return pq + pc;
    case kFFfn2: return 0;
    default: return 2 * (pq + pc + pf);  // o, cross-o (CTA units)
  }
}
// the scheduling unit of a phase: a pair (cluster) or a CTA
__device__ __forceinline__ int f_units(int p, int G) { return f_pair(p) ? G / 2 : G; }
__device__ __forceinline__ int f_first(const FusedArgs& a, int p, int cta, int G) {
  const int u = f_pair(p) ? cta / 2 : cta, n = f_units(p, G);
  return ((u - f_offset(a, p)) % n + n) % n;
}
// item i of phase p; `half` = cluster rank for pair items
__device__ __forceinline__ FItem f_item(const FusedArgs& a, int p, int i, int half) {
  FItem it;
  if (p == kFO || p == kFCo) {
    const int hg = f_head_group(a), groups = a.H / hg;
    it.n = i / groups;
    it.sub = i % groups;
    it.kb0 = it.sub * hg * (a.hd / 64);
    it.nkb = hg * (a.hd / 64);
  } else if (p == kFFfn2) {
    const int fg = f_ffn_group(a), groups = a.F / 128 / fg;
    it.n = i / groups;
    it.sub = i % groups;
    it.kb0 = it.sub * 2 * fg;
    it.nkb = 2 * fg;
  } else {
    const int kh = a.D / 128;  // K blocks per half
    it.n = i;
    it.sub = 0;
    it.kb0 = half * kh;
    it.nkb = kh;
  }
  return it;
}

// ----------------------------------------------------------- grid barrier
// Flag barrier (one propagation hop): every worker warp of a CTA adds 1 to the
// CTA's own 128-byte flag line with a release reduction right after its own
// writes of the phase (the warps' write-acknowledgement waits overlap instead
// of one CTA-wide fence after the slowest warp), and worker thread i of every
// CTA acquire-polls the line of CTA i until it reaches 11 x the barrier index.
// Every wait is bounded; a timeout or an abort raised elsewhere sets the abort
// word and every CTA leaves its phase loop.
constexpr unsigned kFusedWorkerWarps = kFusedWorkers / 32;
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The flag is re-read back to back; the abort word and the clock are checked
// every 16th read only, so a poll iteration is one L2 round trip.
__device__ __forceinline__ bool poll_ge(const FusedArgs& a, const unsigned* p, unsigned target,
                                        FusedSmemTail* tl) {
  if (ld_acquire(p) >= target) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (unsigned it = 1;; ++it) {
    if (ld_acquire(p) >= target) return true;
    if ((it & 15) == 0 && (ld_acquire(a.sync + 1) != 0 || globaltimer_ns() - t0 > kWaitLimitNs)) {
      if (ld_acquire(a.sync + 1) == 0) record_error(a.status, kErrWaitFull);
      atomicExch(a.sync + 1, 1u);
      tl->abort = 1;
      return false;
    }
  }
}

__device__ __forceinline__ bool grid_sync(const FusedArgs& a, unsigned& epoch, FusedSmemTail* tl) {
  // __syncwarp orders the warp's writes before lane 0's release reduction
  // (cumulative at gpu scope)
  __syncwarp();
  ++epoch;
  const int wt = threadIdx.x - 32;
  if ((threadIdx.x & 31) == 0) red_release_add(a.flags + blockIdx.x * 32, 1u);
  // one hop: worker thread i of every CTA waits for CTA i's eleven arrivals
  if (wt < static_cast<int>(gridDim.x)) poll_ge(a, a.flags + wt * 32, epoch * kFusedWorkerWarps, tl);
  bar_workers();
  return tl->abort == 0;
}

// -------------------------------------------------------- B operand staging
// Write 8 bf16 (16 bytes) as chunk c of row r of K block kb, 128-byte swizzle
// (the layout a TMA SWIZZLE_128B load produces and the UMMA descriptor reads).
__device__ __forceinline__ void stage_chunk(uint8_t* stg, int kb, int r, int c, uint4 v) {
  *reinterpret_cast<uint4*>(stg + kb * kBBlock + r * 128 + ((c ^ (r & 7)) << 4)) = v;
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  u.x = pack_bf16(f[0], f[1]);
  u.y = pack_bf16(f[2], f[3]);
  u.z = pack_bf16(f[4], f[5]);
  u.w = pack_bf16(f[6], f[7]);
  return u;
}

// modulation chunk c of block l at step s for feature f: bf16(bf16(t_mod) + modulation)
__device__ __forceinline__ float f_mod(const FusedArgs& a, int step, int l, int c, int f) {
  const float t = rbf(a.tmod[static_cast<long long>(step) * 6 * a.D + c * a.D + f]);
  return rbf(t + bf2f(a.modulation[(static_cast<long long>(l) * 6 + c) * a.D + f]));
}

__device__ __forceinline__ void ld_bf8(const __nv_bfloat16* p, float* o) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = __low2float(h[i]);
    o[2 * i + 1] = __high2float(h[i]);
  }
}
__device__ __forceinline__ void ld_f8(const float* p, float* o) {
  const float4 a0 = *reinterpret_cast<const float4*>(p), a1 = *reinterpret_cast<const float4*>(p + 4);
  o[0] = a0.x; o[1] = a0.y; o[2] = a0.z; o[3] = a0.w;
  o[4] = a1.x; o[5] = a1.y; o[6] = a1.z; o[7] = a1.w;
}

// LayerNorm of the residual rows into the B staging.  mode 0: AdaLN with
// chunks (c0, c0+1); mode 1: affine norm3 of block l.  Each lane owns the
// 8-wide column chunks lane + 32u (u < NCH, D = 256 NCH).
//
// The per-column constants (1 + scale and shift, or the norm3 weight and
// bias) do not depend on the residual: ln_const_prefetch stores them as fp32
// into shared memory behind the B operand at the end of the phase before,
// after this CTA's own items of that phase (the staging is free then; with
// the CTA offsets of the schedule the LayerNorm-GEMM CTAs are idle in the
// phase before, so the prefetch is off the critical path), and every item of
// the phase reads them there.  The residual rows are loaded up front so the L2
// round trips overlap: the warp's first two rows together, the third while
// the first two are normalised.
__device__ __forceinline__ void bf8_unpack(const uint4& u, float* o) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = __low2float(h[i]);
    o[2 * i + 1] = __high2float(h[i]);
  }
}

// fp32 [D] multiplier then [D] addend at stg + kStgLnConst; worker thread t
// handles the 8-wide column chunk t.
__device__ void ln_const_prefetch(const FusedArgs& a, uint8_t* stg, int step, int l, int mode, int c0) {
  const int D = a.D;
  for (int ch = threadIdx.x - 32; ch < D / 8; ch += kFusedWorkers) {
    const int f0 = ch * 8;
    float m[8], ad[8];
    if (mode == 0) {
      float t0[8], t1[8], w0[8], w1[8];
      const float* tm = a.tmod + static_cast<long long>(step) * 6 * D;
      ld_f8(tm + c0 * D + f0, t0);
      ld_f8(tm + (c0 + 1) * D + f0, t1);
      ld_bf8(a.modulation + (static_cast<long long>(l) * 6 + c0) * D + f0, w0);
      ld_bf8(a.modulation + (static_cast<long long>(l) * 6 + c0 + 1) * D + f0, w1);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ad[e] = rbf(rbf(t0[e]) + w0[e]);        // shift
        m[e] = 1.f + rbf(rbf(t1[e]) + w1[e]);   // 1 + scale
      }
    } else {
      ld_bf8(a.norm3_w + static_cast<long long>(l) * D + f0, m);
      ld_bf8(a.norm3_b + static_cast<long long>(l) * D + f0, ad);
    }
    if (mode == 0) {
      // AdaLN: bf16 (1 + scale) and shift pairs, [D / 2] bf16x2 each (the
      // reference's modulate works on bf16 tensors; the staging applies them
      // as a packed bf16 multiply, then a packed bf16 add)
      uint4* cm = reinterpret_cast<uint4*>(stg + kStgLnConst) + ch;
      uint4* ca = reinterpret_cast<uint4*>(stg + kStgLnConst) + D / 8 + ch;
      *cm = make_uint4(pack_bf16(m[0], m[1]), pack_bf16(m[2], m[3]), pack_bf16(m[4], m[5]), pack_bf16(m[6], m[7]));
      *ca = make_uint4(pack_bf16(ad[0], ad[1]), pack_bf16(ad[2], ad[3]), pack_bf16(ad[4], ad[5]),
                       pack_bf16(ad[6], ad[7]));
    } else {
      float* cm = reinterpret_cast<float*>(stg + kStgLnConst) + f0;
      float* ca = cm + D;
      reinterpret_cast<float4*>(cm)[0] = make_float4(m[0], m[1], m[2], m[3]);
      reinterpret_cast<float4*>(cm)[1] = make_float4(m[4], m[5], m[6], m[7]);
      reinterpret_cast<float4*>(ca)[0] = make_float4(ad[0], ad[1], ad[2], ad[3]);
      reinterpret_cast<float4*>(ca)[1] = make_float4(ad[4], ad[5], ad[6], ad[7]);
    }
  }
}

// L2 load kept at its place in the program (volatile asm): the residual rows
// of the next LayerNorm rows are issued before the current row is
// normalised, and the compiler would otherwise sink them to their first use.
__device__ __forceinline__ float4 ld_cg_f4_early(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_cg_u4_early(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Half rows: this CTA's D / 2 columns [half * D / 2, ...) of the bf16
// residual row r, lane chunks lane + 32u (u < NCH, D / 2 = 256 NCH), 8 values
// per 16-byte load kept packed; rows >= R read as zeros.
template <int NCH>
__device__ __forceinline__ void ln_load_half(const FusedArgs& a, int r, int lane, int half, uint4 (&v)[NCH]) {
  const __nv_bfloat16* xr = a.x + static_cast<long long>(r) * a.D + half * (NCH * 256);
#pragma unroll
  for (int u = 0; u < NCH; ++u) {
    const int ch = lane + 32 * u;
    v[u] = r < a.R ? ld_cg_u4_early(xr + ch * 8) : make_uint4(0, 0, 0, 0);
  }
}

// Shifted sums of a half row: sum (x - c) and sum (x - c)^2 with c = x[r][0]
// (the same shift in both halves keeps the one-pass variance well conditioned).
template <int NCH>
__device__ __forceinline__ void ln_half_sums(const uint4 (&x)[NCH], float c, float& s1, float& s2) {
  s1 = 0.f;
  s2 = 0.f;
#pragma unroll
  for (int u = 0; u < NCH; ++u) {
    float f[8];
    bf8_unpack(x[u], f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float d = f[i] - c;
      s1 += d;
      s2 += d * d;
    }
  }
}

__device__ __forceinline__ bool mbar_wait_cl(const FusedArgs& a, uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_error(a.status, code);
      return false;
    }
  }
  return true;
}

// LayerNorm staging of a pair item.  mode 0: AdaLN (constants 1 + scale,
// shift); mode 1: affine norm3.  The warp's three rows r0 = w, r1 = w + 11,
// r2 = w + 22 are processed together (independent instruction streams).  The
// two CTAs of the pair exchange their half-row sums: lane 0 of every worker
// warp stores them into the peer's xstat and arrives on the peer's xstat_bar,
// then waits for the peer's eleven arrivals on its own.  With `st` (the row
// sums the residual GEMM before wrote, [32][2] fp64) the sums and the exchange
// are skipped.  Rows >= R are staged as zeros; a row >= 32 (the third row of
// the last warp) does not exist.  Returns false on a timed-out exchange.
template <int NCH>
__device__ bool stage_layernorm_pair_t(const FusedArgs& a, uint8_t* stg, FusedSmemTail* tl, int mode, int half,
                                       uint32_t parity, const double* st) {
  constexpr int DH = NCH * 256;  // columns of this half
  const int D = a.D;
  const int wid = (threadIdx.x >> 5) - 1, lane = threadIdx.x & 31;
  const int r0 = wid, r1 = wid + 11, r2 = wid + 22;
  const bool has2 = r2 < kFusedRows;
  uint4 xa[NCH], xb[NCH], xc[NCH];  // the residual rows (bf16, packed), all loads in flight together
  ln_load_half<NCH>(a, r0, lane, half, xa);
  ln_load_half<NCH>(a, r1, lane, half, xb);
  ln_load_half<NCH>(a, has2 ? r2 : kFusedRows, lane, half, xc);
  float ra, ba, rb, bb, rc, bc;
  // mean = S1 / D, var = S2 / D - mean^2 (fp64); n = x * rstd - mean * rstd
  auto stats64 = [&](const double* s, int r, float& rs, float& b) {
    const double m = __ldcg(s) / D;
    const double var = fmax(__ldcg(s + 1) / D - m * m, 0.0);
    rs = r < a.R ? rsqrtf(static_cast<float>(var) + a.eps) : 0.f;
    b = -static_cast<float>(m) * rs;
  };
  if (st != nullptr) {
    stats64(st + 2 * r0, r0, ra, ba);
    stats64(st + 2 * r1, r1, rb, bb);
    if (has2) stats64(st + 2 * r2, r2, rc, bc); else rc = bc = 0.f;
  } else {
    // the shift of the one-pass variance: a value common to both halves (the
    // first element of the row)
    const float ca = r0 < a.R ? bf2f(a.x[static_cast<long long>(r0) * D]) : 0.f;
    const float cb = r1 < a.R ? bf2f(a.x[static_cast<long long>(r1) * D]) : 0.f;
    const float cc = (has2 && r2 < a.R) ? bf2f(a.x[static_cast<long long>(r2) * D]) : 0.f;
    float s[6];
    ln_half_sums<NCH>(xa, ca, s[0], s[1]);
    ln_half_sums<NCH>(xb, cb, s[2], s[3]);
    ln_half_sums<NCH>(xc, cc, s[4], s[5]);
  #pragma unroll
    for (int o = 16; o > 0; o >>= 1)
  #pragma unroll
      for (int i = 0; i < 6; ++i) s[i] += __shfl_xor_sync(0xffffffffu, s[i], o);
    // exchange with the peer
    const uint32_t peer = half ^ 1;
    if (lane == 0) {
      st_cluster_v2(cluster_map(&tl->xstat[r0][0], peer), s[0], s[1]);
      st_cluster_v2(cluster_map(&tl->xstat[r1][0], peer), s[2], s[3]);
      if (has2) st_cluster_v2(cluster_map(&tl->xstat[r2][0], peer), s[4], s[5]);
      mbar_arrive_cluster(cluster_map(&tl->xstat_bar, peer));
    }
    const bool ok = mbar_wait_cl(a, &tl->xstat_bar, parity, kErrWaitFull);
    if (!ok) return false;
    const float2 pa = *reinterpret_cast<const float2*>(&tl->xstat[r0][0]);
    const float2 pb = *reinterpret_cast<const float2*>(&tl->xstat[r1][0]);
    const float2 pc = has2 ? *reinterpret_cast<const float2*>(&tl->xstat[r2][0]) : make_float2(0.f, 0.f);
    // mean = c + S1 / D, var = S2 / D - (S1 / D)^2; n = x * rstd - mean * rstd
    auto stats = [&](float c, float s1, float s2, int r, float& rs, float& b) {
      const float m1 = s1 / D;
      const float var = fmaxf(s2 / D - m1 * m1, 0.f);
      rs = r < a.R ? rsqrtf(var + a.eps) : 0.f;
      b = -(c + m1) * rs;
    };
    stats(ca, s[0] + pa.x, s[1] + pa.y, r0, ra, ba);
    stats(cb, s[2] + pb.x, s[3] + pb.y, r1, rb, bb);
    stats(cc, s[4] + pc.x, s[5] + pc.y, has2 ? r2 : kFusedRows, rc, bc);
  }
  if (mode == 0) {
    // AdaLN: bf16(n) * bf16(1 + scale) + bf16(shift), packed bf16 pairs
    const uint4* cm = reinterpret_cast<const uint4*>(stg + kStgLnConst) + half * (DH / 8);
    const uint4* cadd = reinterpret_cast<const uint4*>(stg + kStgLnConst) + D / 8 + half * (DH / 8);
#pragma unroll
    for (int u = 0; u < NCH; ++u) {
      const int ch = lane + 32 * u;  // chunk within this half: local K block ch >> 3
      const uint4 m4 = cm[ch], a4 = cadd[ch];
      const uint32_t mw[4] = {m4.x, m4.y, m4.z, m4.w}, aw[4] = {a4.x, a4.y, a4.z, a4.w};
      float fa[8], fb[8], fc[8];
      bf8_unpack(xa[u], fa);
      bf8_unpack(xb[u], fb);
      bf8_unpack(xc[u], fc);
      uint32_t oa[4], ob[4], oc[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 mv = *reinterpret_cast<const __nv_bfloat162*>(&mw[e]);
        const __nv_bfloat162 av = *reinterpret_cast<const __nv_bfloat162*>(&aw[e]);
        const int i0 = 2 * e;
        __nv_bfloat162 na = __floats2bfloat162_rn(fmaf(fa[i0], ra, ba), fmaf(fa[i0 + 1], ra, ba));
        __nv_bfloat162 nb = __floats2bfloat162_rn(fmaf(fb[i0], rb, bb), fmaf(fb[i0 + 1], rb, bb));
        __nv_bfloat162 nc = __floats2bfloat162_rn(fmaf(fc[i0], rc, bc), fmaf(fc[i0 + 1], rc, bc));
        // the reference's modulate on bf16 tensors: bf16(bf16(n * (1 + scale)) + shift)
        na = __hadd2(__hmul2(na, mv), av);
        nb = __hadd2(__hmul2(nb, mv), av);
        nc = __hadd2(__hmul2(nc, mv), av);
        oa[e] = *reinterpret_cast<uint32_t*>(&na);
        ob[e] = *reinterpret_cast<uint32_t*>(&nb);
        oc[e] = *reinterpret_cast<uint32_t*>(&nc);
      }
      stage_chunk(stg, ch >> 3, r0, ch & 7, r0 < a.R ? make_uint4(oa[0], oa[1], oa[2], oa[3]) : make_uint4(0, 0, 0, 0));
      stage_chunk(stg, ch >> 3, r1, ch & 7, r1 < a.R ? make_uint4(ob[0], ob[1], ob[2], ob[3]) : make_uint4(0, 0, 0, 0));
      if (has2)
        stage_chunk(stg, ch >> 3, r2, ch & 7, r2 < a.R ? make_uint4(oc[0], oc[1], oc[2], oc[3]) : make_uint4(0, 0, 0, 0));
    }
  } else {
    // affine norm3 (fp32 weight and bias, one rounding at the store)
    const float4* cm = reinterpret_cast<const float4*>(stg + kStgLnConst) + half * (DH / 4);
    const float4* cadd = reinterpret_cast<const float4*>(stg + kStgLnConst) + D / 4 + half * (DH / 4);
#pragma unroll
    for (int u = 0; u < NCH; ++u) {
      const int ch = lane + 32 * u;
      const float4 m0 = cm[2 * ch], m1 = cm[2 * ch + 1], a0 = cadd[2 * ch], a1 = cadd[2 * ch + 1];
      const float mv[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float fa[8], fb[8], fc[8];
      bf8_unpack(xa[u], fa);
      bf8_unpack(xb[u], fb);
      bf8_unpack(xc[u], fc);
      float oa[8], ob[8], oc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        oa[e] = fmaf(fa[e], ra, ba) * mv[e] + av[e];
        ob[e] = fmaf(fb[e], rb, bb) * mv[e] + av[e];
        oc[e] = fmaf(fc[e], rc, bc) * mv[e] + av[e];
      }
      stage_chunk(stg, ch >> 3, r0, ch & 7, r0 < a.R ? pack8(oa) : make_uint4(0, 0, 0, 0));
      stage_chunk(stg, ch >> 3, r1, ch & 7, r1 < a.R ? pack8(ob) : make_uint4(0, 0, 0, 0));
      if (has2) stage_chunk(stg, ch >> 3, r2, ch & 7, r2 < a.R ? pack8(oc) : make_uint4(0, 0, 0, 0));
    }
  }
  return true;
}

__device__ bool stage_layernorm_pair(const FusedArgs& a, uint8_t* stg, FusedSmemTail* tl, int mode, int half,
                                     uint32_t parity, const double* st) {
  return (a.D >> 9) == 1 ? stage_layernorm_pair_t<1>(a, stg, tl, mode, half, parity, st)
                         : stage_layernorm_pair_t<2>(a, stg, tl, mode, half, parity, st);
}

// Copy columns [col0, col0 + 64 * nkb) of a bf16 [R, ld] buffer into the
// staging (nkb <= 8: at most 6 16-byte chunks per worker thread).  All loads
// are issued before the first shared-memory store so they overlap.
__device__ void stage_copy(const FusedArgs& a, uint8_t* stg, const __nv_bfloat16* src, long long ld,
                           int col0, int nkb) {
  constexpr int kMaxPer = (kFusedRows * 64 + kFusedWorkers - 1) / kFusedWorkers;  // 8 K blocks
  const int per_row = nkb * 8;
  const int total = kFusedRows * per_row;
  uint4 v[kMaxPer];
#pragma unroll
  for (int u = 0; u < kMaxPer; ++u) {
    const int idx = threadIdx.x - 32 + u * kFusedWorkers;
    const int r = idx / per_row, ch = idx % per_row;
    v[u] = make_uint4(0, 0, 0, 0);
    if (idx < total && r < a.R) v[u] = __ldcg(reinterpret_cast<const uint4*>(src + r * ld + col0 + ch * 8));
  }
#pragma unroll
  for (int u = 0; u < kMaxPer; ++u) {
    const int idx = threadIdx.x - 32 + u * kFusedWorkers;
    const int r = idx / per_row, ch = idx % per_row;
    if (idx < total) stage_chunk(stg, ch >> 3, r, ch & 7, v[u]);
  }
}

// ------------------------------------------------------------- epilogues
// Per-feature constants of an epilogue, loaded before the accumulator wait so
// their latency overlaps the MMA: bias, the RMSNorm weight (qkv q/k, cross-q)
// or the residual gate (o, ffn.2); plus the RoPE (cos, sin) of every token for
// the q/k features.
// The epilogue runs on 8 warps: warps 2..5 take the tokens 0..15 and warps
// 6..9 the tokens 16..31 of the TMEM lane quarter warp % 4 (one output
// feature per lane), so two warps share every scheduler.
constexpr int kEpiTokens = kFusedRows / 2;

struct EpiConst {
  float bias, mul;
  const float2* rope;  // [16 tokens][16 pairs] of this warp's features (shared memory)
};

__device__ __forceinline__ void epi_load(const FusedArgs& a, uint8_t* stg, int p, int step, int l,
                                         const FItem& it, int f, int t0, EpiConst& c) {
  const int HD = a.HD;
  c.mul = 1.f;
  switch (p) {
    case kFQkv: {
      const int type = f / HD, ff = f % HD;
      c.bias = bf2f(a.qkv_b[static_cast<long long>(l) * 3 * HD + f]);
      if (type == 2) return;
      c.mul = bf2f((type == 0 ? a.norm_q : a.norm_k)[static_cast<long long>(l) * HD + ff]);
      // this warp's 16 rotation pairs (lanes 2i, 2i+1 share pair i) for its
      // tokens -> shared memory
      const int lane = threadIdx.x & 31, q = (threadIdx.x >> 5) & 3;
      const int pi0 = (ff % a.hd - lane) >> 1;
      float2* sr = reinterpret_cast<float2*>(stg + kStgRope) + (q * kFusedRows + t0) * 16;
      float2 cs[kEpiTokens * 16 / 32];
#pragma unroll
      for (int k = 0; k < kEpiTokens * 16 / 32; ++k) {
        const int idx = lane + 32 * k, j = t0 + (idx >> 4), pl = idx & 15;
        cs[k] = j < a.R ? a.rope[(j % a.Sa) * (a.hd >> 1) + pi0 + pl] : make_float2(1.f, 0.f);
      }
#pragma unroll
      for (int k = 0; k < kEpiTokens * 16 / 32; ++k) sr[lane + 32 * k] = cs[k];
      __syncwarp();
      c.rope = sr;
      return;
    }
    case kFO:
    case kFCo:
    case kFFfn2: {
      // the tile's last split item adds the bias to the sum of the split
      // partials and applies the residual gate (residual_finalize)
      c.bias = 0.f;
      return;
    }
    case kFCq:
      c.bias = bf2f(a.cq_b[static_cast<long long>(l) * HD + f]);
      c.mul = bf2f(a.cnorm_q[static_cast<long long>(l) * HD + f]);
      return;
    default:
      c.bias = bf2f(a.ffn0_b[static_cast<long long>(l) * a.F + f]);
      return;
  }
}

// Per-token sums over the 32 lanes for the 16 tokens of a warp: after the
// recursive halving (15 shuffles) lanes l and l ^ 16 hold the half sums of
// token l & 15, one more exchange completes them.
__device__ __forceinline__ float warp_transpose_sum16(float (&v)[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
    const bool upper = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = upper ? v[i] : v[i + w];
      const float keep = upper ? v[i + w] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 16);
}

// Epilogue of one output feature f (this lane) for the tokens t0 .. t0 + 15.
__device__ __forceinline__ void gemm_epilogue(const FusedArgs& a, int p, int step, int l, const FItem& it, int f,
                                              int t0, const EpiConst& c, float (&v)[kEpiTokens]) {
  const int lane = threadIdx.x & 31;
  const int R = a.R, D = a.D, HD = a.HD;
  switch (p) {
    case kFQkv: {
      const int type = f / HD, ff = f % HD;
      if (type == 2) {
#pragma unroll
        for (int j = 0; j < kEpiTokens; ++j)
          if (t0 + j < R) a.va[(t0 + j) * HD + ff] = f2bf(rbf(v[j] + c.bias));
        return;
      }
      double* ssq = a.ssq + ((static_cast<long long>(step) * a.L + l) * 3 + type) * kFusedRows;
      __nv_bfloat16* dst = type == 0 ? a.q : a.ka;
#pragma unroll
      for (int j = 0; j < kEpiTokens; ++j) {
        const float y = rbf(v[j] + c.bias);
        v[j] = y * y;
        const float z = rbf(y * c.mul);
        const float pz = __shfl_xor_sync(0xffffffffu, z, 1);
        const float2 cs = c.rope[j * 16 + (lane >> 1)];
        const float o = (lane & 1) ? (pz * cs.y + z * cs.x) : (z * cs.x - pz * cs.y);
        if (t0 + j < R) dst[(t0 + j) * HD + ff] = f2bf(o);
      }
      const float mine = warp_transpose_sum16(v);  // lanes l, l ^ 16: token t0 + (l & 15)
      // fp64: the sum of the fp32 warp partials is exact, whatever order they
      // arrive in (the launch is deterministic)
      if (lane < 16 && t0 + lane < R) atomicAdd(ssq + t0 + lane, static_cast<double>(mine));
      return;
    }
    case kFO:
    case kFCo:
    case kFFfn2: {
      // this split item's partial tile -> its slot ([split][tile][token][128]
      // fp32, one 128-byte row per warp and token); the last split item of
      // the tile completes the residual add (residual_finalize)
      float* slot = a.slots + ((static_cast<long long>(it.sub) * (D / 128) + it.n) * kFusedRows) * 128 + (f & 127);
#pragma unroll
      for (int j = 0; j < kEpiTokens; ++j)
        if (t0 + j < R) slot[(t0 + j) * 128] = v[j];
      return;
    }
    case kFCq: {
      double* ssq = a.ssq + ((static_cast<long long>(step) * a.L + l) * 3 + 2) * kFusedRows;
#pragma unroll
      for (int j = 0; j < kEpiTokens; ++j) {
        const float y = rbf(v[j] + c.bias);
        v[j] = y * y;
        if (t0 + j < R) a.qc[(t0 + j) * HD + f] = f2bf(rbf(y * c.mul));
      }
      const float mine = warp_transpose_sum16(v);
      if (lane < 16 && t0 + lane < R) atomicAdd(ssq + t0 + lane, static_cast<double>(mine));
      return;
    }
    default:  // ffn.0 + GELU(tanh)
#pragma unroll
      for (int j = 0; j < kEpiTokens; ++j)
        if (t0 + j < R) a.fh[(t0 + j) * a.F + f] = f2bf(gelu_tanh(rbf(v[j] + c.bias)));
      return;
  }
}

// Residual GEMMs (o, cross-o, ffn.2): after the 8 epilogue warps of a split
// item have stored its partial tile, one thread publishes it (release
// increment of the tile's counter, cumulative over the CTA's stores through
// the barrier) and waits (bounded) until every split item of the tile has;
// the counters only grow within a launch (target = splits x uses so far).
// Then each split item completes its share of the tile's tokens: the split
// partials summed in split order (deterministic) plus the bias, and the
// residual add as the reference's bf16 tensors (mot.py:130-149):
// x = bf16(x + bf16(gate * bf16(o))).
__device__ __forceinline__ void bar_epilogue() {
  asm volatile("barrier.sync 2, 256;" ::: "memory");
}
// The [32][2] row sums written by residual GEMM p of (step, block l).
__device__ __forceinline__ double* ln_stat_slot(const FusedArgs& a, int p, int step, int l) {
  const int k = p == kFO ? 0 : (p == kFCo ? 1 : 2);
  return a.lnstat + ((static_cast<long long>(step) * a.L + l) * 3 + k) * kFusedRows * 2;
}
constexpr int kFinMaxSplits = 8;  // split partials held in flight per thread
__device__ void residual_finalize(const FusedArgs& a, FusedSmemTail* tl, int p, int step, int l, const FItem& it) {
  const int splits = f_count(a, p) / (a.D / 128);
  // row sums for the LayerNorm that follows (cross-q after o, ffn.0 after
  // cross-o, the next block's qkv after ffn.2; none after the last block)
  double* st = (p == kFFfn2 && l == a.L - 1) ? nullptr : ln_stat_slot(a, p, step, l);
  bar_epilogue();
  if (threadIdx.x == 64) {
    unsigned* ctr = a.tile_ctr + (p == kFO ? 0 : (p == kFCo ? 1 : 2)) * (kFusedMaxD / 128) + it.n;
    red_release_add(ctr, 1u);
    const unsigned target = static_cast<unsigned>(splits) * static_cast<unsigned>(step * a.L + l + 1);
    tl->fin = poll_ge(a, ctr, target, tl) ? 1 : 0;
  }
  bar_epilogue();
  if (!tl->fin) return;
  // this item's tokens, 4 consecutive features per thread and step
  const int tb = it.sub * kFusedRows / splits, te = min(a.R, (it.sub + 1) * kFusedRows / splits);
  const long long sstride = static_cast<long long>(a.D / 128) * kFusedRows * 128;  // floats per split
  const __nv_bfloat16* bptr = (p == kFO ? a.o_b : (p == kFCo ? a.co_b : a.ffn2_b)) + static_cast<long long>(l) * a.D;
  const int cg = p == kFO ? 2 : 5;  // gate_msa (o) / gate_mlp (ffn.2); cross-o has no gate
  for (int idx = threadIdx.x - 64; idx < (te - tb) * 32; idx += 256) {
    const int tok = tb + (idx >> 5), fl = (idx & 31) * 4, f0 = it.n * 128 + fl;
    const long long xoff = static_cast<long long>(tok) * a.D + f0;
    const float* slot = a.slots + (static_cast<long long>(it.n) * kFusedRows + tok) * 128 + fl;
    // every load in flight before the first use
    const uint2 xr = __ldcg(reinterpret_cast<const uint2*>(a.x + xoff));
    float4 part[kFinMaxSplits];
#pragma unroll
    for (int sp = 0; sp < kFinMaxSplits; ++sp)
      part[sp] = sp < splits ? __ldcg(reinterpret_cast<const float4*>(slot + sp * sstride)) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = kFinMaxSplits; sp < splits; ++sp) {  // more splits than held in flight (F > 4096)
      const float4 q = __ldcg(reinterpret_cast<const float4*>(slot + sp * sstride));
      part[kFinMaxSplits - 1] = make_float4(part[kFinMaxSplits - 1].x + q.x, part[kFinMaxSplits - 1].y + q.y,
                                            part[kFinMaxSplits - 1].z + q.z, part[kFinMaxSplits - 1].w + q.w);
    }
    const uint2 br = *reinterpret_cast<const uint2*>(bptr + f0);
    float g[4] = {1.f, 1.f, 1.f, 1.f};
    if (p != kFCo) {
      const float4 tm = *reinterpret_cast<const float4*>(a.tmod + static_cast<long long>(step) * 6 * a.D + cg * a.D + f0);
      const uint2 mr = *reinterpret_cast<const uint2*>(a.modulation + (static_cast<long long>(l) * 6 + cg) * a.D + f0);
      const float tv[4] = {tm.x, tm.y, tm.z, tm.w};
      const __nv_bfloat162 m0 = *reinterpret_cast<const __nv_bfloat162*>(&mr.x);
      const __nv_bfloat162 m1 = *reinterpret_cast<const __nv_bfloat162*>(&mr.y);
      const float mv[4] = {__low2float(m0), __high2float(m0), __low2float(m1), __high2float(m1)};
#pragma unroll
      for (int e = 0; e < 4; ++e) g[e] = rbf(rbf(tv[e]) + mv[e]);
    }
    float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int sp = 0; sp < kFinMaxSplits; ++sp) {  // split order
      sum[0] += part[sp].x;
      sum[1] += part[sp].y;
      sum[2] += part[sp].z;
      sum[3] += part[sp].w;
    }
    const __nv_bfloat162 x0 = *reinterpret_cast<const __nv_bfloat162*>(&xr.x);
    const __nv_bfloat162 x1 = *reinterpret_cast<const __nv_bfloat162*>(&xr.y);
    const __nv_bfloat162 b0 = *reinterpret_cast<const __nv_bfloat162*>(&br.x);
    const __nv_bfloat162 b1 = *reinterpret_cast<const __nv_bfloat162*>(&br.y);
    const float xv[4] = {__low2float(x0), __high2float(x0), __low2float(x1), __high2float(x1)};
    const float bv[4] = {__low2float(b0), __high2float(b0), __low2float(b1), __high2float(b1)};
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = xv[e] + rbf(g[e] * rbf(sum[e] + bv[e]));
    *reinterpret_cast<uint2*>(a.x + xoff) = make_uint2(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]));
    if (st != nullptr) {
      // the next LayerNorm's row sums: this warp holds the token's 128 features of
      // the tile (lane = 4 features), summed in a fixed shuffle order, then one
      // fp64 add per tile (sums of fp32 values: exact in fp64, order-free)
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float xb = rbf(o[e]);
        s1 += xb;
        s2 += xb * xb;
      }
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, m);
        s2 += __shfl_xor_sync(0xffffffffu, s2, m);
      }
      if ((threadIdx.x & 31) == 0) {
        atomicAdd(st + 2 * tok, static_cast<double>(s1));
        atomicAdd(st + 2 * tok + 1, static_cast<double>(s2));
      }
    }
  }
}

// One GEMM work item on the workers (the weight tiles arrive through the ring).
// Pair items (qkv, cross-q, ffn.0) run on both CTAs of a cluster (`half` =
// cluster rank): each stages and multiplies its K half, then the epilogue
// warps of the TMEM lane quarters the peer owns (rank 0 owns quarters 0-1 =
// output rows 0-63 of the tile, rank 1 quarters 2-3) send their partial sums
// to the peer (kStgXacc, [token][64] fp32) and the owners add them and finish.
__device__ void gemm_item(const FusedArgs& a, uint8_t* ring, uint8_t* stg, FusedSmemTail* tl,
                          int p, int step, int l, const FItem& it, uint32_t& ring_it,
                          uint32_t& items_done, uint32_t& pair_done, uint32_t& xstat_done) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool pair = f_pair(p);
  const int half = pair ? static_cast<int>(cluster_ctarank()) : 0;
  const uint32_t pparity = pair_done & 1;
  // 1. B operand
  switch (p) {
    case kFQkv:
    case kFCq:
    case kFFfn0: {
      // the row sums of the residual GEMM before (none for block 0's qkv: the
      // step's encoder wrote its rows), else the pair exchanges half-row sums
      const double* st = p == kFCq ? ln_stat_slot(a, kFO, step, l)
                                   : (p == kFFfn0 ? ln_stat_slot(a, kFCo, step, l)
                                                  : (l > 0 ? ln_stat_slot(a, kFFfn2, step, l - 1) : nullptr));
      if (!stage_layernorm_pair(a, stg, tl, p == kFCq ? 1 : 0, half, xstat_done & 1, st)) tl->abort = 1;
      if (st == nullptr) ++xstat_done;
      break;
    }
    case kFO: stage_copy(a, stg, a.ao, a.HD, it.kb0 * 64, it.nkb); break;
    case kFCo: stage_copy(a, stg, a.ci, a.HD, it.kb0 * 64, it.nkb); break;
    default: stage_copy(a, stg, a.fh, a.F, it.kb0 * 64, it.nkb); break;
  }
  fence_async_smem();
  bar_workers();
  // pair: expect the peer's partial accumulators (8 KB bulk copy) on xacc_bar
  if (pair && threadIdx.x == 32) mbar_arrive_expect_tx(&tl->xacc_bar, kXaccBytes);
  // 2. MMA: kFusedIssuers issuing threads (lane 0 of warps 1, 6, 7, 8; issuer
  // j takes the K blocks k = j mod kFusedIssuers) into separate TMEM
  // accumulators summed by the epilogue.  A single thread's tcgen05.mma issue
  // rate (with its barrier wait and commit per K block) bounds a skinny
  // (N = 32) GEMM; independent issuers multiply it.  Descriptors advance in
  // their address field (address >> 4): kATile per ring slot, kBBlock per B K
  // block.
  const int j = warp == 1 ? 0 : warp - (kFusedIssuer1 - 1);
  if ((warp == 1 || (warp >= kFusedIssuer1 && warp < kFusedIssuer1 + kFusedIssuers - 1)) && lane == 0) {
    const uint32_t idesc = umma_idesc_bf16(128, kFusedRows);
    const uint64_t da0 = umma_desc_sw128(ring), db0 = umma_desc_sw128(stg);
    const uint32_t acc = tl->tmem + j * kFusedRows;
    bool ok = tl->abort == 0;
    for (int k = j; k < it.nkb && ok; k += kFusedIssuers) {
      const uint32_t r = ring_it + k, s = r % kFusedRing;
      ok = mbar_wait(&tl->full[s], (r / kFusedRing) & 1, a.status, kErrWaitFull);
      if (!ok) break;
      tc_fence_after();
      const uint64_t da = da0 + static_cast<uint64_t>(s * (kATile >> 4));
      const uint64_t db = db0 + static_cast<uint64_t>(k * (kBBlock >> 4));
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16_ss(acc, da + 2 * kk, db + 2 * kk, idesc, (k > j || kk != 0) ? 1u : 0u);
      umma_commit(&tl->empty[s]);
    }
    if (!ok) tl->abort = 1;
    umma_commit(&tl->accum);  // kFusedIssuers arrivals complete the phase
  }
  const int nkb = it.nkb;
  ring_it += nkb;
  // 3. epilogue (warps 2..9: TMEM lane quarter warp % 4, tokens t0 .. t0 + 15)
  if (warp >= 2 && warp <= 9) {
    const int q = warp & 3, t0 = warp >= 6 ? kEpiTokens : 0;
    const int f = it.n * 128 + q * 32 + lane;
    const bool keep = !pair || ((q >> 1) == half);  // pair: this CTA finishes its half of the rows
    EpiConst c;
    if (keep) epi_load(a, stg, p, step, l, it, f, t0, c);
    const bool ok = mbar_wait(&tl->accum, items_done & 1, a.status, kErrWaitAccum);
    tc_fence_after();
    if (!ok) tl->abort = 1;
    // the issuers' accumulators (an issuer without K blocks left its
    // accumulator stale: selected out), one TMEM wait
    float v[kEpiTokens];
    const uint32_t tq = tl->tmem + (static_cast<uint32_t>(q * 32) << 16) + t0;
    {
      uint32_t r[kFusedIssuers][16];
#pragma unroll
      for (int jj = 0; jj < kFusedIssuers; ++jj) tmem_ld16_nowait(tq + jj * kFusedRows, r[jj]);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < kEpiTokens; ++i) {
        float t = __uint_as_float(r[0][i]);
#pragma unroll
        for (int jj = 1; jj < kFusedIssuers; ++jj) t += jj < nkb ? __uint_as_float(r[jj][i]) : 0.f;
        v[i] = t;
      }
    }
    if (pair) {
      const int fl = (q & 1) * 32 + lane;
      if (!keep) {
        // partial sums of the peer's rows -> this CTA's send buffer; the
        // first sending warp then moves all 8 KB to the peer in one bulk copy
        float* xsend = reinterpret_cast<float*>(stg + kStgXsend);  // [token][64]
#pragma unroll
        for (int jj = 0; jj < kEpiTokens; ++jj) xsend[(t0 + jj) * 64 + fl] = v[jj];
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tl->xsend_bar);
        const int first_give = half == 0 ? 2 : 4;  // lowest warp of the sending quarters
        if (warp == first_give && lane == 0) {
          if (!mbar_wait(&tl->xsend_bar, pparity, a.status, kErrWaitAccum)) {
            tl->abort = 1;
          } else {
            bulk_copy_to_peer(cluster_map(stg + kStgXacc, half ^ 1), xsend, kXaccBytes,
                              cluster_map(&tl->xacc_bar, half ^ 1));
            bulk_wait_read();  // the send buffer is reused by the next pair item
          }
        }
      } else {
        const float* xacc = reinterpret_cast<const float*>(stg + kStgXacc);  // [token][64]
        if (!mbar_wait_cl(a, &tl->xacc_bar, pparity, kErrWaitAccum)) tl->abort = 1;
#pragma unroll
        for (int jj = 0; jj < kEpiTokens; ++jj) v[jj] += xacc[(t0 + jj) * 64 + fl];
      }
    }
    if (keep && ok && !tl->abort) gemm_epilogue(a, p, step, l, it, f, t0, c, v);
    if (p == kFO || p == kFCo || p == kFFfn2) residual_finalize(a, tl, p, step, l, it);
    tc_fence_before();
  }
  ++items_done;
  if (pair) ++pair_done;
  bar_workers();
}

// --------------------------------------------------------------- attention
// One (head, key split) of an attention over [source1 (Sv1 keys) ; source2 (S2
// keys)] for the R query rows: 8 worker warps = 2 query groups x 4 blocks of
// 64 keys.  Source 2 keys are scaled per key (RMSNorm of the fresh k); q rows
// by qscale.  Writes either the final output (nsplit == 1) or a split partial
// merged by the last-arriving CTA of the head.
struct AttnItem {
  const __nv_bfloat16* k1;  // source 1 rows: k1 + j * ts1 (head offset applied)
  const __nv_bfloat16* v1;
  long long ts1;
  int S1;
  const __nv_bfloat16* k2;  // source 2 rows: k2 + j * ts2
  const __nv_bfloat16* v2;
  long long ts2;
  int S2;
  const double* kscale2;    // [S2] sum of squares of the fresh keys (null: 1)
  const __nv_bfloat16* qp;  // q rows: qp + r * qts (head offset applied)
  long long qts;
  const double* qscale;     // [R] sum of squares of q rows (null: 1)
  const uint8_t* mask2d;    // [R, S1 + S2] (row stride mrs) or null
  long long mrs;
  const uint8_t* key_mask;  // [S1 + S2] or null
  int k0, k1end;            // key range of this split
  __nv_bfloat16* out;       // final output rows: out + r * ots (head offset applied)
  long long ots;
  float* part;              // this split's partial [32][66] (nsplit > 1)
  float* part_head;         // all splits of the head
  unsigned* counter;        // arrival counter of the head
  int nsplit;
};

// Staging of an attention item (1024-byte aligned): V / K [256 keys][64] each
// and the q rows replicated four times [4 x 32][64], all in the 128-byte
// swizzle the tcgen05 descriptors read (16-byte chunk c of row r at r * 128 +
// (c ^ (r & 7)) * 16), then the attend bytes [32][256], the key mask [256] and
// the per-key logit factors [256] fp32.
struct AttnSmem {
  uint8_t *sK, *sV, *sQ;
  uint8_t *sM, *sKm;
  float* sKsc;
};
__device__ __forceinline__ AttnSmem attn_smem(uint8_t* stg) {
  AttnSmem m;
  m.sV = stg;
  m.sK = stg + 256 * 128;
  m.sQ = stg + 2 * 256 * 128;
  m.sM = m.sQ + 4 * kFusedRows * 128;
  m.sKm = m.sM + kFusedRows * 256;
  m.sKsc = reinterpret_cast<float*>(m.sKm + 256);
  return m;
}
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}
static_assert(2 * 256 * 128 + 4 * kFusedRows * 128 + kFusedRows * 256 + 256 + 256 * 4 <= kFusedStaging,
              "attention staging");
static_assert(kFusedRing * kATile + kFusedStaging + sizeof(FusedSmemTail) + 1024 <= 232448,
              "fused shared memory within the 227 KB per-CTA limit");
// TMEM of the attention items: S [128 lanes][256 keys] fp32, then softmax warp
// w's O partial [128][64] fp32 over its own S columns [64 w, 64 w + 64); P
// [128][256] as bf16 pairs (the GEMM accumulators use columns [0, 128) in
// their own phases)
constexpr uint32_t kAttnColS = 0, kAttnColP = 256;
constexpr uint32_t kFusedTmemCols = 512;
static_assert(kFusedMaxSplits * (kFusedRows * 64 + kFusedRows * 2) * 4 + (kFusedMaxSplits + 1) * kFusedRows * 4 <=
                  kFusedStaging,
              "split partials of a head fit the staging");

// The part of an item that no earlier phase of the launch writes: the source
// 1 rows (video cache or context K / V), the attend bytes and the key mask.
// A CTA issues it for its next attention item at the end of the phase before
// (one cp.async group), so the HBM reads overlap that phase and its barrier.
__device__ void attn_stage_const(const FusedArgs& a, uint8_t* stg, const AttnItem& t) {
  const AttnSmem m = attn_smem(stg);
  const int nkeys = t.k1end - t.k0;
  for (int idx = threadIdx.x - 32; idx < 256 * 8; idx += kFusedWorkers) {
    const int r = idx >> 3, c = idx & 7;
    const int j = t.k0 + r;
    if (r < nkeys && j >= t.S1) continue;  // a fresh key: staged after the barrier
    const bool valid = r < nkeys;            // keys past the split read as zeros
    cp_async16(m.sK + sw128_off(r, c), valid ? t.k1 + j * t.ts1 + c * 8 : a.q, valid);
    cp_async16(m.sV + sw128_off(r, c), valid ? t.v1 + j * t.ts1 + c * 8 : a.q, valid);
  }
  if (t.mask2d != nullptr) {
    if (t.mrs % 16 == 0 && (reinterpret_cast<uintptr_t>(t.mask2d) & 15) == 0 && t.k0 % 16 == 0) {
      for (int idx = threadIdx.x - 32; idx < kFusedRows * 16; idx += kFusedWorkers) {
        const int r = idx >> 4, c = idx & 15;
        const int j = t.k0 + 16 * c;
        int n = t.k1end - j;
        n = n < 0 ? 0 : (n > 16 ? 16 : n);
        if (r >= a.R) n = 0;
        const uint8_t* src = n > 0 ? t.mask2d + r * t.mrs + j : t.mask2d;
        asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(m.sM + r * 256 + 16 * c)),
                     "l"(src), "r"(n)
                     : "memory");
      }
    } else {
      for (int idx = threadIdx.x - 32; idx < kFusedRows * 256; idx += kFusedWorkers) {
        const int r = idx >> 8, jj = idx & 255;
        m.sM[idx] = (jj < nkeys && r < a.R) ? t.mask2d[r * t.mrs + t.k0 + jj] : 0;
      }
    }
  }
  for (int jj = threadIdx.x - 32; jj < 256; jj += kFusedWorkers)
    m.sKm[jj] = jj < nkeys ? (t.key_mask != nullptr ? t.key_mask[t.k0 + jj] : 1) : 0;
  cp_async_commit();
}

__device__ void attention_item(const FusedArgs& a, uint8_t* stg, FusedSmemTail* tl, const AttnItem& t,
                               bool prefetched, uint32_t& attn_it, uint32_t& pv_it) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const AttnSmem m = attn_smem(stg);
  const int nkeys = t.k1end - t.k0;
  // the q chunk and the q-row scale of this thread, loaded first so their L2
  // latency overlaps the staging below (rows >= R stay zero)
  const int qi = threadIdx.x - 32, qr = qi >> 3, qc = qi & 7;
  const bool qthread = qi < kFusedRows * 8;
  uint4 qraw = make_uint4(0u, 0u, 0u, 0u);
  double qss = 0.0;
  if (qthread && qr < a.R) {
    qraw = __ldcg(reinterpret_cast<const uint4*>(t.qp + qr * t.qts + qc * 8));
    if (t.qscale != nullptr) qss = __ldcg(t.qscale + qr);
  }
  if (!prefetched) attn_stage_const(a, stg, t);
  // fresh keys (source 2): written by the phase before
  for (int idx = threadIdx.x - 32; idx < 256 * 8; idx += kFusedWorkers) {
    const int r = idx >> 3, c = idx & 7;
    const int j = t.k0 + r;
    if (r >= nkeys || j < t.S1) continue;
    cp_async16(m.sK + sw128_off(r, c), t.k2 + (j - t.S1) * t.ts2 + c * 8, true);
    cp_async16(m.sV + sw128_off(r, c), t.v2 + (j - t.S1) * t.ts2 + c * 8, true);
  }
  cp_async_commit();
  // q rows scaled by their RMSNorm scale and rounded to bf16, written four times
  // (TMEM lane quarter w of S reads rows 32 w .. 32 w + 31)
  if (qthread) {
    const float sc = (t.qscale != nullptr && qr < a.R) ? rsqrtf(static_cast<float>(qss) / a.HD + a.eps) : 1.f;
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&qraw);
    const uint4 u = make_uint4(pack_bf16(__low2float(h2[0]) * sc, __high2float(h2[0]) * sc),
                               pack_bf16(__low2float(h2[1]) * sc, __high2float(h2[1]) * sc),
                               pack_bf16(__low2float(h2[2]) * sc, __high2float(h2[2]) * sc),
                               pack_bf16(__low2float(h2[3]) * sc, __high2float(h2[3]) * sc));
#pragma unroll
    for (int rep = 0; rep < 4; ++rep) *reinterpret_cast<uint4*>(m.sQ + sw128_off(rep * kFusedRows + qr, qc)) = u;
  }
  cp_async_wait<0>();
  fence_async_smem();  // the staged K / V / Q (generic-proxy writes) before the MMAs read them
  tc_fence_before();
  bar_workers();
  tc_fence_after();

  // S = Q K^T: M = 128 (four copies of the 32 queries), N = the item's keys
  // rounded up to 16, K = 64
  const uint32_t par = attn_it & 1;
  ++attn_it;
  const int nk16 = (nkeys + 15) & ~15;
  if (threadIdx.x == 32) {
    const uint32_t idesc = umma_idesc_bf16(128, nk16);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      umma_bf16_ss(tl->tmem + kAttnColS, umma_desc_sw128(m.sQ) + 2 * kk, umma_desc_sw128(m.sK) + 2 * kk, idesc,
                   kk > 0 ? 1u : 0u);
    umma_commit(&tl->attn_s);
  }
  // softmax warps 4..7: warp w owns keys [64 w, 64 w + 64) of the item for every
  // query (its TMEM lane quarter holds all 32 query rows).  It writes its P
  // columns [32 w, 32 w + 32), issues P.V over its own keys into its own S
  // columns (no other warp reads them) and reads back its lanes' O rows: the
  // four warps never wait for one another.  Rows of the other lane quarters in
  // that product are zero or stale and are not read.
  // quarter partials O [4][32][kCombRow] (padded rows: conflict-free stores) and
  // (m, l) [4][32][2] over K and Q, which only the S MMA reads: a warp writes
  // them after S is complete (V stays: other warps' P.V may still read it)
  constexpr int kCombRow = 64 + 4;
  static_assert(4 * kFusedRows * (kCombRow + 2) * 4 <= 256 * 128 + 4 * kFusedRows * 128, "quarter partials");
  float* comb = reinterpret_cast<float*>(m.sK);
  float* cml = comb + 4 * kFusedRows * kCombRow;
  const bool smx = warp >= 4 && warp < 8;
  const int wq = warp - 4, q = lane;
  const uint32_t lane_addr = tl->tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  bool ok = true;
  if (smx && 64 * wq < nkeys) {
    // per-key logit factor of the warp's keys: scale_log2 x the RMSNorm scale of
    // a fresh key, 0 for a key outside the split or masked out by the key mask
    float* kfw = m.sKsc + 64 * wq;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int jj = 64 * wq + 32 * h + lane, j = t.k0 + jj;
      float ks = 1.f;
      if (t.kscale2 != nullptr && j >= t.S1 && jj < nkeys)
        ks = rsqrtf(static_cast<float>(__ldcg(t.kscale2 + (j - t.S1))) / a.HD + a.eps);
      kfw[32 * h + lane] = (jj < nkeys && m.sKm[jj] != 0) ? ks * a.scale_log2 : 0.f;
    }
    __syncwarp();
    bool got = mbar_wait(&tl->attn_s, par, a.status, kErrWaitAccum);
    ok = __all_sync(0xffffffffu, got);
    float mq = -INFINITY, lq = 0.f;
    if (ok) {
      tc_fence_after();
      float sv[64];
      tmem_ld32(lane_addr + kAttnColS + 64 * wq, sv);
      tmem_ld32(lane_addr + kAttnColS + 64 * wq + 32, sv + 32);
      const bool v0 = q < a.R;
      // attend bits of row q for the warp's 64 keys
      uint32_t mb0 = 0xffffffffu, mb1 = 0xffffffffu;
      if (t.mask2d != nullptr) {
        uint32_t w[16];
        const uint4* src = reinterpret_cast<const uint4*>(m.sM + q * 256 + 64 * wq);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 u = src[i];
          w[4 * i] = u.x;
          w[4 * i + 1] = u.y;
          w[4 * i + 2] = u.z;
          w[4 * i + 3] = u.w;
        }
        uint32_t all1 = 0x01010101u;
#pragma unroll
        for (int i = 0; i < 16; ++i) all1 &= w[i];
        if (all1 != 0x01010101u) {  // not every byte 1: byte by byte
          mb0 = mb1 = 0u;
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              mb0 |= (((w[i] >> (8 * k)) & 0xffu) != 0u ? 1u : 0u) << (4 * i + k);
              mb1 |= (((w[8 + i] >> (8 * k)) & 0xffu) != 0u ? 1u : 0u) << (4 * i + k);
            }
        }
      }
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float kf = m.sKsc[64 * wq + i];
        const bool bit = ((i < 32 ? mb0 >> i : mb1 >> (i - 32)) & 1u) != 0u;
        sv[i] = (v0 && kf != 0.f && bit) ? sv[i] * kf : -INFINITY;
      }
      // short dependency chains (one warp per SM sub-partition runs this): a
      // tree maximum and four partial sums
      float t32[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) t32[i] = fmaxf(sv[i], sv[i + 32]);
#pragma unroll
      for (int w2 = 16; w2 >= 1; w2 >>= 1)
#pragma unroll
        for (int i = 0; i < w2; ++i) t32[i] = fmaxf(t32[i], t32[i + w2]);
      const float mx = t32[0];
      const float base = mx == -INFINITY ? 0.f : mx;
      uint32_t pk[32];
      float psa[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const float p0 = exp2f(sv[i] - base), p1 = exp2f(sv[i + 1] - base);
        psa[(i >> 1) & 3] += p0 + p1;
        pk[i / 2] = pack_bf16(p0, p1);
      }
      const float ps = (psa[0] + psa[1]) + (psa[2] + psa[3]);
      tmem_st16(lane_addr + kAttnColP + 32 * wq, pk);
      tmem_st16(lane_addr + kAttnColP + 32 * wq + 16, pk + 16);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      mq = mx;
      lq = ps;
      // P.V over this warp's keys < nkeys (16 per step): A = its P columns, B =
      // the V rows as staged ([keys, dims]: MN-major), D = its S columns
      if (lane == 0) {
        tc_fence_after();
        const uint32_t idesc = umma_idesc_bf16_bmn(128, 64);
        const int steps = (min(64, nkeys - 64 * wq) + 15) / 16;
        for (int kk = 0; kk < steps; ++kk)
          umma_bf16_ts(lane_addr - (static_cast<uint32_t>(wq * 32) << 16) + kAttnColS + 64 * wq,
                       tl->tmem + kAttnColP + 32 * wq + 8 * kk, umma_desc_sw128_mn(m.sV + (4 * wq + kk) * 2048),
                       idesc, kk > 0 ? 1u : 0u);
        umma_commit(&tl->attn_o[wq]);
      }
      __syncwarp();
      // attn_o[w] completes only on items with keys for warp w: its own count
      got = mbar_wait(&tl->attn_o[wq], pv_it & 1, a.status, kErrWaitAccum);
      ++pv_it;
      ok = __all_sync(0xffffffffu, got);
    }
    if (ok) {
      tc_fence_after();
      float* orow = comb + (wq * kFusedRows + q) * kCombRow;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float ov[32];
        tmem_ld32(lane_addr + kAttnColS + 64 * wq + 32 * c, ov);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i)
          reinterpret_cast<float4*>(orow + 32 * c)[i] = make_float4(ov[4 * i], ov[4 * i + 1], ov[4 * i + 2], ov[4 * i + 3]);
      }
      cml[(wq * kFusedRows + q) * 2] = mq;
      cml[(wq * kFusedRows + q) * 2 + 1] = lq;
    } else if (lane == 0) {
      tl->abort = 1;
    }
  } else if (smx) {
    // no keys of this item: a zero partial, written once S (which reads K and
    // Q) is complete
    const bool got = mbar_wait(&tl->attn_s, par, a.status, kErrWaitAccum);
    if (!__all_sync(0xffffffffu, got) && lane == 0) tl->abort = 1;
    float* orow = comb + (wq * kFusedRows + q) * kCombRow;
#pragma unroll
    for (int i = 0; i < 16; ++i) reinterpret_cast<float4*>(orow)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    cml[(wq * kFusedRows + q) * 2] = -INFINITY;
    cml[(wq * kFusedRows + q) * 2 + 1] = 0.f;
  }
  bar_workers();
  const int nsplit = t.nsplit;
  // merge the 4 key blocks: the split's (O, m, l), four dims per thread; every
  // thread derives its row's block weights itself (no serial pass).  A split
  // partial is O [32][64] followed by (m, l) [32][2] (kSplitStride floats).
  __nv_bfloat16* out = t.out;
  float* part = t.part;
  const long long ots = t.ots;
  for (int idx = threadIdx.x - 32; idx < kFusedRows * 16; idx += kFusedWorkers) {
    const int r = idx >> 4, d = (idx & 15) * 4;
    float mb[4], lb[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const float2 ml = *reinterpret_cast<const float2*>(cml + (b * kFusedRows + r) * 2);
      mb[b] = ml.x;
      lb[b] = ml.y;
    }
    const float M = fmaxf(fmaxf(mb[0], mb[1]), fmaxf(mb[2], mb[3]));
    const float base = M == -INFINITY ? 0.f : M;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float L = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const float w = exp2f(mb[b] - base);
      L += w * lb[b];
      const float4 ov = *reinterpret_cast<const float4*>(comb + (b * kFusedRows + r) * kCombRow + d);
      acc.x += w * ov.x;
      acc.y += w * ov.y;
      acc.z += w * ov.z;
      acc.w += w * ov.w;
    }
    if (nsplit == 1) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      if (r < a.R) {
        uint2 pk;
        pk.x = pack_bf16(acc.x * inv, acc.y * inv);
        pk.y = pack_bf16(acc.z * inv, acc.w * inv);
        *reinterpret_cast<uint2*>(out + r * ots + d) = pk;
      }
    } else {
      *reinterpret_cast<float4*>(part + r * 64 + d) = acc;
      if (d == 0) *reinterpret_cast<float2*>(part + kFusedRows * 64 + r * 2) = make_float2(M, L);
    }
  }
  if (nsplit == 1) {
    bar_workers();
    return;
  }
  // publish the partial (CTA barrier, then one fence + counter atomic), and
  // the last arriving split merges: its counter thread fences again before
  // the CTA reads the other splits' partials through L2
  bar_workers();
  if (threadIdx.x == 32) {
    __threadfence();
    const bool last = atomicAdd(t.counter, 1u) == static_cast<unsigned>(nsplit - 1);
    if (last) __threadfence();
    tl->last = last ? 1 : 0;
  }
  bar_workers();
  if (tl->last) {
    // every split's partial -> shared memory in one cp.async group (L2 reads,
    // kSplitStride floats each), then the output rows
    float* sp_all = reinterpret_cast<float*>(stg);
    const float* part_head = t.part_head;
    const int nchunk = nsplit * kSplitStride / 4;
    for (int c = threadIdx.x - 32; c < nchunk; c += kFusedWorkers)
      cp_async16(sp_all + c * 4, part_head + c * 4, true);
    cp_async_commit();
    cp_async_wait<0>();
    bar_workers();
    // every output element: its row's split weights (recomputed per thread,
    // no serial pass), then the weighted sum over the splits
    for (int idx = threadIdx.x - 32; idx < a.R * 16; idx += kFusedWorkers) {
      const int r = idx >> 4, d = (idx & 15) * 4;
      float M = -INFINITY;
#pragma unroll
      for (int sp = 0; sp < kFusedMaxSplits; ++sp)
        if (sp < nsplit) M = fmaxf(M, sp_all[sp * kSplitStride + kFusedRows * 64 + r * 2]);
      const float base = M == -INFINITY ? 0.f : M;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      float L = 0.f;
#pragma unroll
      for (int sp = 0; sp < kFusedMaxSplits; ++sp) {
        if (sp < nsplit) {
          const float2 ml = *reinterpret_cast<const float2*>(sp_all + sp * kSplitStride + kFusedRows * 64 + r * 2);
          const float w = exp2f(ml.x - base);
          L += w * ml.y;
          const float4 ov = *reinterpret_cast<const float4*>(sp_all + sp * kSplitStride + r * 64 + d);
          acc.x += w * ov.x;
          acc.y += w * ov.y;
          acc.z += w * ov.z;
          acc.w += w * ov.w;
        }
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      uint2 pk;
      pk.x = pack_bf16(acc.x * inv, acc.y * inv);
      pk.y = pack_bf16(acc.z * inv, acc.w * inv);
      *reinterpret_cast<uint2*>(out + r * ots + d) = pk;
    }
  }
  bar_workers();
}


// Attention work items.  Joint attention item i = (head, key split); cross
// attention item h = head.  Their CTAs start after the qkv CTAs (joint) and
// after the cross-q CTAs (cross), so that they are idle in the phase before
// and can prefetch their constant K / V there.
__device__ __forceinline__ int attn_joint_first(const FusedArgs& a, int cta, int G) {
  const int off = 2 * (3 * a.HD / 128);  // after the qkv pairs
  return ((cta - off) % G + G) % G;
}
__device__ __forceinline__ int attn_cross_first(const FusedArgs& a, int cta, int G) {
  const int off = 2 * (3 * a.HD / 128 + a.HD / 128 + a.F / 128);  // after every pair CTA
  return ((cta - off) % G + G) % G;
}

__device__ AttnItem joint_item(const FusedArgs& a, int step, int l, int i) {
  const int h = i / a.splits, sp = i % a.splits;
  const double* ssq = a.ssq + (static_cast<long long>(step) * a.L + l) * 3 * kFusedRows;
  AttnItem t;
  t.k1 = a.vk[l] + h * a.hd;
  t.v1 = a.vv[l] + h * a.hd;
  t.ts1 = a.v_ts;
  t.S1 = a.Sv;
  t.k2 = a.ka + h * a.hd;
  t.v2 = a.va + h * a.hd;
  t.ts2 = a.HD;
  t.S2 = a.Sa;
  t.kscale2 = ssq + kFusedRows;
  t.qp = a.q + h * a.hd;
  t.qts = a.HD;
  t.qscale = ssq;
  t.mask2d = a.mask2d;
  t.mrs = a.Sv + a.Sa;
  t.key_mask = nullptr;
  t.k0 = sp * a.kps;
  t.k1end = min(a.Sv + a.Sa, t.k0 + a.kps);
  t.out = a.ao + h * a.hd;
  t.ots = a.HD;
  t.part_head = a.apart + static_cast<long long>(h) * a.splits * kSplitStride;
  t.part = t.part_head + sp * kSplitStride;
  t.counter = a.sync + 2 + (static_cast<long long>(step) * a.L + l) * a.H + h;
  t.nsplit = a.splits;
  return t;
}

__device__ AttnItem cross_item(const FusedArgs& a, int step, int l, int h) {
  const double* ssq = a.ssq + (static_cast<long long>(step) * a.L + l) * 3 * kFusedRows;
  const __nv_bfloat16* kv = a.ckv + static_cast<long long>(l) * 2 * a.HD;  // [C][L][2HD]
  AttnItem t;
  t.k1 = kv + h * a.hd;
  t.v1 = kv + a.HD + h * a.hd;
  t.ts1 = static_cast<long long>(a.L) * 2 * a.HD;
  t.S1 = a.C;
  t.k2 = nullptr;
  t.v2 = nullptr;
  t.ts2 = 0;
  t.S2 = 0;
  t.kscale2 = nullptr;
  t.qp = a.qc + h * a.hd;
  t.qts = a.HD;
  t.qscale = ssq + 2 * kFusedRows;
  t.mask2d = nullptr;
  t.mrs = 0;
  t.key_mask = a.ctx_mask;
  t.k0 = 0;
  t.k1end = a.C;
  t.out = a.ci + h * a.hd;
  t.ots = a.HD;
  t.part = nullptr;
  t.part_head = nullptr;
  t.counter = nullptr;
  t.nsplit = 1;
  return t;
}

// ------------------------------------------------------------------ kernel
__global__ void __launch_bounds__(kFusedThreads, 1) fused_chunk_kernel(const __grid_constant__ FusedArgs a) {
  extern __shared__ uint8_t fused_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fused_smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem;
  uint8_t* stg = smem + kFusedRing * kATile;
  FusedSmemTail* tl = reinterpret_cast<FusedSmemTail*>(smem + fused_tail_offset());
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, G = gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFusedRing; ++s) {
      mbar_init(&tl->full[s], 1);
      mbar_init(&tl->empty[s], 1);
    }
    mbar_init(&tl->accum, kFusedIssuers);
    mbar_init(&tl->xstat_bar, kFusedWorkers / 32);  // one arrival per peer worker warp
    mbar_init(&tl->xacc_bar, 1);                    // own expect_tx arrival + the peer's bulk copy
    mbar_init(&tl->xsend_bar, 4);                   // lane 0 of this CTA's 4 sending warps
    mbar_init(&tl->attn_s, 1);
    for (int w = 0; w < 4; ++w) mbar_init(&tl->attn_o[w], 1);
    tl->abort = 0;
    fence_mbar_init();
    for (int p = 0; p < 6; ++p) tma_prefetch_desc(&a.tm[p]);
  }
  if (warp == 1) {
    tmem_alloc(&tl->tmem, kFusedTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp >= 4 && warp < 8) {
    // the attention items' P columns outside a softmax warp's own quarter of
    // the keys stay zero for the whole launch
    const uint32_t z[16] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    const uint32_t pbase = tl->tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + kAttnColP;
#pragma unroll
    for (int c = 0; c < 8; ++c) tmem_st16(pbase + 16 * c, z);
    tmem_wait_st();
  }

  if (warp == 0) {
    // ------------------------------------------------ weight producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      uint32_t it = 0;
      for (int step = 0; step < a.N && !tl->abort; ++step)
        for (int l = 0; l < a.L && !tl->abort; ++l)
          for (int p = 0; p < 6 && !tl->abort; ++p) {
            const int cnt = f_count(a, p), rows = f_rows(a, p);
            const int half = f_pair(p) ? static_cast<int>(cluster_ctarank()) : 0;
            for (int i = f_first(a, p, cta, G); i < cnt && !tl->abort; i += f_units(p, G)) {
              const FItem itm = f_item(a, p, i, half);
              for (int k = 0; k < itm.nkb; ++k) {
                const int s = it % kFusedRing;
                if (it >= kFusedRing &&
                    !mbar_wait(&tl->empty[s], ((it / kFusedRing) - 1) & 1, a.status, kErrWaitEmpty)) {
                  tl->abort = 1;
                  break;
                }
                mbar_arrive_expect_tx(&tl->full[s], kATile);
                tma_load_2d(ring + s * kATile, &a.tm[p], &tl->full[s], (itm.kb0 + k) * 64,
                            l * rows + itm.n * 128, pol);
                ++it;
              }
            }
          }
      // drain: the last issued tiles have landed (consumed on the normal path)
      const uint32_t first = it > kFusedRing ? it - kFusedRing : 0;
      for (uint32_t j = first; j < it; ++j)
        mbar_wait(&tl->full[j % kFusedRing], (j / kFusedRing) & 1, a.status, kErrWaitFull);
    }
  } else {
    // ------------------------------------------------------ workers
    uint32_t ring_it = 0, items_done = 0, epoch = 0, pair_done = 0, xstat_done = 0, attn_it = 0, pv_it = 0;
    const int rank = static_cast<int>(cluster_ctarank());
    const int R = a.R, D = a.D;
    const bool has_qkv = f_first(a, kFQkv, cta, G) < f_count(a, kFQkv);
    const bool has_cq = f_first(a, kFCq, cta, G) < f_count(a, kFCq);
    const bool has_ffn0 = f_first(a, kFFfn0, cta, G) < f_count(a, kFFfn0);
    for (int step = 0; step < a.N && !tl->abort; ++step) {
      if (step == 0) {
        // action_encoder of the first step: x = bf16(enc_w latent + enc_b); later
        // steps encode right after their head / Euler update (same warp, same row)
        for (int idx = cta * kFusedWorkers + threadIdx.x - 32; idx < R * D; idx += G * kFusedWorkers) {
          const int r = idx / D, f = idx % D;
          float acc = bf2f(a.enc_b[f]);
          for (int c = 0; c < a.A; ++c) acc += bf2f(a.enc_w[f * a.A + c]) * bf2f(__ldcg(a.latent + r * a.A + c));
          a.x[idx] = f2bf(acc);
        }
        if (has_qkv) ln_const_prefetch(a, stg, step, 0, 0, 0);
        if (!grid_sync(a, epoch, tl)) break;
      }
      for (int l = 0; l < a.L && !tl->abort; ++l) {
        // qkv
        for (int i = f_first(a, kFQkv, cta, G); i < f_count(a, kFQkv); i += f_units(kFQkv, G))
          gemm_item(a, ring, stg, tl, kFQkv, step, l, f_item(a, kFQkv, i, rank), ring_it, items_done, pair_done, xstat_done);
        // constant K / V of the first joint item, on CTAs without a qkv item
        // (one that has one would delay its barrier arrival)
        if (!has_qkv && attn_joint_first(a, cta, G) < a.H * a.splits)
          attn_stage_const(a, stg, joint_item(a, step, l, attn_joint_first(a, cta, G)));
        if (!grid_sync(a, epoch, tl)) break;
        // joint attention: items (head, split); the first item's constant
        // K / V were prefetched at the end of the qkv phase
        for (int i = attn_joint_first(a, cta, G); i < a.H * a.splits; i += G)
          attention_item(a, stg, tl, joint_item(a, step, l, i), !has_qkv && i == attn_joint_first(a, cta, G),
                         attn_it, pv_it);
        if (!grid_sync(a, epoch, tl)) break;
        for (int i = f_first(a, kFO, cta, G); i < f_count(a, kFO); i += f_units(kFO, G))
          gemm_item(a, ring, stg, tl, kFO, step, l, f_item(a, kFO, i, rank), ring_it, items_done, pair_done, xstat_done);
        if (has_cq) ln_const_prefetch(a, stg, step, l, 1, 0);
        if (!grid_sync(a, epoch, tl)) break;
        for (int i = f_first(a, kFCq, cta, G); i < f_count(a, kFCq); i += f_units(kFCq, G))
          gemm_item(a, ring, stg, tl, kFCq, step, l, f_item(a, kFCq, i, rank), ring_it, items_done, pair_done, xstat_done);
        if (a.C > 0 && attn_cross_first(a, cta, G) < a.H)
          attn_stage_const(a, stg, cross_item(a, step, l, attn_cross_first(a, cta, G)));
        if (!grid_sync(a, epoch, tl)) break;
        // cross attention: one item per head over the context (constant K / V
        // prefetched at the end of the cross-q phase)
        for (int h = attn_cross_first(a, cta, G); h < a.H && a.C > 0; h += G)
          attention_item(a, stg, tl, cross_item(a, step, l, h), h == attn_cross_first(a, cta, G), attn_it,
                         pv_it);
        if (!grid_sync(a, epoch, tl)) break;
        for (int i = f_first(a, kFCo, cta, G); i < f_count(a, kFCo); i += f_units(kFCo, G))
          gemm_item(a, ring, stg, tl, kFCo, step, l, f_item(a, kFCo, i, rank), ring_it, items_done, pair_done, xstat_done);
        if (has_ffn0) ln_const_prefetch(a, stg, step, l, 0, 3);
        if (!grid_sync(a, epoch, tl)) break;
        for (int i = f_first(a, kFFfn0, cta, G); i < f_count(a, kFFfn0); i += f_units(kFFfn0, G))
          gemm_item(a, ring, stg, tl, kFFfn0, step, l, f_item(a, kFFfn0, i, rank), ring_it, items_done, pair_done, xstat_done);
        if (!grid_sync(a, epoch, tl)) break;
        for (int i = f_first(a, kFFfn2, cta, G); i < f_count(a, kFFfn2); i += f_units(kFFfn2, G))
          gemm_item(a, ring, stg, tl, kFFfn2, step, l, f_item(a, kFFfn2, i, rank), ring_it, items_done, pair_done, xstat_done);
        if (has_qkv && l + 1 < a.L) ln_const_prefetch(a, stg, step, l + 1, 0, 0);
        if (!grid_sync(a, epoch, tl)) break;
      }
      if (tl->abort) break;
      // head + Euler update + the next step's action_encoder: one CTA per token
      // row (row-local, no barrier between).  The row goes to shared memory
      // first; warps take the velocity channels, one thread per channel
      // updates the latent, every thread re-encodes features of the row.
      for (int r = cta; r < R; r += G) {
        const int wi = warp - 1, wt = threadIdx.x - 32;
        float* svel = &tl->stat[0][0];
        float* slat = &tl->stat[kFusedRows / 2][0];
        __nv_bfloat16* xres = a.x + static_cast<long long>(r) * D;
        float* xrow = reinterpret_cast<float*>(stg);
        for (int f = wt; f < D; f += kFusedWorkers) xrow[f] = bf2f(__ldcg(xres + f));
        bar_workers();
        for (int c = wi; c < a.A; c += 11) {
          float acc = 0.f;
#pragma unroll 4
          for (int ch = lane; ch < D / 8; ch += 32) {
            const float4 x0 = *reinterpret_cast<const float4*>(xrow + ch * 8);
            const float4 x1 = *reinterpret_cast<const float4*>(xrow + ch * 8 + 4);
            const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            float wv[8];
            ld_bf8(a.head_w + static_cast<long long>(c) * D + ch * 8, wv);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc += xv[e] * wv[e];
          }
          acc = warp_sum(acc);
          if (lane == 0) svel[c] = rbf(acc + bf2f(a.head_b[c]));
        }
        bar_workers();
        if (wt < a.A) {
          const float vel = svel[wt];
          const float d = rbf(a.deltas.t[step]);
          const float lat = bf2f(f2bf(bf2f(__ldcg(a.latent + r * a.A + wt)) + rbf(vel * d)));
          if (a.trace != nullptr) a.trace[(static_cast<long long>(step) * R + r) * a.A + wt] = f2bf(vel);
          a.latent[r * a.A + wt] = f2bf(lat);
          slat[wt] = lat;
        }
        bar_workers();
        if (step + 1 < a.N) {
#pragma unroll 3
          for (int f = wt; f < D; f += kFusedWorkers) {
            float acc = bf2f(a.enc_b[f]);
            for (int c = 0; c < a.A; ++c) acc += bf2f(a.enc_w[f * a.A + c]) * slat[c];
            xres[f] = f2bf(acc);
          }
        }
        bar_workers();  // xrow (staging) is reused by the next row / the prefetch below
      }
      if (has_qkv && step + 1 < a.N) ln_const_prefetch(a, stg, step + 1, 0, 0, 0);
      if (!grid_sync(a, epoch, tl)) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tl->tmem, kFusedTmemCols);
  }
  // the peer CTA may still write into this CTA's shared memory (DSMEM) until
  // it is done too
  cluster_barrier();
}

cudaError_t fused_init_attributes() {
  return cudaFuncSetAttribute(fused_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(fused_smem_bytes()));
}

cudaError_t launch_fused_chunk(const FusedArgs& a, int grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kFusedThreads);
  cfg.dynamicSmemBytes = fused_smem_bytes();
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, fused_chunk_kernel, a);
}

int fused_max_ctas() {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(kFusedThreads);
  cfg.dynamicSmemBytes = fused_smem_bytes();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, fused_chunk_kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return 2 * clusters;
}

}  // namespace fam
