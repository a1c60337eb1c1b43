// Host runtime of the video DiT prefill (WanVideoDiT.prepare +
// MoT.prefill_video_cache_tensor): large-M GEMMs with activations as the MMA
// A operand (128-token tiles) and weights as B, fused epilogues (bias, GELU,
// gated fp32 residual with the per-token first-frame / rest modulation),
// row kernels for the LayerNorms and the q/k RMSNorm + 3-D RoPE that write K
// and V straight into the caller's per-block cache, and the first-frame-causal
// flash attention as a mask descriptor.
//
// Chain per block l:
//   resid_norm(AdaLN msa) -> gemm qkv -> qkv_post(RMSNorm, RoPE; K,V -> cache)
//   -> attention(first-frame causal) -> gemm o (+= gate_msa) -> resid_norm(norm3)
//   -> gemm cross-q -> rms_rows -> cross attention -> gemm cross-o (+=)
//   -> resid_norm(AdaLN mlp) -> gemm ffn.0 (+GELU) -> gemm ffn.2 (+= gate_mlp)
// The last block stops after its K/V when the final token states are not
// requested (nothing after them reaches the cache).
#include <string.h>

#include <cmath>
#include <memory>
#include <vector>

#include "../../include/fam.h"
#include "fam_internal.h"
#include "fam_kernels.h"

using namespace fam;

namespace {

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }
const __nv_bfloat16* bf(const void* p) { return static_cast<const __nv_bfloat16*>(p); }

struct VLayout {
  size_t x, h, qkv, q, ao, qc, ci, fh, patch, tmod, sin, th1, th2, cemb, ch1, ckv, apart, ctr, vt, skp, skf;
  size_t total;
};

VLayout vlayout(const fam_video_config& c, int B, int S, int C) {
  VLayout w = {};
  const size_t M = static_cast<size_t>(B) * S, BC = static_cast<size_t>(B) * C;
  const size_t D = c.hidden_dim, HD = static_cast<size_t>(c.num_heads) * c.head_dim, F = c.ffn_dim;
  const size_t Kp = static_cast<size_t>(c.in_dim) * c.patch_t * c.patch_h * c.patch_w;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes);
    return o;
  };
  w.x = take(M * D * 4);
  w.h = take(M * D * 2);
  w.qkv = take(M * 3 * HD * 2);
  w.q = take(M * HD * 2);
  w.ao = take(M * HD * 2);
  w.qc = take(M * HD * 2);
  w.ci = take(M * HD * 2);
  w.fh = take(M * F * 2);
  w.patch = take(M * Kp * 2);
  w.tmod = take(2 * static_cast<size_t>(B) * 6 * D * 4);
  w.sin = take(2 * static_cast<size_t>(B) * c.freq_dim * 2);
  w.th1 = take(2 * static_cast<size_t>(B) * D * 2);
  w.th2 = take(2 * static_cast<size_t>(B) * D * 2);
  w.cemb = take(BC * D * 2);
  w.ch1 = take(BC * D * 2);
  w.ckv = take(static_cast<size_t>(c.num_layers) * BC * 2 * HD * 2);
  // attention runs unsplit at these query counts; a small area for safety
  w.apart = take(attn_partial_bytes(B, c.num_heads, S, c.head_dim, 1));
  w.ctr = take(static_cast<size_t>(B) * c.num_heads * attn_query_tiles(S) * 4);
  w.vt = take(attention_tc_vt_bytes(B, c.num_heads, S));  // V^T of the tcgen05 self attention
  w.skp = take(gemm_sk_scratch_bytes());                   // split-round partials of the GEMMs
  w.skf = take(static_cast<size_t>(gemm_num_sms()) * sizeof(unsigned));
  w.total = off;
  return w;
}

struct VCallKey {
  std::vector<uintptr_t> ptrs;
  std::vector<float> vals;
  bool operator==(const VCallKey& o) const { return ptrs == o.ptrs && vals == o.vals; }
};

}  // namespace

struct fam_video_expert {
  fam_video_config cfg;
  fam_video_weights w;
  std::vector<fam_action_layer> layers;
  cudaStream_t cap_stream = nullptr;
  cudaGraphExec_t graph = nullptr;
  VCallKey key;
  int* status = nullptr;
  int launch_count = 0;
};

namespace {

struct VCtx {
  fam_video_expert* e;
  const fam_video_io* io;
  char* ws;
  VLayout L;
  int B, S, M, BC, tpf;
  cudaStream_t st;
  bool pdl;
};

template <typename T>
T* wp(const VCtx& c, size_t off) {
  return reinterpret_cast<T*>(c.ws + off);
}

#define V_TRY(expr)                                           \
  do {                                                        \
    cudaError_t _e = (expr);                                  \
    if (_e != cudaSuccess) return check_cuda(_e, #expr);      \
  } while (0)
#define V_TRYI(expr) \
  do {               \
    int _r = (expr); \
    if (_r) return _r; \
  } while (0)
#define V_LAUNCH(expr)       \
  do {                       \
    V_TRY(expr);             \
    ++c.e->launch_count;     \
  } while (0)

// Activations [M, K] (A) x weights [N, K] (B).  kind: store bf16 / store f32 /
// residual (gated by modulation chunk `gate_chunk` of block modulation mod_w,
// -1 = gate 1).
int gemm_x(const VCtx& c, const void* act, long long lda, int M, const void* W, const void* bias,
           int N, int K, int kind, int act_kind, void* out, long long ldo, bool out_f32,
           const void* mod_w = nullptr, int gate_chunk = -1) {
  GemmEpilogue e = {};
  e.features_on_a = 0;
  e.kind = kind;
  e.act = act_kind;
  e.out = out;
  e.out_sa = ldo;
  e.out_sb = 1;
  e.out_bf16 = out_f32 ? 0 : 1;
  e.bias = bf(bias);
  if (kind == kEpiResidual && gate_chunk >= 0) {
    const int D = c.e->cfg.hidden_dim;
    e.gate_w = bf(mod_w) + gate_chunk * D;
    e.gate_t = wp<float>(c, c.L.tmod) + gate_chunk * D;
    e.tokens_per_batch = c.S;
    e.first_frame_tokens = c.tpf;
    e.gate_bstride = 2LL * 6 * D;
    e.gate_gstride = 6LL * D;
  }
  GemmPlan p;
  V_TRYI(gemm_plan(&p, act, lda, W, K, M, N, K, 1, 0, e, false, true, c.e->status, wp<float>(c, c.L.skp),
                   wp<unsigned>(c, c.L.skf), gemm_sk_scratch_bytes(), false, /*allow_pair=*/true));
  V_LAUNCH(gemm_launch(p, c.st, c.pdl));
  return 0;
}

ModRows vmod(const VCtx& c, const void* mod_w) {
  ModRows m = {};
  const int D = c.e->cfg.hidden_dim;
  m.tmod = wp<float>(c, c.L.tmod);
  m.mod_w = bf(mod_w);
  m.tokens_per_batch = c.S;
  m.first_frame_tokens = c.tpf;
  m.bstride = 2LL * 6 * D;
  m.gstride = 6LL * D;
  return m;
}

int enqueue_prefill(const VCtx& c) {
  const fam_video_config& g = c.e->cfg;
  const fam_video_weights& w = c.e->w;
  const fam_video_io& io = *c.io;
  const int D = g.hidden_dim, HD = g.num_heads * g.head_dim, F = g.ffn_dim, Lyr = g.num_layers;
  const int M = c.M, S = c.S, B = c.B;
  const int Kp = g.in_dim * g.patch_t * g.patch_h * g.patch_w;
  c.e->launch_count = 0;
  const size_t ctr_bytes = static_cast<size_t>(B) * g.num_heads * attn_query_tiles(S) * 4;
  V_TRY(cudaMemsetAsync(wp<void>(c, c.L.ctr), 0, ctr_bytes, c.st));
  V_TRY(cudaMemsetAsync(wp<void>(c, c.L.skf), 0, static_cast<size_t>(gemm_num_sms()) * sizeof(unsigned), c.st));

  // ---- time MLP on (first frame t=0, rest t) per sample
  StepTimes ts = {};
  for (int b = 0; b < B; ++b) {
    ts.t[2 * b] = 0.0f;
    ts.t[2 * b + 1] = io.timesteps[b];
  }
  V_LAUNCH(launch_sinusoid(ts, 2 * B, g.freq_dim, wp<__nv_bfloat16>(c, c.L.sin), c.st, false));
  auto gemm_rows = [&](const void* act, int rows, int K, const void* W, const void* bias, int N,
                       int act_kind, void* out, bool f32) -> int {
    // few rows: weights as A (features on the 128-row MMA side)
    GemmEpilogue e = {};
    e.features_on_a = 1;
    e.kind = kEpiStore;
    e.act = act_kind;
    e.out = out;
    e.out_sa = 1;
    e.out_sb = N;
    e.out_bf16 = f32 ? 0 : 1;
    e.bias = bf(bias);
    GemmPlan p;
    V_TRYI(gemm_plan(&p, W, K, act, K, N, rows, K, 1, 0, e, true, false, c.e->status));
    V_LAUNCH(gemm_launch(p, c.st, c.pdl));
    return 0;
  };
  V_TRYI(gemm_rows(wp<void>(c, c.L.sin), 2 * B, g.freq_dim, w.time0_w, w.time0_b, D, kActSilu,
                   wp<void>(c, c.L.th1), false));
  V_TRYI(gemm_rows(wp<void>(c, c.L.th1), 2 * B, D, w.time2_w, w.time2_b, D, kActSilu,
                   wp<void>(c, c.L.th2), false));
  V_TRYI(gemm_rows(wp<void>(c, c.L.th2), 2 * B, D, w.tproj_w, w.tproj_b, 6 * D, kActNone,
                   wp<void>(c, c.L.tmod), true));
  if (io.t_out != nullptr)  // t itself (before the SiLU of the projection input), for the output head
    V_TRYI(gemm_rows(wp<void>(c, c.L.th1), 2 * B, D, w.time2_w, w.time2_b, D, kActNone, io.t_out, false));
  // ---- patch embedding: patchify + GEMM into the fp32 residual stream
  PatchArgs pa = {bf(io.latents), wp<__nv_bfloat16>(c, c.L.patch), B, g.in_dim, io.frames,
                  io.height, io.width, g.patch_t, g.patch_h, g.patch_w};
  V_LAUNCH(launch_patchify(pa, c.st));
  V_TRYI(gemm_x(c, wp<void>(c, c.L.patch), Kp, M, w.patch_w, w.patch_b, D, Kp, kEpiStore,
                kActNone, wp<void>(c, c.L.x), D, true));
  // ---- text embedding + every block's cross K/V (step invariant)
  if (c.BC > 0) {
    V_TRYI(gemm_x(c, io.context, g.text_dim, c.BC, w.text0_w, w.text0_b, D, g.text_dim, kEpiStore,
                  kActGeluTanh, wp<void>(c, c.L.ch1), D, false));
    V_TRYI(gemm_x(c, wp<void>(c, c.L.ch1), D, c.BC, w.text2_w, w.text2_b, D, D, kEpiStore, kActNone,
                  wp<void>(c, c.L.cemb), D, false));
    // Cross K / V of every block, context-token major: ckv[row][l * 2HD + (K | V)]
    // (row = b * C + t); the K half RMSNorm'd with block l's norm_k.
    const long long ld = static_cast<long long>(Lyr) * 2 * HD;
    __nv_bfloat16* ckv_all = wp<__nv_bfloat16>(c, c.L.ckv);
    // projections stored block-major in one allocation (as the Python packer lays
    // them out): one GEMM over all blocks, one RMSNorm launch over (row, block)
    bool stacked = true;
    for (int l = 1; l < Lyr && stacked; ++l) {
      const fam_action_layer& l0 = c.e->layers[0];
      const fam_action_layer& ly = c.e->layers[l];
      stacked = bf(ly.ckv_w) == bf(l0.ckv_w) + static_cast<size_t>(l) * 2 * HD * D &&
                bf(ly.ckv_b) == bf(l0.ckv_b) + static_cast<size_t>(l) * 2 * HD &&
                bf(ly.cnorm_k) == bf(l0.cnorm_k) + static_cast<size_t>(l) * HD;
    }
    if (stacked) {
      const fam_action_layer& l0 = c.e->layers[0];
      V_TRYI(gemm_x(c, wp<void>(c, c.L.cemb), D, c.BC, l0.ckv_w, l0.ckv_b, static_cast<int>(ld), D,
                    kEpiStore, kActNone, ckv_all, ld, false));
      RmsRowsArgs r = {};
      r.in = ckv_all;
      r.in_stride = 2 * HD;  // (row, block) slice rr = row * L + l starts at rr * 2HD
      r.w = bf(l0.cnorm_k);
      r.w_period = Lyr;
      r.w_stride = HD;
      r.out = ckv_all;
      r.out_stride = 2 * HD;
      r.N = HD;
      r.eps = g.eps;
      V_LAUNCH(launch_rms_rows(r, c.BC * Lyr, c.st, c.pdl));
    } else {
      for (int l = 0; l < Lyr; ++l) {
        const fam_action_layer& ly = c.e->layers[l];
        __nv_bfloat16* ckv = ckv_all + static_cast<size_t>(l) * 2 * HD;
        V_TRYI(gemm_x(c, wp<void>(c, c.L.cemb), D, c.BC, ly.ckv_w, ly.ckv_b, 2 * HD, D, kEpiStore,
                      kActNone, ckv, ld, false));
        RmsRowsArgs r = {};
        r.in = ckv;
        r.in_stride = ld;
        r.w = bf(ly.cnorm_k);
        r.out = ckv;
        r.out_stride = ld;
        r.N = HD;
        r.eps = g.eps;
        V_LAUNCH(launch_rms_rows(r, c.BC, c.st, c.pdl));
      }
    }
  }

  const float scale_log2 = 1.4426950408889634f / std::sqrt(static_cast<float>(g.head_dim));
  float* x = wp<float>(c, c.L.x);
  __nv_bfloat16* h = wp<__nv_bfloat16>(c, c.L.h);
  for (int l = 0; l < Lyr; ++l) {
    const fam_action_layer& ly = c.e->layers[l];
    const bool last_cache_only = (l == Lyr - 1) && io.hidden_out == nullptr;
    // AdaLN (shift_msa, scale_msa)
    ResidNormArgs r0 = {};
    r0.x = x;
    r0.norm_mode = kNormAdaLN;
    r0.shift_chunk = 0;
    r0.gate_chunk = -1;
    r0.nmod = vmod(c, ly.modulation);
    r0.h = h;
    r0.h_stride = D;
    r0.D = D;
    r0.eps = g.eps;
    V_LAUNCH(launch_resid_norm(r0, M, c.st, c.pdl));
    V_TRYI(gemm_x(c, h, D, M, ly.qkv_w, ly.qkv_b, 3 * HD, D, kEpiStore, kActNone,
                  wp<void>(c, c.L.qkv), 3 * HD, false));
    QkvPostArgs qa = {};
    qa.qkv_bf16 = wp<__nv_bfloat16>(c, c.L.qkv);
    qa.nsplit = 0;
    qa.norm_q = bf(ly.norm_q);
    qa.norm_k = bf(ly.norm_k);
    qa.rope = reinterpret_cast<const float2*>(io.rope);
    qa.rows_per_batch = S;
    qa.q_out = wp<__nv_bfloat16>(c, c.L.q);
    qa.k_out = static_cast<__nv_bfloat16*>(io.cache_k[l]);
    qa.v_out = static_cast<__nv_bfloat16*>(io.cache_v[l]);
    qa.out_stride = HD;
    qa.HD = HD;
    qa.head_dim = g.head_dim;
    qa.eps = g.eps;
    V_LAUNCH(launch_qkv_post(qa, M, c.st, c.pdl));
    if (last_cache_only) break;

    AttnArgs aa = {};
    aa.q = qa.q_out;
    aa.q_bs = static_cast<long long>(S) * HD;
    aa.q_ts = HD;
    aa.k1 = qa.k_out;
    aa.v1 = qa.v_out;
    aa.kv1_bs = static_cast<long long>(S) * HD;
    aa.kv1_ts = HD;
    aa.S1 = S;
    aa.first_frame_tokens = io.first_frame_causal ? c.tpf : 0;
    aa.Sq = S;
    aa.H = g.num_heads;
    aa.scale_log2 = scale_log2;
    aa.out = wp<__nv_bfloat16>(c, c.L.ao);
    aa.out_bs = static_cast<long long>(S) * HD;
    aa.out_ts = HD;
    aa.nsplit = 1;
    aa.keys_per_split = S;
    aa.part = wp<float>(c, c.L.apart);
    aa.counters = wp<int>(c, c.L.ctr);
    if (attention_tc_eligible(g.head_dim, B, g.num_heads, S, S, 0, false, aa.first_frame_tokens, aa.q_ts, aa.kv1_ts,
                              aa.out_ts)) {
      V_LAUNCH(launch_attention_tc(aa.q, aa.q_ts, aa.k1, aa.v1, aa.kv1_ts, aa.out, aa.out_ts, B, S, S, g.num_heads,
                                   aa.first_frame_tokens, nullptr, 0, aa.scale_log2, wp<__nv_bfloat16>(c, c.L.vt),
                                   c.e->status, c.st, c.pdl));
      ++c.e->launch_count;  // V^T transpose + attention
    } else {
      V_LAUNCH(launch_attention(aa, B, g.head_dim, c.st, c.pdl));
    }
    V_TRYI(gemm_x(c, aa.out, HD, M, ly.o_w, ly.o_b, D, HD, kEpiResidual, kActNone, x, D, true,
                  ly.modulation, 2));
    // norm3 + cross attention (no gate)
    ResidNormArgs r1 = {};
    r1.x = x;
    r1.norm_mode = kNormAffine;
    r1.norm_w = bf(ly.norm3_w);
    r1.norm_b = bf(ly.norm3_b);
    r1.gate_chunk = -1;
    r1.h = h;
    r1.h_stride = D;
    r1.D = D;
    r1.eps = g.eps;
    V_LAUNCH(launch_resid_norm(r1, M, c.st, c.pdl));
    if (c.BC > 0) {
      V_TRYI(gemm_x(c, h, D, M, ly.cq_w, ly.cq_b, HD, D, kEpiStore, kActNone, wp<void>(c, c.L.qc),
                    HD, false));
      RmsRowsArgs rq = {};
      rq.in = wp<__nv_bfloat16>(c, c.L.qc);
      rq.in_stride = HD;
      rq.w = bf(ly.cnorm_q);
      rq.out = wp<__nv_bfloat16>(c, c.L.qc);
      rq.out_stride = HD;
      rq.N = HD;
      rq.eps = g.eps;
      V_LAUNCH(launch_rms_rows(rq, M, c.st, c.pdl));
      AttnArgs ca = {};
      ca.q = rq.out;
      ca.q_bs = static_cast<long long>(S) * HD;
      ca.q_ts = HD;
      const __nv_bfloat16* ckv = wp<__nv_bfloat16>(c, c.L.ckv) + static_cast<size_t>(l) * 2 * HD;
      ca.k1 = ckv;
      ca.v1 = ckv + HD;
      ca.kv1_bs = static_cast<long long>(io.context_tokens) * Lyr * 2 * HD;
      ca.kv1_ts = static_cast<long long>(Lyr) * 2 * HD;
      ca.S1 = io.context_tokens;
      ca.key_mask = io.context_mask;
      ca.key_mask_bs = io.context_tokens;
      ca.Sq = S;
      ca.H = g.num_heads;
      ca.scale_log2 = scale_log2;
      ca.out = wp<__nv_bfloat16>(c, c.L.ci);
      ca.out_bs = static_cast<long long>(S) * HD;
      ca.out_ts = HD;
      ca.nsplit = 1;
      ca.keys_per_split = io.context_tokens;
      ca.part = wp<float>(c, c.L.apart);
      ca.counters = wp<int>(c, c.L.ctr);
      // the tcgen05 kernel with the context as the key source (its V^T fits the
      // self attention's buffer while the context is no longer than the video)
      if (io.context_tokens <= S &&
          attention_tc_eligible(g.head_dim, B, g.num_heads, S, io.context_tokens, 0, false, 0, ca.q_ts, ca.kv1_ts,
                                ca.out_ts)) {
        V_LAUNCH(launch_attention_tc(ca.q, ca.q_ts, ca.k1, ca.v1, ca.kv1_ts, ca.out, ca.out_ts, B, S,
                                     io.context_tokens, g.num_heads, 0, io.context_mask, io.context_tokens,
                                     ca.scale_log2, wp<__nv_bfloat16>(c, c.L.vt), c.e->status, c.st, c.pdl));
        ++c.e->launch_count;  // V^T transpose + attention
      } else {
        V_LAUNCH(launch_attention(ca, B, g.head_dim, c.st, c.pdl));
      }
      V_TRYI(gemm_x(c, ca.out, HD, M, ly.co_w, ly.co_b, D, HD, kEpiResidual, kActNone, x, D, true));
    }
    // AdaLN (shift_mlp, scale_mlp) + FFN + gate_mlp
    ResidNormArgs r2 = {};
    r2.x = x;
    r2.norm_mode = kNormAdaLN;
    r2.shift_chunk = 3;
    r2.gate_chunk = -1;
    r2.nmod = vmod(c, ly.modulation);
    r2.h = h;
    r2.h_stride = D;
    r2.D = D;
    r2.eps = g.eps;
    V_LAUNCH(launch_resid_norm(r2, M, c.st, c.pdl));
    V_TRYI(gemm_x(c, h, D, M, ly.ffn0_w, ly.ffn0_b, F, D, kEpiStore, kActGeluTanh,
                  wp<void>(c, c.L.fh), F, false));
    V_TRYI(gemm_x(c, wp<void>(c, c.L.fh), F, M, ly.ffn2_w, ly.ffn2_b, D, F, kEpiResidual, kActNone,
                  x, D, true, ly.modulation, 5));
  }
  if (io.hidden_out != nullptr)
    V_TRY(cudaMemcpyAsync(io.hidden_out, x, static_cast<size_t>(M) * D * 4, cudaMemcpyDeviceToDevice,
                          c.st));
  return 0;
}

int vvalidate(const fam_video_expert* e, const fam_video_io* io, int* S, int* tpf) {
  if (e == nullptr || io == nullptr) return set_error("video: null expert or io");
  const fam_video_config& g = e->cfg;
  if (io->batch <= 0 || io->batch > kMaxSteps / 2) return set_error("video: batch must be in [1, %d]", kMaxSteps / 2);
  if (io->frames % g.patch_t || io->height % g.patch_h || io->width % g.patch_w)
    return set_error("video: latent grid not divisible by the patch size");
  if (io->latents == nullptr || io->timesteps == nullptr || io->rope == nullptr ||
      io->cache_k == nullptr || io->cache_v == nullptr)
    return set_error("video: null latents / timesteps / rope / cache");
  if (io->context_tokens > 0 && io->context == nullptr) return set_error("video: context missing");
  *tpf = (io->height / g.patch_h) * (io->width / g.patch_w);
  *S = (io->frames / g.patch_t) * *tpf;
  const size_t need = vlayout(g, io->batch, *S, io->context_tokens).total;
  if (io->workspace == nullptr || io->workspace_bytes < need)
    return set_error("video: workspace of %zu bytes needed, %zu given", need, io->workspace_bytes);
  return 0;
}

}  // namespace

extern "C" {

int fam_video_expert_create(const fam_video_config* cfg, const fam_video_weights* w,
                            fam_video_expert** out) {
  if (cfg == nullptr || w == nullptr || out == nullptr || w->layers == nullptr)
    return set_error("video: null argument");
  if (cfg->head_dim != 64 && cfg->head_dim != 128) return set_error("video: head_dim must be 64 or 128");
  if (cfg->hidden_dim % 64 || cfg->ffn_dim % 64 || cfg->text_dim % 8 || cfg->freq_dim % 64 ||
      (cfg->in_dim * cfg->patch_t * cfg->patch_h * cfg->patch_w) % 8)
    return set_error("video: widths must be multiples of 64 (patch length of 8)");
  if (cfg->hidden_dim > 4096) return set_error("video: hidden_dim <= 4096");
  int rc = check_cuda(gemm_init_attributes(), "gemm attributes");
  if (rc) return rc;
  rc = check_cuda(attn_init_attributes(), "attention attributes");
  if (rc) return rc;
  auto e = std::make_unique<fam_video_expert>();
  e->cfg = *cfg;
  e->w = *w;
  e->layers.assign(w->layers, w->layers + cfg->num_layers);
  e->w.layers = e->layers.data();
  e->status = device_status_word();
  if (e->status == nullptr) return set_error("video: no device status word");
  rc = check_cuda(cudaStreamCreateWithFlags(&e->cap_stream, cudaStreamNonBlocking), "stream create");
  if (rc) return rc;
  *out = e.release();
  return FAM_OK;
}

int fam_video_expert_destroy(fam_video_expert* e) {
  if (e == nullptr) return FAM_OK;
  if (e->graph) cudaGraphExecDestroy(e->graph);
  if (e->cap_stream) cudaStreamDestroy(e->cap_stream);
  delete e;
  return FAM_OK;
}

int fam_video_workspace_size(const fam_video_expert* e, int32_t batch, int32_t tokens,
                             int32_t context_tokens, size_t* bytes) {
  if (e == nullptr || bytes == nullptr || batch <= 0 || tokens <= 0 || context_tokens < 0)
    return set_error("video: bad argument");
  *bytes = vlayout(e->cfg, batch, tokens, context_tokens).total;
  return FAM_OK;
}

int fam_video_launch_count(const fam_video_expert* e, int32_t* count) {
  if (e == nullptr || count == nullptr) return set_error("video: null argument");
  *count = e->launch_count;
  return FAM_OK;
}

int fam_video_prefill(fam_video_expert* e, const fam_video_io* io, int32_t use_graph, void* stream) {
  int S = 0, tpf = 0;
  int rc = vvalidate(e, io, &S, &tpf);
  if (rc) return rc;
  VCtx c;
  c.e = e;
  c.io = io;
  c.ws = static_cast<char*>(io->workspace);
  c.B = io->batch;
  c.S = S;
  c.M = io->batch * S;
  c.BC = io->batch * io->context_tokens;
  c.tpf = io->frames / e->cfg.patch_t > 1 ? tpf : S;  // a single frame is all "first frame"
  c.L = vlayout(e->cfg, c.B, S, io->context_tokens);
  cudaStream_t user = static_cast<cudaStream_t>(stream);
  if (!use_graph) {
    c.st = user;
    c.pdl = true;
    rc = enqueue_prefill(c);
    if (rc) return rc;
    return check_cuda(cudaGetLastError(), "fam_video_prefill launch");
  }
  VCallKey key;
  key.ptrs = {reinterpret_cast<uintptr_t>(io->workspace), reinterpret_cast<uintptr_t>(io->latents),
              reinterpret_cast<uintptr_t>(io->context), reinterpret_cast<uintptr_t>(io->context_mask),
              reinterpret_cast<uintptr_t>(io->rope), reinterpret_cast<uintptr_t>(io->hidden_out),
              reinterpret_cast<uintptr_t>(io->t_out),
              static_cast<uintptr_t>(io->batch), static_cast<uintptr_t>(io->frames),
              static_cast<uintptr_t>(io->height), static_cast<uintptr_t>(io->width),
              static_cast<uintptr_t>(io->context_tokens), static_cast<uintptr_t>(io->first_frame_causal)};
  for (int l = 0; l < e->cfg.num_layers; ++l) {
    key.ptrs.push_back(reinterpret_cast<uintptr_t>(io->cache_k[l]));
    key.ptrs.push_back(reinterpret_cast<uintptr_t>(io->cache_v[l]));
  }
  key.vals.assign(io->timesteps, io->timesteps + io->batch);
  if (e->graph == nullptr || !(key == e->key)) {
    if (e->graph) {
      cudaGraphExecDestroy(e->graph);
      e->graph = nullptr;
    }
    c.st = e->cap_stream;
    c.pdl = true;
    rc = check_cuda(cudaStreamBeginCapture(c.st, cudaStreamCaptureModeThreadLocal), "begin capture");
    if (rc) return rc;
    rc = enqueue_prefill(c);
    cudaGraph_t g = nullptr;
    cudaError_t ce = cudaStreamEndCapture(c.st, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (ce != cudaSuccess) return check_cuda(ce, "end capture");
    ce = cudaGraphInstantiate(&e->graph, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) {
      e->graph = nullptr;
      return check_cuda(ce, "graph instantiate");
    }
    e->key = key;
  }
  return check_cuda(cudaGraphLaunch(e->graph, user), "graph launch");
}

}  // extern "C"
