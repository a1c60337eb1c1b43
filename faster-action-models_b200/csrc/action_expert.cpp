// Host runtime of the action expert: owns the weight tensor maps, lays out the
// caller's workspace, enqueues one action chunk (or one model evaluation) as a
// chain of programmatic-dependent launches, and captures that chain into a
// CUDA graph that is replayed while the call's pointers and sizes repeat.
//
// Launch chain of one Euler step (per block l of L):
//   gemm qkv (split-K) -> qkv_post -> joint attention (video cache ++ action)
//   -> gemm o (split-K) -> resid_norm(gate_msa, norm3) -> gemm cross-q ->
//   rms_rows -> cross attention -> gemm cross-o -> resid_norm(AdaLN mlp)
//   -> gemm ffn.0 (+GELU) -> gemm ffn.2 (split-K) -> resid_norm(gate_mlp, next AdaLN)
// then head + Euler update.  Step-invariant work is hoisted to the chunk
// prologue: the time MLP of every step's timestep, the text embedding and
// every block's cross-attention K/V (RMSNorm'd K) of the context.
#include <string.h>

#include <cmath>
#include <memory>
#include <vector>

#include "../../include/fam.h"
#include "action_fused.h"
#include "fam_internal.h"
#include "fam_kernels.h"

using namespace fam;

namespace {

constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

const __nv_bfloat16* bf(const void* p) { return static_cast<const __nv_bfloat16*>(p); }

// Token-tile width of the chain's split-K weights-as-A GEMMs: 64 for 65..256
// token rows, else the plan's own width.  Measured at 256 rows (batch 8 of 32
// action tokens, graphs over weights beyond L2): 64-wide tiles with fewer
// k-splits beat 256-wide tiles with more — qkv 12.8 -> 8.1 us, o / cross-q /
// cross-o -> 6.1 us, ffn.2 > 13 -> 8.8 us — and leave fewer fp32 partials for
// the row kernel that sums them.
int chain_tile_n(int rows) { return rows > 64 && rows <= 256 ? 64 : 0; }

// Split-K: with 64-wide token tiles about 256 CTAs, at least four 64-wide K
// blocks per split; otherwise tiles x splits fills ~one wave of 148 SMs, at
// least two K blocks per split.
int choose_splits(int n_out, int k, int rows) {
  const int tn = chain_tile_n(rows);
  const int bn = tn > 0 ? tn : gemm_pick_bn(rows);
  const int tiles = ((n_out + 127) / 128) * ((rows + bn - 1) / bn);
  const int kb = (k + 63) / 64;
  const int min_kb = tn > 0 ? 4 : 2;
  int s = tn > 0 ? (256 + tiles / 2) / tiles : 148 / tiles;
  if (s < 1) s = 1;
  if (s > kb / min_kb) s = kb / min_kb > 0 ? kb / min_kb : 1;
  const int kps = (kb + s - 1) / s;
  return (kb + kps - 1) / kps;
}

struct WsLayout {
  size_t x, h, part, q, ka, va, ao, qc, ci, fh, apart, ctr, tmod, sin, th1, th2, cemb, ch1, ckv, vel;
  size_t fsync, fssq, fpart;  // fused-kernel barrier / merge counters, RMS sums, split partials
  size_t fx, fslots;          // fused-kernel bf16 residual [32][D], residual GEMM split partials
  size_t fsync_bytes, fssq_bytes;
  size_t total;
  int s_qkv, s_o, s_cq, s_co, s_f2;
};

// Words of the fused kernel's sync block before its flag lines: go, abort,
// the joint-attention merge counters [N][L][H], the residual tile counters.
size_t fused_sync_words(int N, int L, int H) {
  return 2 + static_cast<size_t>(N) * L * H + 3 * (kFusedMaxD / 128);
}

WsLayout layout(const fam_action_config& c, int B, int Sa, int C, int N) {
  WsLayout w = {};
  const size_t rows = static_cast<size_t>(B) * Sa, crow = static_cast<size_t>(B) * C;
  const int D = c.hidden_dim, HD = c.num_heads * c.head_dim, F = c.ffn_dim;
  w.s_qkv = choose_splits(3 * HD, D, static_cast<int>(rows));
  w.s_o = choose_splits(D, HD, static_cast<int>(rows));
  w.s_cq = choose_splits(HD, D, static_cast<int>(rows));
  w.s_co = choose_splits(D, HD, static_cast<int>(rows));
  w.s_f2 = choose_splits(D, F, static_cast<int>(rows));
  size_t part_elems = 0;
  auto upd = [&](size_t e) { part_elems = e > part_elems ? e : part_elems; };
  upd(static_cast<size_t>(w.s_qkv) * rows * 3 * HD);
  upd(static_cast<size_t>(w.s_o) * rows * D);
  upd(static_cast<size_t>(w.s_cq) * rows * HD);
  upd(static_cast<size_t>(w.s_co) * rows * D);
  upd(static_cast<size_t>(w.s_f2) * rows * D);
  const int nsplit_joint = 8;  // upper bound used for the partial buffer
  size_t apart = attn_partial_bytes(B, c.num_heads, Sa, c.head_dim, 64);
  (void)nsplit_joint;
  const int q_tiles = attn_query_tiles(Sa);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes);
    return o;
  };
  w.x = take(rows * D * 4);
  w.h = take(rows * (D > HD ? D : HD) * 2);
  w.part = take(part_elems * 4);
  w.q = take(rows * HD * 2);
  w.ka = take(rows * HD * 2);
  w.va = take(rows * HD * 2);
  w.ao = take(rows * HD * 2);
  w.qc = take(rows * HD * 2);
  w.ci = take(rows * HD * 2);
  w.fh = take(rows * F * 2);
  w.apart = take(apart);
  w.ctr = take(static_cast<size_t>(B) * c.num_heads * q_tiles * 4);
  w.tmod = take(static_cast<size_t>(N) * 6 * D * 4);
  w.sin = take(static_cast<size_t>(N) * c.freq_dim * 2);
  w.th1 = take(static_cast<size_t>(N) * D * 2);
  w.th2 = take(static_cast<size_t>(N) * D * 2);
  w.cemb = take(crow * D * 2);
  w.ch1 = take(crow * D * 2);
  w.ckv = take(static_cast<size_t>(c.num_layers) * crow * 2 * HD * 2);
  w.vel = take(rows * c.action_dim * 2);
  // fused persistent kernel (batch 1): counters, per-token RMS sums, split partials
  // [go, abort, merge counters, residual tile counters] padded to a 128-byte
  // line, then one flag line per CTA
  w.fsync_bytes = ((fused_sync_words(N, c.num_layers, c.num_heads) + 31) / 32 * 32 +
                   static_cast<size_t>(kFusedMaxCtas) * 32) * 4;
  // RMS sums of squares [N][L][3][32], then the LayerNorm row sums [N][L][3][32][2]
  w.fssq_bytes = static_cast<size_t>(N) * c.num_layers * 3 * kFusedRows * 8 * 3;
  w.fsync = take(w.fsync_bytes);
  w.fssq = take(w.fssq_bytes);
  w.fpart = take(static_cast<size_t>(c.num_heads) * 64 * kFusedRows * 66 * 4);
  w.fx = take(static_cast<size_t>(kFusedRows) * D * 2);
  // residual GEMM split partials: at most max(heads, F / 128) splits per tile
  w.fslots = take(static_cast<size_t>(std::max(c.num_heads, F / 128)) * kFusedRows * D * 4);
  w.total = off;
  return w;
}

// Everything that identifies a captured launch sequence.
struct CallKey {
  std::vector<uintptr_t> ptrs;
  std::vector<float> vals;
  bool operator==(const CallKey& o) const { return ptrs == o.ptrs && vals == o.vals; }
};

}  // namespace

struct fam_action_expert {
  fam_action_config cfg;
  fam_action_weights w;
  std::vector<fam_action_layer> layers;
  cudaStream_t cap_stream = nullptr;
  cudaGraphExec_t graph = nullptr;
  CallKey graph_key;
  int* status = nullptr;
  int launch_count = 0;  // kernels enqueued by the last chunk / step call
  bool has_stacks = false;
  fam_action_stacks stacks = {};
  CUtensorMap tm[6];     // stacked weights for the fused kernel
  int num_sms = 0;  // CTAs of the fused kernel's grid (2-CTA clusters, all co-resident)
  int mode = FAM_ACTION_AUTO;
  int last_path = 0;
  cudaEvent_t kernel_start = nullptr, kernel_stop = nullptr;  // measurement hook
};

namespace {

struct Ctx {
  fam_action_expert* e;
  const fam_action_io* io;
  char* ws;
  WsLayout L;
  int rows, crow;
  cudaStream_t st;
  bool pdl;
};

template <typename T>
T* wsp(const Ctx& c, size_t off) {
  return reinterpret_cast<T*>(c.ws + off);
}

#define FAM_TRY(expr)                                  \
  do {                                                 \
    cudaError_t _e = (expr);                           \
    if (_e != cudaSuccess) return check_cuda(_e, #expr); \
  } while (0)
#define FAM_TRYI(expr)  \
  do {                  \
    int _r = (expr);    \
    if (_r) return _r;  \
  } while (0)
// A kernel launch of the chain (counted for fam_action_launch_count).
#define FAM_LAUNCH(expr)    \
  do {                      \
    FAM_TRY(expr);          \
    ++c.e->launch_count;    \
  } while (0)

// out = act(A-weights x B-activations + bias) or split partials.
int gemm_w(const Ctx& c, const void* W, const void* bias, int n_out, int k, const void* act,
           long long act_ld, int rows, int splits, int act_kind, void* out, long long out_ld,
           bool out_f32) {
  GemmEpilogue e = {};
  e.features_on_a = 1;
  e.act = act_kind;
  e.out = out;
  e.out_sa = 1;
  e.out_sb = out_ld;
  if (splits > 1) {
    e.kind = kEpiPartial;
    e.split_stride = static_cast<long long>(rows) * out_ld;
  } else {
    e.kind = kEpiStore;
    e.out_bf16 = out_f32 ? 0 : 1;
    e.bias = bf(bias);
  }
  GemmPlan p;
  FAM_TRYI(gemm_plan(&p, W, k, act, act_ld, n_out, rows, k, splits, splits > 1 ? chain_tile_n(rows) : 0, e, true,
                     false, c.e->status));
  FAM_LAUNCH(gemm_launch(p, c.st, c.pdl));
  return 0;
}

ModRows step_mod(const Ctx& c, int step, const void* mod_w, int tokens_per_batch) {
  ModRows m = {};
  m.tmod = wsp<float>(c, c.L.tmod) + static_cast<size_t>(step) * 6 * c.e->cfg.hidden_dim;
  m.mod_w = bf(mod_w);
  m.tokens_per_batch = tokens_per_batch;
  m.first_frame_tokens = 0;
  m.bstride = 0;
  m.gstride = 0;
  return m;
}

// Time MLP of every step + text embedding + per-block cross K/V.
int enqueue_prologue(const Ctx& c, const float* timesteps, int N) {
  const fam_action_config& g = c.e->cfg;
  const fam_action_weights& w = c.e->w;
  const int D = g.hidden_dim, HD = g.num_heads * g.head_dim;
  StepTimes st = {};
  for (int i = 0; i < N; ++i) st.t[i] = timesteps[i];
  // First launch of the chain follows a memset node: plain stream order.
  FAM_LAUNCH(launch_sinusoid(st, N, g.freq_dim, wsp<__nv_bfloat16>(c, c.L.sin), c.st, false));
  // time_embedding: Linear -> SiLU -> Linear ; time_projection: SiLU -> Linear
  FAM_TRYI(gemm_w(c, w.time0_w, w.time0_b, D, g.freq_dim, wsp<void>(c, c.L.sin), g.freq_dim, N, 1,
                  kActSilu, wsp<void>(c, c.L.th1), D, false));
  FAM_TRYI(gemm_w(c, w.time2_w, w.time2_b, D, D, wsp<void>(c, c.L.th1), D, N, 1, kActSilu,
                  wsp<void>(c, c.L.th2), D, false));
  FAM_TRYI(gemm_w(c, w.tproj_w, w.tproj_b, 6 * D, D, wsp<void>(c, c.L.th2), D, N, 1, kActNone,
                  wsp<void>(c, c.L.tmod), 6 * D, true));
  if (c.crow > 0) {
    // text_embedding: Linear -> GELU(tanh) -> Linear
    FAM_TRYI(gemm_w(c, w.text0_w, w.text0_b, D, g.text_dim, c.io->context, g.text_dim, c.crow, 1,
                    kActGeluTanh, wsp<void>(c, c.L.ch1), D, false));
    FAM_TRYI(gemm_w(c, w.text2_w, w.text2_b, D, D, wsp<void>(c, c.L.ch1), D, c.crow, 1, kActNone,
                    wsp<void>(c, c.L.cemb), D, false));
    // Cross K / V of every block, context-token major: ckv[row][l * 2HD + (K | V)]
    // (row = b * C + t); the K half RMSNorm'd with block l's norm_k.
    const int L = g.num_layers;
    const long long ld = static_cast<long long>(L) * 2 * HD;
    __nv_bfloat16* ckv_all = wsp<__nv_bfloat16>(c, c.L.ckv);
    const fam_action_stacks& s = c.e->stacks;
    if (c.e->has_stacks && s.ckv_w != nullptr && s.ckv_b != nullptr && s.cnorm_k != nullptr) {
      // one GEMM over the stacked projections, one RMSNorm launch over (row, block)
      FAM_TRYI(gemm_w(c, s.ckv_w, s.ckv_b, L * 2 * HD, D, wsp<void>(c, c.L.cemb), D, c.crow, 1,
                      kActNone, ckv_all, ld, false));
      RmsRowsArgs r = {};
      r.nsplit = 0;
      r.in = ckv_all;
      r.in_stride = 2 * HD;  // (row, block) slice rr = row * L + l starts at rr * 2HD
      r.w = bf(s.cnorm_k);
      r.w_period = L;
      r.w_stride = HD;
      r.out = ckv_all;
      r.out_stride = 2 * HD;
      r.N = HD;
      r.eps = g.eps;
      FAM_LAUNCH(launch_rms_rows(r, c.crow * L, c.st, c.pdl));
    } else {
      for (int l = 0; l < L; ++l) {
        const fam_action_layer& ly = c.e->layers[l];
        __nv_bfloat16* ckv = ckv_all + static_cast<size_t>(l) * 2 * HD;
        FAM_TRYI(gemm_w(c, ly.ckv_w, ly.ckv_b, 2 * HD, D, wsp<void>(c, c.L.cemb), D, c.crow, 1,
                        kActNone, ckv, ld, false));
        RmsRowsArgs r = {};
        r.nsplit = 0;
        r.in = ckv;
        r.in_stride = ld;
        r.w = bf(ly.cnorm_k);
        r.out = ckv;
        r.out_stride = ld;
        r.N = HD;
        r.eps = g.eps;
        FAM_LAUNCH(launch_rms_rows(r, c.crow, c.st, c.pdl));
      }
    }
  }
  return 0;
}

// One model evaluation at step index `step`; velocity -> vel; Euler when apply.
int enqueue_step(const Ctx& c, int step, const void* latent, void* vel, float delta, bool apply) {
  const fam_action_config& g = c.e->cfg;
  const fam_action_weights& w = c.e->w;
  const fam_action_io& io = *c.io;
  const int D = g.hidden_dim, HD = g.num_heads * g.head_dim, F = g.ffn_dim, Lyr = g.num_layers;
  const int rows = c.rows, Sa = io.action_tokens;
  float* x = wsp<float>(c, c.L.x);
  __nv_bfloat16* h = wsp<__nv_bfloat16>(c, c.L.h);
  float* part = wsp<float>(c, c.L.part);

  EncodeArgs ea = {};
  ea.latent = bf(latent);
  ea.enc_w = bf(w.enc_w);
  ea.enc_b = bf(w.enc_b);
  ea.x = x;
  ea.h = h;
  ea.mod = step_mod(c, step, c.e->layers[0].modulation, Sa);
  ea.A = g.action_dim;
  ea.D = D;
  ea.eps = g.eps;
  FAM_LAUNCH(launch_encode_adaln(ea, rows, c.st, c.pdl));

  const float scale_log2 = 1.4426950408889634f / std::sqrt(static_cast<float>(g.head_dim));
  for (int l = 0; l < Lyr; ++l) {
    const fam_action_layer& ly = c.e->layers[l];
    // --- self / joint attention
    FAM_TRYI(gemm_w(c, ly.qkv_w, nullptr, 3 * HD, D, h, D, rows, c.L.s_qkv, kActNone, part, 3 * HD, true));
    QkvPostArgs qa = {};
    qa.partials = part;
    qa.split_stride = static_cast<long long>(rows) * 3 * HD;
    qa.nsplit = c.L.s_qkv;
    qa.bias = bf(ly.qkv_b);
    qa.norm_q = bf(ly.norm_q);
    qa.norm_k = bf(ly.norm_k);
    qa.rope = static_cast<const float2*>(w.rope);
    qa.rows_per_batch = Sa;
    qa.q_out = wsp<__nv_bfloat16>(c, c.L.q);
    qa.k_out = wsp<__nv_bfloat16>(c, c.L.ka);
    qa.v_out = wsp<__nv_bfloat16>(c, c.L.va);
    qa.out_stride = HD;
    qa.HD = HD;
    qa.head_dim = g.head_dim;
    qa.eps = g.eps;
    if (c.L.s_qkv == 1) {  // single split: partial buffer holds fp32 (no bias)
      qa.nsplit = 1;
    }
    FAM_LAUNCH(launch_qkv_post(qa, rows, c.st, c.pdl));

    AttnArgs aa = {};
    aa.q = wsp<__nv_bfloat16>(c, c.L.q);
    aa.q_bs = static_cast<long long>(Sa) * HD;
    aa.q_ts = HD;
    if (io.video_tokens > 0) {
      aa.k1 = bf(io.video_k[l]);
      aa.v1 = bf(io.video_v[l]);
      aa.kv1_bs = io.video_batch_stride;
      aa.kv1_ts = io.video_token_stride;
      aa.S1 = io.video_tokens;
      aa.kv1_const = 1;  // the video cache is a call input
    }
    aa.k2 = wsp<__nv_bfloat16>(c, c.L.ka);
    aa.v2 = wsp<__nv_bfloat16>(c, c.L.va);
    aa.kv2_bs = static_cast<long long>(Sa) * HD;
    aa.kv2_ts = HD;
    aa.S2 = Sa;
    aa.mask2d = io.attn_mask;
    aa.mask_rs = io.video_tokens + Sa;
    aa.Sq = Sa;
    aa.H = g.num_heads;
    aa.scale_log2 = scale_log2;
    aa.out = wsp<__nv_bfloat16>(c, c.L.ao);
    aa.out_bs = static_cast<long long>(Sa) * HD;
    aa.out_ts = HD;
    aa.part = wsp<float>(c, c.L.apart);
    aa.counters = wsp<int>(c, c.L.ctr);
    const int skv = io.video_tokens + Sa;
    aa.nsplit = attn_auto_splits(io.batch * g.num_heads * attn_query_tiles(Sa), skv,
                                 &aa.keys_per_split);
    aa.status = c.e->status;
    FAM_LAUNCH(launch_attention_auto(aa, io.batch, g.head_dim, c.st, c.pdl));

    FAM_TRYI(gemm_w(c, ly.o_w, nullptr, D, HD, aa.out, HD, rows, c.L.s_o, kActNone, part, D, true));
    ResidNormArgs r1 = {};
    r1.x = x;
    r1.round_residual = 1;  // the reference keeps the residual in bf16
    r1.partials = part;
    r1.split_stride = static_cast<long long>(rows) * D;
    r1.nsplit = c.L.s_o;
    r1.bias = bf(ly.o_b);
    r1.gate_chunk = 2;  // gate_msa
    r1.norm_mode = kNormAffine;
    r1.norm_w = bf(ly.norm3_w);
    r1.norm_b = bf(ly.norm3_b);
    r1.mod = step_mod(c, step, ly.modulation, Sa);
    r1.h = h;
    r1.h_stride = D;
    r1.D = D;
    r1.eps = g.eps;
    FAM_LAUNCH(launch_resid_norm(r1, rows, c.st, c.pdl));

    // --- cross attention (no gate)
    if (c.crow > 0) {
      FAM_TRYI(gemm_w(c, ly.cq_w, nullptr, HD, D, h, D, rows, c.L.s_cq, kActNone, part, HD, true));
      RmsRowsArgs rq = {};
      rq.partials = part;
      rq.split_stride = static_cast<long long>(rows) * HD;
      rq.nsplit = c.L.s_cq;
      rq.bias = bf(ly.cq_b);
      rq.w = bf(ly.cnorm_q);
      rq.out = wsp<__nv_bfloat16>(c, c.L.qc);
      rq.out_stride = HD;
      rq.N = HD;
      rq.eps = g.eps;
      FAM_LAUNCH(launch_rms_rows(rq, rows, c.st, c.pdl));
      AttnArgs ca = {};
      ca.q = rq.out;
      ca.q_bs = static_cast<long long>(Sa) * HD;
      ca.q_ts = HD;
      // context-token-major cross K / V of every block (prologue layout)
      const long long cld = static_cast<long long>(g.num_layers) * 2 * HD;
      const __nv_bfloat16* ckv = wsp<__nv_bfloat16>(c, c.L.ckv) + static_cast<size_t>(l) * 2 * HD;
      ca.k1 = ckv;
      ca.v1 = ckv + HD;
      ca.kv1_bs = static_cast<long long>(io.context_tokens) * cld;
      ca.kv1_ts = cld;
      ca.S1 = io.context_tokens;
      ca.key_mask = io.context_mask;
      ca.key_mask_bs = io.context_tokens;
      ca.Sq = Sa;
      ca.H = g.num_heads;
      ca.scale_log2 = scale_log2;
      ca.out = wsp<__nv_bfloat16>(c, c.L.ci);
      ca.out_bs = static_cast<long long>(Sa) * HD;
      ca.out_ts = HD;
      ca.nsplit = 1;
      ca.keys_per_split = io.context_tokens;
      ca.counters = wsp<int>(c, c.L.ctr);
      ca.part = wsp<float>(c, c.L.apart);
      ca.status = c.e->status;
      FAM_LAUNCH(launch_attention_auto(ca, io.batch, g.head_dim, c.st, c.pdl));
      FAM_TRYI(gemm_w(c, ly.co_w, nullptr, D, HD, ca.out, HD, rows, c.L.s_co, kActNone, part, D, true));
    }
    ResidNormArgs r2 = {};
    r2.x = x;
    r2.round_residual = 1;  // the reference keeps the residual in bf16
    r2.partials = c.crow > 0 ? part : nullptr;
    r2.split_stride = static_cast<long long>(rows) * D;
    r2.nsplit = c.L.s_co;
    r2.bias = bf(ly.co_b);
    r2.gate_chunk = -1;
    r2.norm_mode = kNormAdaLN;
    r2.shift_chunk = 3;  // shift_mlp, scale_mlp
    r2.nmod = step_mod(c, step, ly.modulation, Sa);
    r2.h = h;
    r2.h_stride = D;
    r2.D = D;
    r2.eps = g.eps;
    FAM_LAUNCH(launch_resid_norm(r2, rows, c.st, c.pdl));

    // --- FFN
    FAM_TRYI(gemm_w(c, ly.ffn0_w, ly.ffn0_b, F, D, h, D, rows, 1, kActGeluTanh,
                    wsp<void>(c, c.L.fh), F, false));
    FAM_TRYI(gemm_w(c, ly.ffn2_w, nullptr, D, F, wsp<void>(c, c.L.fh), F, rows, c.L.s_f2, kActNone,
                    part, D, true));
    ResidNormArgs r3 = {};
    r3.x = x;
    r3.round_residual = 1;  // the reference keeps the residual in bf16
    r3.partials = part;
    r3.split_stride = static_cast<long long>(rows) * D;
    r3.nsplit = c.L.s_f2;
    r3.bias = bf(ly.ffn2_b);
    r3.gate_chunk = 5;  // gate_mlp
    r3.mod = step_mod(c, step, ly.modulation, Sa);
    r3.D = D;
    r3.eps = g.eps;
    if (l + 1 < Lyr) {  // next block's AdaLN (shift_msa, scale_msa)
      r3.norm_mode = kNormAdaLN;
      r3.shift_chunk = 0;
      r3.nmod = step_mod(c, step, c.e->layers[l + 1].modulation, Sa);
      r3.h = h;
      r3.h_stride = D;
    } else {
      r3.norm_mode = kNormNone;
    }
    FAM_LAUNCH(launch_resid_norm(r3, rows, c.st, c.pdl));
  }
  HeadArgs ha = {};
  ha.x = x;
  ha.head_w = bf(w.head_w);
  ha.head_b = bf(w.head_b);
  ha.velocity = static_cast<__nv_bfloat16*>(vel);
  ha.latent = const_cast<__nv_bfloat16*>(bf(latent));
  ha.delta = delta;
  ha.apply_euler = apply ? 1 : 0;
  ha.rows = rows;
  ha.A = g.action_dim;
  ha.D = D;
  FAM_LAUNCH(launch_head_euler(ha, c.st, c.pdl));
  return 0;
}

int validate_io(const fam_action_expert* e, const fam_action_io* io, int N) {
  if (e == nullptr || io == nullptr) return set_error("null expert or io");
  if (io->batch <= 0 || io->action_tokens <= 0) return set_error("batch and action_tokens must be > 0");
  if (io->action_tokens > 1024) return set_error("action_tokens %d exceeds the RoPE table", io->action_tokens);
  if (io->action_tokens > e->w.rope_positions)
    return set_error("rope table has %d positions, need %d", e->w.rope_positions, io->action_tokens);
  if (io->context_tokens < 0 || (io->context_tokens > 0 && io->context == nullptr))
    return set_error("context missing");
  if (io->video_tokens < 0 || (io->video_tokens > 0 && (io->video_k == nullptr || io->video_v == nullptr)))
    return set_error("video cache pointers missing");
  if (N <= 0 || N > kMaxSteps) return set_error("num_steps must be in [1, %d]", kMaxSteps);
  size_t need = layout(e->cfg, io->batch, io->action_tokens, io->context_tokens, N).total;
  if (io->workspace == nullptr || io->workspace_bytes < need)
    return set_error("workspace too small: %zu bytes given, %zu needed", io->workspace_bytes, need);
  return 0;
}

int enqueue_chunk(const Ctx& c, void* latent, const float* ts, const float* ds, int N, void* trace) {
  c.e->launch_count = 0;
  const size_t ctr_bytes = static_cast<size_t>(c.io->batch) * c.e->cfg.num_heads *
                           attn_query_tiles(c.io->action_tokens) * 4;
  FAM_TRY(cudaMemsetAsync(wsp<void>(c, c.L.ctr), 0, ctr_bytes, c.st));
  FAM_TRYI(enqueue_prologue(c, ts, N));
  const size_t vel_elems = static_cast<size_t>(c.rows) * c.e->cfg.action_dim;
  for (int i = 0; i < N; ++i) {
    void* vel = trace != nullptr ? static_cast<void*>(static_cast<__nv_bfloat16*>(trace) + i * vel_elems)
                                 : wsp<void>(c, c.L.vel);
    FAM_TRYI(enqueue_step(c, i, latent, vel, ds[i], true));
  }
  return 0;
}

// Whether the fused persistent kernel can run this call.
bool fused_eligible(const fam_action_expert* e, const fam_action_io* io, int N) {
  const fam_action_config& g = e->cfg;
  const int HD = g.num_heads * g.head_dim;
  if (!e->has_stacks || e->num_sms < 64 || e->num_sms > kFusedMaxCtas) return false;
  if (io->batch != 1 || io->action_tokens > kFusedRows || g.head_dim != 64 || g.action_dim > 16) return false;
  if (g.hidden_dim % 512 || HD % 128 || g.ffn_dim % 128 || g.hidden_dim > 1024) return false;
  if (g.num_layers > kFusedMaxLayers || io->context_tokens > 256 || N > kMaxSteps) return false;
  if (3 * HD / 128 + HD / 128 + g.ffn_dim / 128 > e->num_sms / 2) return false;  // one pair item per pair and phase
  const int skv = io->video_tokens + io->action_tokens;
  if ((skv + kFusedKeysPerSplit - 1) / kFusedKeysPerSplit > kFusedMaxSplits) return false;
  if (io->video_tokens > 0 && (io->video_token_stride % 8)) return false;
  return true;
}

int enqueue_chunk_fused(const Ctx& c, void* latent, const float* ts, const float* ds, int N,
                        void* trace) {
  fam_action_expert* e = c.e;
  const fam_action_config& g = e->cfg;
  const fam_action_io& io = *c.io;
  const int HD = g.num_heads * g.head_dim;
  e->launch_count = 0;
  FAM_TRY(cudaMemsetAsync(wsp<void>(c, c.L.fsync), 0, c.L.fsync_bytes, c.st));
  FAM_TRY(cudaMemsetAsync(wsp<void>(c, c.L.fssq), 0, c.L.fssq_bytes, c.st));
  FAM_TRYI(enqueue_prologue(c, ts, N));
  FusedArgs a;
  memset(&a, 0, sizeof(a));
  for (int p = 0; p < 6; ++p) a.tm[p] = e->tm[p];
  const fam_action_stacks& s = e->stacks;
  a.qkv_b = bf(s.qkv_b);
  a.o_b = bf(s.o_b);
  a.cq_b = bf(s.cq_b);
  a.co_b = bf(s.co_b);
  a.ffn0_b = bf(s.ffn0_b);
  a.ffn2_b = bf(s.ffn2_b);
  a.norm_q = bf(s.norm_q);
  a.norm_k = bf(s.norm_k);
  a.cnorm_q = bf(s.cnorm_q);
  a.norm3_w = bf(s.norm3_w);
  a.norm3_b = bf(s.norm3_b);
  a.modulation = bf(s.modulation);
  a.enc_w = bf(e->w.enc_w);
  a.enc_b = bf(e->w.enc_b);
  a.head_w = bf(e->w.head_w);
  a.head_b = bf(e->w.head_b);
  a.tmod = wsp<float>(c, c.L.tmod);
  a.rope = static_cast<const float2*>(e->w.rope);
  for (int l = 0; l < g.num_layers; ++l) {
    a.vk[l] = io.video_tokens > 0 ? bf(io.video_k[l]) : nullptr;
    a.vv[l] = io.video_tokens > 0 ? bf(io.video_v[l]) : nullptr;
  }
  a.v_ts = io.video_token_stride;
  a.Sv = io.video_tokens;
  a.mask2d = io.attn_mask;
  a.ckv = wsp<__nv_bfloat16>(c, c.L.ckv);
  a.ctx_mask = io.context_mask;
  a.C = io.context_tokens;
  a.x = wsp<__nv_bfloat16>(c, c.L.fx);
  a.slots = wsp<float>(c, c.L.fslots);
  a.q = wsp<__nv_bfloat16>(c, c.L.q);
  a.ka = wsp<__nv_bfloat16>(c, c.L.ka);
  a.va = wsp<__nv_bfloat16>(c, c.L.va);
  a.ao = wsp<__nv_bfloat16>(c, c.L.ao);
  a.qc = wsp<__nv_bfloat16>(c, c.L.qc);
  a.ci = wsp<__nv_bfloat16>(c, c.L.ci);
  a.fh = wsp<__nv_bfloat16>(c, c.L.fh);
  a.ssq = wsp<double>(c, c.L.fssq);
  a.lnstat = a.ssq + static_cast<size_t>(N) * g.num_layers * 3 * kFusedRows;
  a.apart = wsp<float>(c, c.L.fpart);
  a.sync = wsp<unsigned>(c, c.L.fsync);
  a.tile_ctr = a.sync + 2 + static_cast<size_t>(N) * g.num_layers * g.num_heads;
  a.flags = a.sync + (fused_sync_words(N, g.num_layers, g.num_heads) + 31) / 32 * 32;
  a.status = e->status;
  a.latent = static_cast<__nv_bfloat16*>(latent);
  a.trace = static_cast<__nv_bfloat16*>(trace);
  for (int i = 0; i < N; ++i) a.deltas.t[i] = ds[i];
  a.N = N;
  a.L = g.num_layers;
  a.R = io.action_tokens;
  a.Sa = io.action_tokens;
  a.D = g.hidden_dim;
  a.HD = HD;
  a.H = g.num_heads;
  a.hd = g.head_dim;
  a.F = g.ffn_dim;
  a.A = g.action_dim;
  {
    // joint-attention splits: as many per head as one wave of CTAs holds
    // (at most kFusedMaxSplits), each a whole number of 32-key steps and at
    // most kFusedKeysPerSplit keys -- a short key list (a visible prefix of
    // the cache) then spreads over more, smaller splits
    const int skv = io.video_tokens + io.action_tokens;
    const int cap = std::min(kFusedMaxSplits, std::max(1, e->num_sms / g.num_heads));
    int kps = ((skv + cap - 1) / cap + 31) / 32 * 32;
    kps = std::min(kFusedKeysPerSplit, std::max(32, kps));
    a.kps = kps;
    a.splits = (skv + kps - 1) / kps;
  }
  a.eps = g.eps;
  a.scale_log2 = 1.4426950408889634f / std::sqrt(static_cast<float>(g.head_dim));
  // measurement hook: plain (not captured) calls only
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  FAM_TRY(cudaStreamIsCapturing(c.st, &cap));
  const bool timed = e->kernel_start != nullptr && cap == cudaStreamCaptureStatusNone;
  if (timed) FAM_TRY(cudaEventRecord(e->kernel_start, c.st));
  FAM_LAUNCH(launch_fused_chunk(a, e->num_sms, c.st));
  if (timed) FAM_TRY(cudaEventRecord(e->kernel_stop, c.st));
  return 0;
}

}  // namespace

extern "C" {

int fam_action_set_mode(fam_action_expert* e, int32_t mode) {
  if (e == nullptr || mode < FAM_ACTION_AUTO || mode > FAM_ACTION_FUSED) return set_error("bad mode");
  if (mode == FAM_ACTION_FUSED && !e->has_stacks) return set_error("fused mode needs stacked weights");
  e->mode = mode;
  return FAM_OK;
}

int fam_action_last_path(const fam_action_expert* e, int32_t* path) {
  if (e == nullptr || path == nullptr) return set_error("null argument");
  *path = e->last_path;
  return FAM_OK;
}

int fam_action_set_kernel_events(fam_action_expert* e, void* start_event, void* stop_event) {
  if (e == nullptr || (start_event == nullptr) != (stop_event == nullptr))
    return set_error("fam_action_set_kernel_events: both events or neither");
  e->kernel_start = static_cast<cudaEvent_t>(start_event);
  e->kernel_stop = static_cast<cudaEvent_t>(stop_event);
  return FAM_OK;
}

int fam_action_expert_create(const fam_action_config* cfg, const fam_action_weights* w,
                             fam_action_expert** out) {
  if (cfg == nullptr || w == nullptr || out == nullptr) return set_error("null argument");
  if (cfg->head_dim != 64 && cfg->head_dim != 128)
    return set_error("head_dim %d unsupported (64 or 128)", cfg->head_dim);
  if (cfg->hidden_dim % 64 || cfg->ffn_dim % 64 || cfg->text_dim % 8 || cfg->freq_dim % 64)
    return set_error("hidden/ffn dims must be multiples of 64, text_dim of 8");
  if (cfg->num_layers <= 0 || w->layers == nullptr) return set_error("no layers");
  if (cfg->action_dim > 64) return set_error("action_dim must be <= 64");
  if (w->rope == nullptr || w->rope_positions <= 0) return set_error("missing RoPE table");
  int rc0 = 0;
  auto e = std::make_unique<fam_action_expert>();
  e->cfg = *cfg;
  e->w = *w;
  e->layers.assign(w->layers, w->layers + cfg->num_layers);
  e->w.layers = e->layers.data();
  rc0 = check_cuda(gemm_init_attributes(), "gemm attributes");
  if (rc0) return rc0;
  rc0 = check_cuda(attn_init_attributes(), "attention attributes");
  if (rc0) return rc0;
  e->status = device_status_word();
  if (e->status == nullptr) return set_error("could not allocate the device status word");
  int rc = check_cuda(cudaStreamCreateWithFlags(&e->cap_stream, cudaStreamNonBlocking), "stream create");
  if (rc) return rc;
  if (w->stacks != nullptr) {
    const fam_action_stacks& s = *w->stacks;
    const int D = cfg->hidden_dim, HD = cfg->num_heads * cfg->head_dim, F = cfg->ffn_dim;
    const uint64_t L = static_cast<uint64_t>(cfg->num_layers);
    const void* base[6] = {s.qkv_w, s.o_w, s.cq_w, s.co_w, s.ffn0_w, s.ffn2_w};
    const uint64_t rows[6] = {3ull * HD, static_cast<uint64_t>(D), static_cast<uint64_t>(HD),
                              static_cast<uint64_t>(D), static_cast<uint64_t>(F), static_cast<uint64_t>(D)};
    const uint64_t cols[6] = {static_cast<uint64_t>(D), static_cast<uint64_t>(HD), static_cast<uint64_t>(D),
                              static_cast<uint64_t>(HD), static_cast<uint64_t>(D), static_cast<uint64_t>(F)};
    bool ok = true;
    for (int p = 0; p < 6 && ok; ++p)
      ok = base[p] != nullptr && make_tmap_bf16_2d(&e->tm[p], base[p], L * rows[p], cols[p], cols[p], 128);
    if (ok) {
      e->stacks = s;
      e->w.stacks = &e->stacks;
      e->has_stacks = true;
      rc = check_cuda(fused_init_attributes(), "fused kernel attributes");
      if (rc) return rc;
      e->num_sms = fused_max_ctas();  // co-resident CTAs in 2-CTA clusters (0: fused path off)
    } else {
      e->w.stacks = nullptr;
    }
  }
  *out = e.release();
  return FAM_OK;
}

int fam_action_expert_destroy(fam_action_expert* e) {
  if (e == nullptr) return FAM_OK;
  if (e->graph) cudaGraphExecDestroy(e->graph);
  if (e->cap_stream) cudaStreamDestroy(e->cap_stream);
  delete e;
  return FAM_OK;
}

int fam_action_workspace_size(const fam_action_expert* e, int32_t batch, int32_t action_tokens,
                              int32_t context_tokens, int32_t max_steps, size_t* bytes) {
  if (e == nullptr || bytes == nullptr) return set_error("null argument");
  if (batch <= 0 || action_tokens <= 0 || context_tokens < 0 || max_steps <= 0)
    return set_error("bad sizes");
  *bytes = layout(e->cfg, batch, action_tokens, context_tokens, max_steps).total;
  return FAM_OK;
}

int fam_action_chunk(fam_action_expert* e, const fam_action_io* io, void* latent,
                     const float* timesteps, const float* deltas, int32_t num_steps,
                     void* velocity_trace, int32_t use_graph, void* stream) {
  FAM_TRYI(validate_io(e, io, num_steps));
  if (latent == nullptr || timesteps == nullptr || deltas == nullptr) return set_error("null latent/schedule");
  Ctx c;
  c.e = e;
  c.io = io;
  c.ws = static_cast<char*>(io->workspace);
  c.L = layout(e->cfg, io->batch, io->action_tokens, io->context_tokens, num_steps);
  c.rows = io->batch * io->action_tokens;
  c.crow = io->batch * io->context_tokens;
  cudaStream_t user = static_cast<cudaStream_t>(stream);
  const bool fused_ok = fused_eligible(e, io, num_steps);
  if (e->mode == FAM_ACTION_FUSED && !fused_ok)
    return set_error("fam_action_chunk: the fused kernel cannot run this call (batch 1, <= 32 tokens, "
                     "head_dim 64, widths multiple of 128, stacked weights)");
  const bool fused = fused_ok && e->mode != FAM_ACTION_CHAIN;
  e->last_path = fused ? 2 : 1;
  auto enqueue = [&](const Ctx& cc) {
    return fused ? enqueue_chunk_fused(cc, latent, timesteps, deltas, num_steps, velocity_trace)
                 : enqueue_chunk(cc, latent, timesteps, deltas, num_steps, velocity_trace);
  };
  if (!use_graph) {
    c.st = user;
    c.pdl = true;
    FAM_TRYI(enqueue(c));
    return check_cuda(cudaGetLastError(), "fam_action_chunk launch");
  }
  CallKey key;
  key.ptrs = {reinterpret_cast<uintptr_t>(io->workspace), reinterpret_cast<uintptr_t>(latent),
              reinterpret_cast<uintptr_t>(io->context), reinterpret_cast<uintptr_t>(io->context_mask),
              reinterpret_cast<uintptr_t>(io->attn_mask), reinterpret_cast<uintptr_t>(velocity_trace),
              static_cast<uintptr_t>(io->batch), static_cast<uintptr_t>(io->action_tokens),
              static_cast<uintptr_t>(io->context_tokens), static_cast<uintptr_t>(io->video_tokens),
              static_cast<uintptr_t>(io->video_batch_stride), static_cast<uintptr_t>(io->video_token_stride),
              static_cast<uintptr_t>(num_steps), static_cast<uintptr_t>(fused ? 2 : 1)};
  for (int l = 0; io->video_tokens > 0 && l < e->cfg.num_layers; ++l) {
    key.ptrs.push_back(reinterpret_cast<uintptr_t>(io->video_k[l]));
    key.ptrs.push_back(reinterpret_cast<uintptr_t>(io->video_v[l]));
  }
  key.vals.assign(timesteps, timesteps + num_steps);
  key.vals.insert(key.vals.end(), deltas, deltas + num_steps);
  if (e->graph == nullptr || !(key == e->graph_key)) {
    if (e->graph) {
      cudaGraphExecDestroy(e->graph);
      e->graph = nullptr;
    }
    c.st = e->cap_stream;
    c.pdl = true;
    FAM_TRY(cudaStreamBeginCapture(c.st, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue(c);
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
    e->graph_key = key;
  }
  return check_cuda(cudaGraphLaunch(e->graph, user), "graph launch");
}

int fam_action_launch_count(const fam_action_expert* e, int32_t* count) {
  if (e == nullptr || count == nullptr) return set_error("null argument");
  *count = e->launch_count;
  return FAM_OK;
}

int fam_action_denoise_step(fam_action_expert* e, const fam_action_io* io, const void* latent,
                            float timestep, void* velocity, void* stream) {
  FAM_TRYI(validate_io(e, io, 1));
  if (latent == nullptr || velocity == nullptr) return set_error("null latent/velocity");
  Ctx c;
  c.e = e;
  c.io = io;
  c.ws = static_cast<char*>(io->workspace);
  c.L = layout(e->cfg, io->batch, io->action_tokens, io->context_tokens, 1);
  c.rows = io->batch * io->action_tokens;
  c.crow = io->batch * io->context_tokens;
  c.st = static_cast<cudaStream_t>(stream);
  c.pdl = true;
  const size_t ctr_bytes = static_cast<size_t>(io->batch) * e->cfg.num_heads * attn_query_tiles(io->action_tokens) * 4;
  e->launch_count = 0;
  FAM_TRY(cudaMemsetAsync(wsp<void>(c, c.L.ctr), 0, ctr_bytes, c.st));
  FAM_TRYI(enqueue_prologue(c, &timestep, 1));
  FAM_TRYI(enqueue_step(c, 0, latent, velocity, 0.0f, false));
  return check_cuda(cudaGetLastError(), "fam_action_denoise_step launch");
}

}  // extern "C"
