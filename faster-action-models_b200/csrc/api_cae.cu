// C ABI of the compact action expert (fam_cae_*) and the Action-VAE decoder.
#include <string.h>

#include "../../include/fam.h"
#include "fam_cae.h"
#include "fam_internal.h"

using namespace fam;

namespace {

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// Workspace: context K | context V | slice partial sums | packed block weights | status word.
struct CaeWsLayout {
  size_t k, v, part, wpack, status, total;
};

CaeWsLayout cae_ws_layout(const fam_action_config& c, int B, int C) {
  CaeWsLayout w;
  // rows of H*d + 8 floats cover both the plain and the padded (staged) layouts
  const size_t kv = align256(static_cast<size_t>(c.num_layers) * B * C * (c.num_heads * c.head_dim + 8) * sizeof(float));
  CaeStagePlan p;
  memset(&p, 0, sizeof(p));
  cae_tensor_table(c.hidden_dim, c.num_heads * c.head_dim, c.ffn_dim, &p);
  w.k = 0;
  w.v = kv;
  w.part = 2 * kv;
  w.wpack = w.part + align256(static_cast<size_t>(kCaeCtxSlices) * B * C * c.hidden_dim * sizeof(float));
  w.status = w.wpack + align256(static_cast<size_t>(c.num_layers) * (p.a_floats + p.f_floats) * sizeof(float));
  w.total = w.status + 256;
  return w;
}

size_t cae_ws(const fam_action_config& c, int B, int C) { return cae_ws_layout(c, B, C).total; }

int check_cae(const fam_action_config* c) {
  if (c == nullptr) return set_error("cae: null config");
  const int HD = c->num_heads * c->head_dim;
  if (c->hidden_dim > kCaeMaxD || HD > kCaeMaxHD || c->head_dim > kCaeMaxHd || c->head_dim % 2 ||
      c->ffn_dim > kCaeMaxF || c->num_layers > kCaeMaxLayers || c->num_layers <= 0 ||
      c->action_dim > 64 || c->freq_dim > 256 || c->freq_dim % 2)
    return set_error("cae: configuration exceeds the compact-expert limits (hidden<=64, H*d<=64, "
                     "d<=32, ffn<=256, blocks<=32, action<=64, freq<=256)");
  return 0;
}

}  // namespace

extern "C" {

int fam_cae_workspace_size(const fam_action_config* cfg, int32_t batch, int32_t context_tokens,
                           size_t* bytes) {
  int rc = check_cae(cfg);
  if (rc) return rc;
  if (bytes == nullptr || batch <= 0 || context_tokens < 0) return set_error("cae: bad sizes");
  *bytes = cae_ws(*cfg, batch, context_tokens > 0 ? context_tokens : 1);
  return FAM_OK;
}

}  // extern "C"

namespace {

// Whether the decode can run in the staged step kernel's epilogue: one
// upsampling stage of stride 2 or 4, the sample's latents as the decoder input,
// whole GroupNorm groups per CTA of the cluster, register-tiled conv tasks of
// 32 channels x 16 positions that divide the 32 warps, the staged weights within a staging
// buffer, and the decode's buffers in the step kernel's dead ones (everything
// below the latent rows).
bool cae_decode_fusable(const CaeStepArgs& sa, const fam_decoder_config& dc, const fam_decoder_weights& dw) {
  if (sa.wpack == nullptr || dw.num_stages != 1 || dw.stages == nullptr) return false;
  const int s = dw.stages[0].stride, h = dc.hidden, nc = sa.plan.nc, T = dc.num_tokens, Z = dc.latent_dim;
  if ((s != 2 && s != 4) || T != sa.S || Z != sa.A || h % 4 || h % nc) return false;
  const int G = h < 8 ? h : 8, cg = h / G, ch = h / nc, Lo = T * s, K = 2 * s;
  if (ch % cg || ch / cg > 32 || ch % 32 || Lo % 16) return false;
  const int nt = (ch / 32) * (Lo / 16);                                    // conv tasks (DecTask)
  if (nt > 32 || 32 % nt) return false;
  if (ch * (4 * 3 + 4) > kDecChunk || ch * K > kDecChunk) return false;    // one staged chunk fits
  if (32 / nt * 16 * 33 * nt > kDecStages * kDecChunk) return false;       // split partials
  if (Z % 4 || h * Z > kDecChunk || T * Z > ch * Lo) return false;         // input_proj staging
  if (dc.action_horizon <= 0 || dc.action_dim <= 0 || dc.action_dim * h > 2 * kDecChunk) return false;
  CaeDecode d;
  memset(&d, 0, sizeof(d));
  d.hidden = h;
  d.tokens = T;
  d.stride = s;
  return cae_decode_floats(d, nc) <= sa.plan.o_lat;
}

// FAM_DECODE_AUTO's rule.  The epilogue decodes each sample on its own
// cluster (at most 4 SMs), so its time is flat in the batch; the separate
// launches spread over h / 4 CTAs per sample and grow with it.  Measured on
// B200 (config-0 expert, 4 Euler steps, 1760 x 3072 features): batch 1,
// hidden 256: 747.8 us epilogue against 718.2 us separate (hidden 128: 708.2
// against 708.0); batch 16, hidden 256: 1486.0 against 1578.2 us (hidden 128:
// 1437.5 against 1482.0).  The crossover at hidden 256 is near batch 4.
bool cae_decode_auto_fuses(int batch) { return batch >= 4; }

int cae_chunk_impl(const fam_action_config* cfg, const fam_cae_weights* w, int32_t batch, int32_t tokens,
                   const void* context, int32_t context_bf16, int32_t context_tokens, const uint8_t* context_mask,
                   float* latent, const float* timesteps, const float* deltas, int32_t num_steps,
                   float* velocity_trace, void* workspace, size_t workspace_bytes, void* stream,
                   const fam_decoder_config* dcfg, const fam_decoder_weights* dw, const int32_t* suite_ids,
                   float* actions, int decode_mode, int32_t* decode_fused) {
  int rc = check_cae(cfg);
  if (rc) return rc;
  if (w == nullptr || w->layers == nullptr || latent == nullptr || timesteps == nullptr ||
      deltas == nullptr)
    return set_error("cae: null argument");
  if (batch <= 0 || tokens <= 0 || tokens > kCaeMaxS) return set_error("cae: tokens must be in [1, %d]", kCaeMaxS);
  if (num_steps <= 0 || num_steps > kMaxSteps) return set_error("cae: num_steps must be in [1, %d]", kMaxSteps);
  if (context_tokens <= 0 || context == nullptr) return set_error("cae: a context is required");
  if (w->rope == nullptr || w->rope_positions < tokens) return set_error("cae: RoPE table too short");
  const size_t need = cae_ws(*cfg, batch, context_tokens);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error("cae: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  const int HD = cfg->num_heads * cfg->head_dim;
  const CaeWsLayout wl = cae_ws_layout(*cfg, batch, context_tokens);
  char* ws = static_cast<char*>(workspace);
  float* ctx_k = reinterpret_cast<float*>(ws + wl.k);
  float* ctx_v = reinterpret_cast<float*>(ws + wl.v);
  float* wpack = reinterpret_cast<float*>(ws + wl.wpack);
  int* status = reinterpret_cast<int*>(ws + wl.status);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  CaeCtxArgs ca;
  memset(&ca, 0, sizeof(ca));
  if (context_bf16)
    ca.ctx_bf16 = static_cast<const __nv_bfloat16*>(context);
  else
    ca.ctx_f32 = static_cast<const float*>(context);
  ca.rows = batch * context_tokens;
  ca.T = cfg->text_dim;
  ca.D = cfg->hidden_dim;
  ca.HD = HD;
  ca.L = cfg->num_layers;
  ca.text0_w = w->text0_w;
  ca.text0_b = w->text0_b;
  ca.text2_w = w->text2_w;
  ca.text2_b = w->text2_b;
  for (int l = 0; l < cfg->num_layers; ++l) ca.layers[l] = w->layers[l];
  ca.ctx_k = ctx_k;
  ca.ctx_v = ctx_v;
  ca.eps = cfg->eps;
  ca.B = batch;
  ca.C = context_tokens;
  ca.H = cfg->num_heads;
  ca.hd = cfg->head_dim;
  ca.part = reinterpret_cast<float*>(ws + wl.part);
  ca.status = status;

  CaeStepArgs sa;
  memset(&sa, 0, sizeof(sa));
  sa.w.enc_w = w->enc_w;
  sa.w.enc_b = w->enc_b;
  sa.w.text0_w = w->text0_w;
  sa.w.text0_b = w->text0_b;
  sa.w.text2_w = w->text2_w;
  sa.w.text2_b = w->text2_b;
  sa.w.time0_w = w->time0_w;
  sa.w.time0_b = w->time0_b;
  sa.w.time2_w = w->time2_w;
  sa.w.time2_b = w->time2_b;
  sa.w.tproj_w = w->tproj_w;
  sa.w.tproj_b = w->tproj_b;
  sa.w.head_w = w->head_w;
  sa.w.head_b = w->head_b;
  for (int l = 0; l < cfg->num_layers; ++l) sa.w.layers[l] = w->layers[l];
  sa.rope = w->rope;
  sa.ctx_k = ctx_k;
  sa.ctx_v = ctx_v;
  sa.ctx_mask = context_mask;
  sa.latent = latent;
  sa.trace = velocity_trace;
  for (int i = 0; i < num_steps; ++i) {
    sa.timesteps.t[i] = timesteps[i];
    sa.deltas.t[i] = deltas[i];
  }
  sa.num_steps = num_steps;
  sa.B = batch;
  sa.S = tokens;
  sa.A = cfg->action_dim;
  sa.D = cfg->hidden_dim;
  sa.HD = HD;
  sa.hd = cfg->head_dim;
  sa.F = cfg->ffn_dim;
  sa.C = context_tokens;
  sa.L = cfg->num_layers;
  sa.freq_dim = cfg->freq_dim;
  sa.eps = cfg->eps;
  sa.status = status;
  // staged step kernel when the split context path and the shared-memory plan
  // both fit: the context launch then writes head-major K/V and packs weights
  if (cae_ctx_split_setup(&ca) && cae_staged_plan(sa, &sa.plan)) {
    ca.kv_packed = 1;
    ca.wpack = wpack;
    ca.plan = sa.plan;
    sa.wpack = wpack;
  }
  const bool fuse = dcfg != nullptr && decode_mode != FAM_DECODE_SEPARATE && cae_decode_fusable(sa, *dcfg, *dw) &&
                    (decode_mode == FAM_DECODE_FUSED || cae_decode_auto_fuses(batch));
  if (fuse) {
    const fam_decoder_stage& g = dw->stages[0];
    CaeDecode& d = sa.dec;
    d.enabled = 1;
    d.hidden = dcfg->hidden;
    d.latent = dcfg->latent_dim;
    d.tokens = dcfg->num_tokens;
    d.stride = g.stride;
    d.horizon = dcfg->action_horizon;
    d.action_dim = dcfg->action_dim;
    d.in_w = dw->in_w;
    d.in_b = dw->in_b;
    d.out_w = dw->out_w;
    d.out_b = dw->out_b;
    d.suite_embed = dw->suite_embed;
    d.suite_ids = suite_ids;
    d.convt_w = g.convt_w;
    d.convt_b = g.convt_b;
    d.gn0_w = g.gn0_w;
    d.gn0_b = g.gn0_b;
    d.c1_w = g.c1_w;
    d.c1_b = g.c1_b;
    d.gn1_w = g.gn1_w;
    d.gn1_b = g.gn1_b;
    d.c2_w = g.c2_w;
    d.c2_b = g.c2_b;
    d.gn2_w = g.gn2_w;
    d.gn2_b = g.gn2_b;
    d.lat_std = dw->latent_std;
    d.lat_mean = dw->latent_mean;
    d.out = actions;
  }
  if (decode_fused != nullptr) *decode_fused = fuse ? 1 : 0;
  rc = check_cuda(launch_cae_context(ca, st, false), "cae context launch");
  if (rc) return rc;
  rc = check_cuda(launch_cae_steps(sa, st, true), "cae steps launch");
  if (rc || dcfg == nullptr || fuse) return rc;
  // the separate decoder after the chunk (its scratch behind the expert's workspace)
  const size_t cae_need = cae_ws(*cfg, batch, context_tokens);
  return fam_action_decode(dcfg, dw, batch, latent, suite_ids, actions, static_cast<char*>(workspace) + cae_need,
                           workspace_bytes - cae_need, stream);
}

}  // namespace

extern "C" {

int fam_cae_chunk(const fam_action_config* cfg, const fam_cae_weights* w, int32_t batch,
                  int32_t tokens, const void* context, int32_t context_bf16, int32_t context_tokens,
                  const uint8_t* context_mask, float* latent, const float* timesteps,
                  const float* deltas, int32_t num_steps, float* velocity_trace, void* workspace,
                  size_t workspace_bytes, void* stream) {
  return cae_chunk_impl(cfg, w, batch, tokens, context, context_bf16, context_tokens, context_mask, latent,
                        timesteps, deltas, num_steps, velocity_trace, workspace, workspace_bytes, stream, nullptr,
                        nullptr, nullptr, nullptr, FAM_DECODE_SEPARATE, nullptr);
}

int fam_cae_decode_workspace_size(const fam_action_config* cfg, const fam_decoder_config* dcfg,
                                  const fam_decoder_weights* dw, int32_t batch, int32_t context_tokens,
                                  size_t* bytes) {
  size_t a = 0, d = 0;
  int rc = fam_cae_workspace_size(cfg, batch, context_tokens, &a);
  if (rc) return rc;
  rc = fam_decoder_workspace_size(dcfg, dw, batch, &d);
  if (rc) return rc;
  *bytes = a + d;
  return FAM_OK;
}

int fam_cae_chunk_decode(const fam_action_config* cfg, const fam_cae_weights* w, int32_t batch, int32_t tokens,
                         const void* context, int32_t context_bf16, int32_t context_tokens,
                         const uint8_t* context_mask, float* latent, const float* timesteps, const float* deltas,
                         int32_t num_steps, float* velocity_trace, const fam_decoder_config* dcfg,
                         const fam_decoder_weights* dw, const int32_t* suite_ids, float* actions,
                         int32_t decode_mode, int32_t* decode_fused, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (dcfg == nullptr || dw == nullptr || actions == nullptr) return set_error("cae decode: null decoder argument");
  if (decode_mode < FAM_DECODE_AUTO || decode_mode > FAM_DECODE_SEPARATE)
    return set_error("cae decode: decode_mode must be FAM_DECODE_AUTO, _FUSED or _SEPARATE");
  size_t need = 0;
  int rc = fam_cae_decode_workspace_size(cfg, dcfg, dw, batch, context_tokens, &need);
  if (rc) return rc;
  if (workspace == nullptr || workspace_bytes < need)
    return set_error("cae decode: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if (dcfg->num_tokens != tokens || dcfg->latent_dim != cfg->action_dim)
    return set_error("cae decode: the decoder takes %d x %d latents, the chunk has %d x %d", dcfg->num_tokens,
                     dcfg->latent_dim, tokens, cfg->action_dim);
  return cae_chunk_impl(cfg, w, batch, tokens, context, context_bf16, context_tokens, context_mask, latent,
                        timesteps, deltas, num_steps, velocity_trace, workspace, workspace_bytes, stream, dcfg, dw,
                        suite_ids, actions, decode_mode, decode_fused);
}

int fam_cae_status(const fam_action_config* cfg, int32_t batch, int32_t context_tokens, const void* workspace,
                   int32_t* status, void* stream) {
  int rc = check_cae(cfg);
  if (rc) return rc;
  if (workspace == nullptr || status == nullptr || batch <= 0 || context_tokens <= 0)
    return set_error("cae: bad status arguments");
  const CaeWsLayout wl = cae_ws_layout(*cfg, batch, context_tokens);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = check_cuda(cudaMemcpyAsync(status, static_cast<const char*>(workspace) + wl.status, sizeof(int32_t),
                                  cudaMemcpyDeviceToHost, st),
                  "cae status copy");
  if (rc) return rc;
  return check_cuda(cudaStreamSynchronize(st), "cae status sync");
}

int fam_decoder_workspace_size(const fam_decoder_config* cfg, const fam_decoder_weights* w,
                               int32_t batch, size_t* bytes) {
  if (cfg == nullptr || w == nullptr || bytes == nullptr || batch <= 0) return set_error("decoder: bad argument");
  if (w->num_stages > kDecMaxStages) return set_error("decoder: at most %d stages", kDecMaxStages);
  if ((w->latent_std == nullptr) != (w->latent_mean == nullptr))
    return set_error("decoder: latent_std and latent_mean are given together or not at all");
  *bytes = 3 * align256(decoder_scratch_floats(*cfg, w->stages, w->num_stages, batch) * sizeof(float));
  return FAM_OK;
}

int fam_action_decode(const fam_decoder_config* cfg, const fam_decoder_weights* w, int32_t batch,
                      const float* z, const int32_t* suite_ids, float* out, void* workspace,
                      size_t workspace_bytes, void* stream) {
  size_t need = 0;
  int rc = fam_decoder_workspace_size(cfg, w, batch, &need);
  if (rc) return rc;
  if (z == nullptr || out == nullptr) return set_error("decoder: null z/out");
  if (workspace == nullptr || workspace_bytes < need)
    return set_error("decoder: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  DecArgs a;
  memset(&a, 0, sizeof(a));
  a.cfg = *cfg;
  a.in_w = w->in_w;
  a.in_b = w->in_b;
  a.out_w = w->out_w;
  a.out_b = w->out_b;
  a.suite_embed = w->suite_embed;
  for (int i = 0; i < w->num_stages; ++i) a.stages[i] = w->stages[i];
  a.num_stages = w->num_stages;
  a.z = z;
  a.lat_std = w->latent_std;
  a.lat_mean = w->latent_mean;
  a.suite_ids = suite_ids;
  a.out = out;
  const size_t part = need / 3;
  a.buf0 = static_cast<float*>(workspace);
  a.buf1 = reinterpret_cast<float*>(static_cast<char*>(workspace) + part);
  a.buf2 = reinterpret_cast<float*>(static_cast<char*>(workspace) + 2 * part);
  a.B = batch;
  return check_cuda(launch_action_decoder(a, static_cast<cudaStream_t>(stream)), "decoder launch");
}

}  // extern "C"
