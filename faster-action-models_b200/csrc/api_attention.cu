// Op-level attention entry points of the C ABI (fam_attention and its
// workspace query).  The model runtimes call launch_attention directly.
#include <cmath>

#include "../../include/fam.h"
#include "fam_internal.h"
#include "fam_kernels.h"
#include "attention_plan.h"

namespace fam {

int attention_prepare(const fam_attention_desc* d, AttnArgs* a, AttnScratch* s) {
  if (d == nullptr) return set_error("attention: null descriptor");
  if (d->head_dim != 64 && d->head_dim != 128)
    return set_error("attention: head_dim %d unsupported (64 or 128)", d->head_dim);
  if (d->batch <= 0 || d->heads <= 0 || d->q_tokens <= 0)
    return set_error("attention: batch, heads and q_tokens must be > 0");
  if (d->kv1_tokens < 0 || d->kv2_tokens < 0 || d->kv1_tokens + d->kv2_tokens <= 0)
    return set_error("attention: no keys");
  if (d->q == nullptr || d->out == nullptr || (d->kv1_tokens > 0 && (!d->k1 || !d->v1)) ||
      (d->kv2_tokens > 0 && (!d->k2 || !d->v2)))
    return set_error("attention: null tensor");
  if ((d->q_token_stride | d->kv1_token_stride | d->kv2_token_stride | d->out_token_stride) & 7)
    return set_error("attention: token strides must be multiples of 8 elements");
  const int skv = d->kv1_tokens + d->kv2_tokens;
  const int q_tiles = attn_query_tiles(d->q_tokens);
  const int units = d->batch * d->heads * q_tiles;
  int splits = d->kv_splits;
  int kps = 0;
  if (splits <= 0) {
    splits = attn_auto_splits(units, skv, &kps);
  } else {
    if (splits > 64) splits = 64;
    kps = (skv + splits - 1) / splits;
    kps = (kps + 63) / 64 * 64;
    splits = (skv + kps - 1) / kps;
  }
  *a = AttnArgs{};
  a->q = static_cast<const __nv_bfloat16*>(d->q);
  a->q_bs = d->q_batch_stride;
  a->q_ts = d->q_token_stride;
  a->k1 = static_cast<const __nv_bfloat16*>(d->k1);
  a->v1 = static_cast<const __nv_bfloat16*>(d->v1);
  a->kv1_bs = d->kv1_batch_stride;
  a->kv1_ts = d->kv1_token_stride;
  a->S1 = d->kv1_tokens;
  a->k2 = static_cast<const __nv_bfloat16*>(d->k2);
  a->v2 = static_cast<const __nv_bfloat16*>(d->v2);
  a->kv2_bs = d->kv2_batch_stride;
  a->kv2_ts = d->kv2_token_stride;
  a->S2 = d->kv2_tokens;
  a->mask2d = d->mask;
  a->mask_rs = d->mask_row_stride;
  a->key_mask = d->key_mask;
  a->key_mask_bs = d->key_mask_batch_stride;
  a->first_frame_tokens = d->first_frame_tokens;
  a->Sq = d->q_tokens;
  a->H = d->heads;
  a->scale_log2 = 1.4426950408889634f / std::sqrt(static_cast<float>(d->head_dim));
  a->out = static_cast<__nv_bfloat16*>(d->out);
  a->out_bs = d->out_batch_stride;
  a->out_ts = d->out_token_stride;
  a->nsplit = splits;
  a->keys_per_split = kps;
  s->partial_bytes = attn_partial_bytes(d->batch, d->heads, d->q_tokens, d->head_dim, splits);
  s->counter_bytes = splits > 1 ? static_cast<size_t>(units) * sizeof(int) : 0;
  s->counter_offset = (s->partial_bytes + 255) / 256 * 256;
  s->total = s->counter_offset + s->counter_bytes;
  return 0;
}

// Points the launch at `scratch` (partials, then the arrival counters) and
// clears the counters on the stream.
cudaError_t attention_bind_scratch(AttnArgs* a, const AttnScratch& s, void* scratch,
                                   cudaStream_t st) {
  if (a->nsplit <= 1) return cudaSuccess;
  a->part = static_cast<float*>(scratch);
  a->counters = reinterpret_cast<int*>(static_cast<char*>(scratch) + s.counter_offset);
  return cudaMemsetAsync(a->counters, 0, s.counter_bytes, st);
}

}  // namespace fam

using namespace fam;

extern "C" {

// Long self attention (one key source of the query length, head_dim 128, no
// explicit or key mask, no forced split) runs the tcgen05 kernel, which needs
// room for V^T after the split scratch.
static bool attention_use_tc(const fam_attention_desc* d, const AttnArgs& a) {
  return d->kv_splits <= 1 && d->kv1_batch_stride == static_cast<long long>(d->kv1_tokens) * d->kv1_token_stride &&
         d->q_batch_stride == static_cast<long long>(d->q_tokens) * d->q_token_stride &&
         d->out_batch_stride == static_cast<long long>(d->q_tokens) * d->out_token_stride &&
         attention_tc_eligible(d->head_dim, d->batch, a.H, a.Sq, a.S1, a.S2, a.mask2d != nullptr, a.first_frame_tokens,
                               a.q_ts, a.kv1_ts, a.out_ts);
}

int fam_attention_workspace_size(const fam_attention_desc* d, size_t* bytes) {
  if (bytes == nullptr) return set_error("attention: null bytes");
  AttnArgs a;
  AttnScratch s;
  const int rc = attention_prepare(d, &a, &s);
  if (rc) return rc;
  *bytes = s.total;
  if (d->kv_splits <= 0 && attention_short_tc_taken(a, d->batch, d->head_dim)) *bytes = 0;  // one CTA per (batch, head)
  else if (attention_use_tc(d, a)) *bytes = (s.total + 255) / 256 * 256 + attention_tc_vt_bytes(d->batch, d->heads, a.S1);
  return FAM_OK;
}

int fam_attention(const fam_attention_desc* d, void* workspace, size_t workspace_bytes,
                  void* stream) {
  AttnArgs a;
  AttnScratch s;
  int rc = attention_prepare(d, &a, &s);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (d->kv_splits <= 0 && attention_short_tc_taken(a, d->batch, d->head_dim)) {
    // short query sets on tcgen05: one CTA per (batch, head), no split scratch
    a.status = device_status_word();
    return check_cuda(launch_attention_auto(a, d->batch, d->head_dim, st, false), "attention launch");
  }
  if (a.nsplit > 1 && (workspace == nullptr || workspace_bytes < s.total))
    return set_error("attention: workspace of %zu bytes needed, %zu given", s.total, workspace_bytes);
  if (attention_use_tc(d, a)) {
    const size_t off = (s.total + 255) / 256 * 256;
    const size_t need = off + attention_tc_vt_bytes(d->batch, d->heads, a.S1);
    if (workspace == nullptr || workspace_bytes < need)
      return set_error("attention: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    return check_cuda(launch_attention_tc(a.q, a.q_ts, a.k1, a.v1, a.kv1_ts, a.out, a.out_ts, d->batch, a.Sq, a.S1,
                                          a.H, a.first_frame_tokens, a.key_mask, a.key_mask_bs, a.scale_log2,
                                          reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(workspace) + off), nullptr,
                                          st, false),
                      "attention launch");
  }
  rc = check_cuda(attention_bind_scratch(&a, s, workspace, st), "attention counters");
  if (rc) return rc;
  return check_cuda(launch_attention(a, d->batch, d->head_dim, st, false), "attention launch");
}

}  // extern "C"
