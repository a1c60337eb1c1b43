// Video output head: WanVideoDiT.post_dit = Head.forward + unpatchify
// (FastWAM/src/fastwam/models/wan22/wan_video_dit.py:290-306, 426-431,
// 634-638), the video half of a joint video + action denoising step.
//   video_head_norm_kernel   LayerNorm (no affine) of the fp32 token state,
//                            then * (1 + scale) + shift with the per-token
//                            (shift, scale) = bf16(modulation + t); one warp
//                            per token, the row in registers
//   video_unpatchify_kernel  'b (f h w) (x y z c) -> b c (f x) (h y) (w z)'
// The Linear between them is fam_gemm.
#include "../../include/fam.h"
#include "fam_common.cuh"
#include "fam_internal.h"

namespace fam {
namespace {

constexpr int kHeadMaxPerLane = 4 * 32;  // D <= 4096: 128 values per lane in float4 groups

__global__ void video_head_norm_kernel(const float* __restrict__ hidden, const __nv_bfloat16* __restrict__ t_rows,
                                       const __nv_bfloat16* __restrict__ mod, int B, int S, int ff, int D, float eps,
                                       __nv_bfloat16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= B * S) return;
  const int b = row / S, s = row - b * S;
  const __nv_bfloat16* t = t_rows + (static_cast<long long>(b) * 2 + (s < ff ? 0 : 1)) * D;
  const float* x = hidden + static_cast<long long>(row) * D;
  float v[kHeadMaxPerLane / 4][4];
  float sum = 0.f;
  const int G = D / 4;
#pragma unroll
  for (int i = 0; i < kHeadMaxPerLane / 4; ++i) {
    const int g = lane + 32 * i;
    if (g < G) {
      const float4 q = *reinterpret_cast<const float4*>(x + 4 * g);
      v[i][0] = q.x; v[i][1] = q.y; v[i][2] = q.z; v[i][3] = q.w;
      sum += q.x + q.y + q.z + q.w;
    }
  }
  const float mean = warp_sum(sum) / D;
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < kHeadMaxPerLane / 4; ++i)
    if (lane + 32 * i < G)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float d = v[i][j] - mean;
        var += d * d;
      }
  const float rstd = rsqrtf(warp_sum(var) / D + eps);
#pragma unroll
  for (int i = 0; i < kHeadMaxPerLane / 4; ++i) {
    const int g = lane + 32 * i;
    if (g >= G) continue;
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int f = 4 * g + j;
      const float tv = bf2f(t[f]);
      const float shift = rbf(tv + bf2f(mod[f]));       // bf16(modulation[0] + t)
      const float scale = rbf(tv + bf2f(mod[D + f]));   // bf16(modulation[1] + t)
      const float n = rbf((v[i][j] - mean) * rstd);     // the bf16 LayerNorm output
      o[j] = n * (1.f + scale) + shift;
    }
    __nv_bfloat162 a = __floats2bfloat162_rn(o[0], o[1]), c = __floats2bfloat162_rn(o[2], o[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&c);
    *reinterpret_cast<uint2*>(out + static_cast<long long>(row) * D + 4 * g) = u;
  }
}

__global__ void video_unpatchify_kernel(const __nv_bfloat16* __restrict__ x, int B, int f, int h, int w, int pt,
                                        int ph, int pw, int C, __nv_bfloat16* __restrict__ out) {
  const long long total = static_cast<long long>(B) * f * h * w * pt * ph * pw * C;
  const int F = f * pt, H = h * ph, W = w * pw;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    // output index (b, c, F, H, W) in row-major order
    long long r = i;
    const int X = static_cast<int>(r % W); r /= W;
    const int Y = static_cast<int>(r % H); r /= H;
    const int T = static_cast<int>(r % F); r /= F;
    const int c = static_cast<int>(r % C);
    const int b = static_cast<int>(r / C);
    const int fi = T / pt, xi = T % pt, hi = Y / ph, yi = Y % ph, wi = X / pw, zi = X % pw;
    const long long tok = (static_cast<long long>(b) * f + fi) * h * w + static_cast<long long>(hi) * w + wi;
    const int col = ((xi * ph + yi) * pw + zi) * C + c;
    out[i] = x[tok * (static_cast<long long>(pt) * ph * pw * C) + col];
  }
}

}  // namespace
}  // namespace fam

using namespace fam;

extern "C" {

int fam_video_head_norm(const float* hidden, const void* t_rows, const void* modulation, int32_t batch,
                        int32_t tokens, int32_t first_frame_tokens, int32_t dim, float eps, void* out, void* stream) {
  if (hidden == nullptr || t_rows == nullptr || modulation == nullptr || out == nullptr || batch <= 0 ||
      tokens <= 0 || dim <= 0 || (dim % 4) || dim > kHeadMaxPerLane * 32)
    return set_error("fam_video_head_norm: bad arguments (dim a multiple of 4, at most %d)", kHeadMaxPerLane * 32);
  const int rows = batch * tokens, per_block = 8;
  video_head_norm_kernel<<<(rows + per_block - 1) / per_block, 32 * per_block, 0, static_cast<cudaStream_t>(stream)>>>(
      hidden, static_cast<const __nv_bfloat16*>(t_rows), static_cast<const __nv_bfloat16*>(modulation), batch, tokens,
      first_frame_tokens, dim, eps, static_cast<__nv_bfloat16*>(out));
  return check_cuda(cudaGetLastError(), "video_head_norm_kernel");
}

int fam_video_unpatchify(const void* x, int32_t batch, int32_t f, int32_t h, int32_t w, int32_t pt, int32_t ph,
                         int32_t pw, int32_t channels, void* out, void* stream) {
  if (x == nullptr || out == nullptr || batch <= 0 || f <= 0 || h <= 0 || w <= 0 || pt <= 0 || ph <= 0 || pw <= 0 ||
      channels <= 0)
    return set_error("fam_video_unpatchify: bad arguments");
  const long long total = static_cast<long long>(batch) * f * h * w * pt * ph * pw * channels;
  long long blocks = (total + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  video_unpatchify_kernel<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), batch, f, h, w, pt, ph, pw, channels, static_cast<__nv_bfloat16*>(out));
  return check_cuda(cudaGetLastError(), "video_unpatchify_kernel");
}

}  // extern "C"
