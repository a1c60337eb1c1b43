// Patch extraction for the video DiT's patch_embedding Conv3d (kernel = stride
// = patch, FastWAM/src/fastwam/models/wan22/wan_video_dit.py:366-367): with
// non-overlapping patches the convolution is a GEMM over rows
//   row = b * S + (f * Hp + hp) * Wp + wp,  S = Fp * Hp * Wp,
//   col = ((c * pt + kt) * ph + kh) * pw + kw  (the Conv3d weight's flattening),
// so this kernel writes the bf16 row matrix the tcgen05 GEMM consumes.
#include "fam_common.cuh"
#include "fam_kernels.h"

namespace fam {

__global__ void patchify_kernel(const PatchArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int Fp = a.F / a.pt, Hp = a.H / a.ph, Wp = a.W / a.pw;
  const long long S = static_cast<long long>(Fp) * Hp * Wp;
  const int K = a.Cin * a.pt * a.ph * a.pw;
  const long long total = a.B * S * K;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = idx / K;
    const int col = static_cast<int>(idx % K);
    const int b = static_cast<int>(row / S);
    const long long tok = row % S;
    const int f = static_cast<int>(tok / (Hp * Wp));
    const int hp = static_cast<int>((tok / Wp) % Hp);
    const int wp = static_cast<int>(tok % Wp);
    const int kw = col % a.pw;
    const int kh = (col / a.pw) % a.ph;
    const int kt = (col / (a.pw * a.ph)) % a.pt;
    const int c = col / (a.pw * a.ph * a.pt);
    const long long src =
        ((((static_cast<long long>(b) * a.Cin + c) * a.F + (f * a.pt + kt)) * a.H + (hp * a.ph + kh)) *
             a.W +
         (wp * a.pw + kw));
    a.out[idx] = a.in[src];
  }
}

cudaError_t launch_patchify(const PatchArgs& a, cudaStream_t st) {
  const long long S = static_cast<long long>(a.F / a.pt) * (a.H / a.ph) * (a.W / a.pw);
  const long long total = a.B * S * a.Cin * a.pt * a.ph * a.pw;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  patchify_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace fam
