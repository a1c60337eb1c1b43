// fam_attention_static_scratch: fam_attention for callers that cannot
// allocate device memory.
//
// Some hosts of this library never call cudaMalloc themselves and cannot
// hand it a workspace: a plugin running inside a process whose allocator
// they do not own, a real-time control loop that forbids allocation after
// start-up, or an FFI caller with no device allocator at all.  This entry
// point serves them: it runs the same split-KV attention kernel, but its
// scratch (the per-split partial results and the arrival counters) lives in
// one file-scope device array that the library image carries.
//
// Contract, stated for the caller:
//   * Maximum scratch: kStaticScratchBytes (8 MiB) per GPU.  Every GPU that
//     loads the library holds this array until the process exits.  A call
//     whose split partials would exceed it is rejected with FAM_ERR_INVALID
//     and a message naming the bytes it would need (use fam_attention with a
//     workspace instead, or pass kv_splits = 1, which needs no scratch).
//   * Nothing is allocated: no cudaMalloc, cudaFree or allocating library
//     routine is called.  The arrival counters are cleared with
//     cudaMemsetAsync on the caller's stream at every call.
//   * Set-up: every call made while its stream is not capturing looks up the
//     array's device address (cudaGetSymbolAddress, with the call's device
//     current), so a context that was reset and reloaded is picked up; a
//     call inside a stream capture reuses the address of the last such call
//     on that device, so make one call on each device before any capture.
//     Under CUDA's lazy module loading (the default) that first call also
//     loads the library's device image, this array included: make it at
//     start-up, before the part of the program that must not allocate.
//   * Kernel: the tcgen05 short-query kernel when the descriptor qualifies
//     (kv_splits = 0, head_dim 64, <= 32 queries, batch x heads >= 128: one CTA
//     per (batch, head), no scratch), else the split-KV mma.sync attention of
//     fam_attention.  The tcgen05 long-self-attention kernel that fam_attention
//     picks for one key source of head_dim 128 needs a transposed-V workspace,
//     so it is not used here.
//   * Every call on a device shares the one array and leaves its contents
//     behind.  Calls that may overlap on the GPU (different streams, or
//     concurrent graphs) race on it: serialize them.
#include <mutex>

#include "../../include/fam.h"
#include "attention_plan.h"
#include "fam_internal.h"
#include "fam_kernels.h"

namespace fam {

constexpr size_t kStaticScratchBytes = 8u << 20;

static __device__ __align__(256) unsigned char g_attention_scratch[kStaticScratchBytes];

static constexpr int kMaxDev = 64;
static void* g_scratch_addr[kMaxDev] = {nullptr};
static std::mutex g_scratch_mu;

// Device address of g_attention_scratch on the current device.  The host-side
// symbol itself is only a stand-in and must never be passed to a kernel.  It is
// looked up again on every call outside a stream capture (cheap), so that a
// context reset that reloaded the module is followed; inside a capture the
// last looked-up address of the device is used.
static int static_scratch(cudaStream_t st, void** out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "attention_static_scratch: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDev) return set_error("attention_static_scratch: device %d out of range", dev);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  rc = check_cuda(cudaStreamIsCapturing(st, &cap), "attention_static_scratch: cudaStreamIsCapturing");
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (cap == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_attention_scratch),
                    "attention_static_scratch: cudaGetSymbolAddress");
    if (rc) return rc;
    g_scratch_addr[dev] = p;
  } else if (g_scratch_addr[dev] == nullptr) {
    return set_error("attention_static_scratch: the first call on device %d must come before any stream "
                     "capture (it looks up the static scratch)", dev);
  }
  *out = g_scratch_addr[dev];
  return 0;
}

}  // namespace fam

using namespace fam;

extern "C" int fam_attention_static_scratch(const fam_attention_desc* d, void* stream) {
  AttnArgs a;
  AttnScratch s;
  int rc = attention_prepare(d, &a, &s);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (d->kv_splits <= 0 && attention_short_tc_taken(a, d->batch, d->head_dim))
    return check_cuda(launch_attention_auto(a, d->batch, d->head_dim, st, false), "attention_static_scratch launch");
  if (s.total > kStaticScratchBytes)
    return set_error(
        "attention_static_scratch: this call needs %zu bytes of scratch, the static array holds "
        "%zu; use fam_attention with a workspace or fewer kv_splits",
        s.total, kStaticScratchBytes);
  if (a.nsplit > 1) {
    void* scratch = nullptr;
    rc = static_scratch(st, &scratch);
    if (rc) return rc;
    rc = check_cuda(attention_bind_scratch(&a, s, scratch, st), "attention_static_scratch counters");
    if (rc) return rc;
  }
  return check_cuda(launch_attention(a, d->batch, d->head_dim, st, false),
                    "attention_static_scratch launch");
}
