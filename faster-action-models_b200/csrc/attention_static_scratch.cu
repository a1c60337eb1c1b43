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
//   * Set-up: the first call on each device (with that device current)
//     looks up the array's device address with cudaGetSymbolAddress.  Make
//     that first call before any stream capture on the device.
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

// Device address of g_attention_scratch on the current device (set up once
// per device).  The host-side symbol itself is only a stand-in and must never
// be passed to a kernel.
static int static_scratch(void** out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "attention_static_scratch: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDev) return set_error("attention_static_scratch: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_attention_scratch),
                    "attention_static_scratch: cudaGetSymbolAddress");
    if (rc) return rc;
    g_scratch_addr[dev] = p;
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
  if (s.total > kStaticScratchBytes)
    return set_error(
        "attention_static_scratch: this call needs %zu bytes of scratch, the static array holds "
        "%zu; use fam_attention with a workspace or fewer kv_splits",
        s.total, kStaticScratchBytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a.nsplit > 1) {
    void* scratch = nullptr;
    rc = static_scratch(&scratch);
    if (rc) return rc;
    rc = check_cuda(attention_bind_scratch(&a, s, scratch, st), "attention_static_scratch counters");
    if (rc) return rc;
  }
  return check_cuda(launch_attention(a, d->batch, d->head_dim, st, false),
                    "attention_static_scratch launch");
}
