// Core of the C ABI: error reporting, the device status word, tensor-map
// encoding, and the op-level GEMM entry point.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "../../include/fam.h"
#include "fam_common.cuh"
#include "fam_internal.h"

namespace fam {

static thread_local char g_last_error[1024] = "";

int set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return FAM_ERR_INVALID;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FAM_OK;
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", what, cudaGetErrorName(e),
           cudaGetErrorString(e));
  return FAM_ERR_CUDA;
}

static constexpr int kMaxDevices = 64;
static int* g_status_words[kMaxDevices] = {nullptr};
static std::mutex g_status_mu;

int* device_status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (g_status_words[dev] == nullptr) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
    g_status_words[dev] = p;
  }
  return g_status_words[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  std::call_once(g_encode_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                       uint64_t row_stride, uint32_t box_rows) {
  if (tmap_encoder() == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
  cuuint32_t box[2] = {64u, box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D bf16 tensor map over [batch, rows, cols] with row stride `row_stride` and
// batch stride `batch_stride` elements; box = 64 columns x box_rows rows x 1,
// 128-byte swizzle, out-of-bounds elements (past a batch's rows) read as zero.
bool make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t batch, uint64_t rows, uint64_t cols,
                       uint64_t row_stride, uint64_t batch_stride, uint32_t box_rows) {
  if (tmap_encoder() == nullptr) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride * 2), static_cast<cuuint64_t>(batch_stride * 2)};
  cuuint32_t box[3] = {64u, box_rows, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D uint8 tensor map over a row-major [rows, cols] byte matrix (row stride in
// bytes), box = box_cols x box_rows, no swizzle, out-of-bounds bytes read as
// zero.
bool make_tmap_u8_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride,
                     uint32_t box_cols, uint32_t box_rows) {
  if (tmap_encoder() == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace fam

using namespace fam;

extern "C" {

int fam_version(int* major, int* minor, int* patch) {
  if (major) *major = FAM_VERSION_MAJOR;
  if (minor) *minor = FAM_VERSION_MINOR;
  if (patch) *patch = FAM_VERSION_PATCH;
  return FAM_OK;
}

int fam_last_error(char* buf, size_t len) {
  if (buf == nullptr || len == 0) return FAM_ERR_INVALID;
  strncpy(buf, g_last_error, len - 1);
  buf[len - 1] = '\0';
  return FAM_OK;
}

int fam_device_status(int* code, int reset, void* stream) {
  int* w = device_status_word();
  if (w == nullptr) return set_error("fam_device_status: no device status word");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  int rc = check_cuda(cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, st),
                      "fam_device_status copy");
  if (rc) return rc;
  rc = check_cuda(cudaStreamSynchronize(st), "fam_device_status sync");
  if (rc) return rc;
  if (reset && v != 0) {
    rc = check_cuda(cudaMemsetAsync(w, 0, sizeof(int), st), "fam_device_status reset");
    if (rc) return rc;
  }
  if (code) *code = v;
  return FAM_OK;
}

namespace fam {
// One thread waits on an mbarrier that nothing will complete: the bounded wait
// gives up after its %globaltimer limit, records kErrWaitFull in the status
// word and the kernel returns normally.
__global__ void selftest_wait_kernel(int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_wait(&bar, 0, status, kErrWaitFull);
  }
}
}  // namespace fam

int fam_selftest_bounded_wait(void* stream) {
  int* w = device_status_word();
  if (w == nullptr) return set_error("fam_selftest_bounded_wait: no device status word");
  fam::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(w);
  return check_cuda(cudaGetLastError(), "fam_selftest_bounded_wait launch");
}

int fam_gemm(const fam_gemm_desc* d, void* stream) {
  if (d == nullptr) return set_error("fam_gemm: null descriptor");
  GemmEpilogue e = {};
  e.kind = d->epilogue;
  e.act = d->activation;
  e.out_bf16 = d->out_dtype == FAM_DTYPE_BF16 ? 1 : 0;
  e.features_on_a = d->features_on_a;
  e.out = d->out;
  e.out_sa = d->out_stride_a;
  e.out_sb = d->out_stride_b;
  e.split_stride = d->out_stride_split;
  e.bias = static_cast<const __nv_bfloat16*>(d->bias);
  e.gate_w = static_cast<const __nv_bfloat16*>(d->gate_w);
  e.gate_t = static_cast<const float*>(d->gate_t);
  e.tokens_per_batch = d->tokens_per_batch;
  e.first_frame_tokens = d->first_frame_tokens;
  e.gate_bstride = d->gate_batch_stride;
  e.gate_gstride = d->gate_group_stride;
  if (e.kind < FAM_EPI_STORE || e.kind > FAM_EPI_RESIDUAL)
    return set_error("fam_gemm: unknown epilogue %d", e.kind);
  if (e.kind == FAM_EPI_RESIDUAL && d->out_dtype != FAM_DTYPE_F32)
    return set_error("fam_gemm: the residual epilogue accumulates into fp32");
  if (e.out == nullptr) return set_error("fam_gemm: null output");
  GemmPlan p;
  float* skp = nullptr;
  unsigned* skf = nullptr;
  size_t skb = 0;
  if (d->scratch != nullptr) {
    const size_t part = gemm_sk_scratch_bytes();
    if (d->scratch_bytes < part + gemm_num_sms() * sizeof(unsigned))
      return set_error("fam_gemm: split-round scratch of %zu bytes needed", part + gemm_num_sms() * sizeof(unsigned));
    skp = static_cast<float*>(d->scratch);
    skf = reinterpret_cast<unsigned*>(static_cast<char*>(d->scratch) + part);
    skb = part;
  }
  int rc;
  if (d->conv_wp > 0) {
    if (d->features_on_a || d->conv_cin <= 0 || d->k != 9 * ((d->conv_cin + 63) / 64) * 64 || d->tile_n != 0)
      return set_error("fam_gemm: convolution needs features_on_a = 0, tile_n = 0 and k = 9 * ceil(cin / 64) * 64");
    rc = gemm_plan_conv3(&p, d->a, d->lda, d->conv_a_rows, d->conv_cin, d->conv_wp, d->m, d->b, d->ldb, d->n,
                         d->splits, e, device_status_word());
  } else {
    rc = gemm_plan(&p, d->a, d->lda, d->b, d->ldb, d->m, d->n, d->k, d->splits, d->tile_n, e,
                   d->a_is_const != 0, d->b_is_const != 0, device_status_word(), skp, skf, skb,
                   d->split_round != 0, d->pair != 0);
  }
  if (rc) return rc;
  return check_cuda(gemm_launch(p, static_cast<cudaStream_t>(stream), d->pdl != 0), "fam_gemm launch");
}

int fam_gemm_split_round_scratch_bytes(size_t* bytes) {
  if (bytes == nullptr) return set_error("fam_gemm_split_round_scratch_bytes: null bytes");
  *bytes = gemm_sk_scratch_bytes() + gemm_num_sms() * sizeof(unsigned);
  return FAM_OK;
}

}  // extern "C"
