/*
 * libfam — B200 (sm_100a) kernels for the per-action-chunk denoising path of
 * the FastWAM world action models.  Plain C ABI: device pointers, sizes and a
 * cudaStream_t passed as void*; no torch types; every entry point returns an
 * int status (FAM_OK == 0) and fam_last_error() describes the last failure of
 * the calling thread.  No entry point allocates device memory during a call
 * except the one-time status word per device and the packed-weight handles
 * documented below; outputs and workspaces are caller-owned.
 *
 * Reference interfaces replaced (paths relative to the reference project):
 *   fam_gemm                  nn.Linear calls of DiTBlock / ActionDiT / WanVideoDiT
 *                             (FastWAM/src/fastwam/models/wan22/wan_video_dit.py:170-246,
 *                              action_dit.py:73-97)
 * The model-level entry points are declared further down with their own
 * citations.
 */
#ifndef FAM_H_
#define FAM_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FAM_API __attribute__((visibility("default")))
#else
#define FAM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FAM_VERSION_MAJOR 0
#define FAM_VERSION_MINOR 1
#define FAM_VERSION_PATCH 0

/* status codes */
#define FAM_OK 0
#define FAM_ERR_INVALID 1  /* bad argument or unsupported shape */
#define FAM_ERR_CUDA 2     /* a CUDA runtime call failed */
#define FAM_ERR_DEVICE 3   /* a kernel reported an error through the status word */

/* dtypes */
#define FAM_DTYPE_BF16 0
#define FAM_DTYPE_F32 1

/* GEMM epilogues */
#define FAM_EPI_STORE 0    /* out = act(acc + bias) */
#define FAM_EPI_PARTIAL 1  /* out[split] = acc (fp32 split-K partials, no bias) */
#define FAM_EPI_RESIDUAL 2 /* out_f32 += gate * (acc + bias) */

#define FAM_ACT_NONE 0
#define FAM_ACT_GELU_TANH 1

FAM_API int fam_version(int* major, int* minor, int* patch);

/* Copies the calling thread's last error message (NUL-terminated). */
FAM_API int fam_last_error(char* buf, size_t len);

/* Reads the current device's status word (0 = healthy; otherwise the code of
 * the first kernel that gave up a bounded wait or rejected its arguments).
 * Synchronizes `stream`.  reset != 0 clears the word afterwards. */
FAM_API int fam_device_status(int* code, int reset, void* stream);

/* D[m][n] = sum_k A[m][k] * B[n][k]  on the tcgen05 tensor cores.
 * A: bf16 [m, k] row stride lda; B: bf16 [n, k] row stride ldb (both K-major,
 * 16-byte aligned, k and strides multiples of 8).  The output element for
 * (m, n) is out[m * out_stride_a + n * out_stride_b] (+ split * out_stride_split
 * for FAM_EPI_PARTIAL).  features_on_a says which index is the output feature
 * (selects bias[feature] and the residual gate); the other index is the token.
 * Residual gate for token t, feature f:
 *   gate_w[f] + gate_t[(t / tokens_per_batch) * gate_batch_stride
 *                      + (first_frame_tokens > 0 && t % tokens_per_batch >= first_frame_tokens
 *                         ? gate_group_stride : 0) + f]
 * (gate_t == NULL: gate 1).  tile_n = 0 picks the MMA N tile (16..256). */
typedef struct fam_gemm_desc {
  const void* a;
  int64_t lda;
  const void* b;
  int64_t ldb;
  int32_t m, n, k;
  int32_t splits;
  int32_t tile_n;
  int32_t epilogue;
  int32_t activation;
  int32_t out_dtype;
  int32_t features_on_a;
  int32_t a_is_const; /* operand is constant across a launch chain (prefetched before the PDL wait) */
  int32_t b_is_const;
  int32_t pdl;        /* launch with programmatic stream serialization */
  void* out;
  int64_t out_stride_a;
  int64_t out_stride_b;
  int64_t out_stride_split;
  const void* bias;   /* bf16 [features] or NULL */
  const void* gate_w; /* bf16 [features] or NULL */
  const void* gate_t; /* f32 or NULL */
  int32_t tokens_per_batch;
  int32_t first_frame_tokens;
  int64_t gate_batch_stride;
  int64_t gate_group_stride;
} fam_gemm_desc;

FAM_API int fam_gemm(const fam_gemm_desc* desc, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FAM_H_ */
