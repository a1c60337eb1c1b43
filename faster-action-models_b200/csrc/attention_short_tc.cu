// tcgen05 attention for a short query set over long key sources: the action
// expert's joint attention (the action tokens of one (batch, head) over that
// sample's video K/V cache followed by the action tokens' own keys,
// FastWAM/src/fastwam/models/wan22/mot.py:88-103 with flash_attention of
// wan_video_dit.py:13-22), head dim 64, at most 32 queries.
//
// One CTA = one (batch, head) over all keys.  The queries are loaded four
// times into the 128-row Q tile, so TMEM lane quarter w (lanes 32 w .. 32 w +
// 31) holds every query's score row after S = Q K^T of a 128-key block.
// Softmax warp w owns keys [32 w, 32 w + 32) of every block for all queries:
// it keeps its own running maximum and sum and writes its probabilities into
// P columns [16 w, 16 w + 16) of its own lanes, whose other P columns stay
// zero, so the O rows of quarter w accumulate P.V over quarter w's keys only.
// Four online softmaxes over disjoint key subsets run side by side and are
// merged once at the end through shared memory.  Warp roles (256 threads):
//   warp 0      TMA producer: the Q copies, then 128-key blocks of K and V from
//               source 1 (the cache) and source 2 (fresh keys) into a 5-stage
//               ring; 3-D tensor maps whose boxes are min(128, keys) rows, so
//               a block that runs past a source's keys reads zeros there (a
//               source shorter than 128 keys leaves the rest of the stage as
//               it was: zeroed at the start, or an earlier block's finite keys,
//               all masked); with an attend mask whose rows and offsets
//               suit TMA, the block's [queries, 128 keys] attend bytes land in
//               the same stage;
//   warp 1      TMEM (S double buffer at columns [0, 256), P double buffer
//               [256, 384), O [384, 448)) and MMA issue: S two blocks ahead of
//               the softmax, P(j).V(j) with A = P in TMEM and B = the V tile as
//               TMA wrote it ([keys, dims] rows: an MN-major operand, no
//               transpose);
//   warps 4..7  softmax quarters, then the merge and the bf16 output rows.
//               With P double-buffered a warp waits for P.V only to rescale O
//               (the running maximum moved by more than kShLazy) and for the
//               P.V two blocks back; the attend bytes of the next block are
//               loaded while this one is processed.
// Every wait is bounded (status word, then the CTA drains its copies and
// frees TMEM).
#include "fam_common.cuh"
#include "fam_internal.h"
#include "fam_kernels.h"

namespace fam {

namespace {

constexpr int kShRows = 128;                 // Q tile rows (4 copies of <= 32 queries), keys per block
constexpr int kShQ = 32;                     // queries per (batch, head)
constexpr int kShHd = 64;                    // head dim: one 128-byte swizzle row
constexpr int kShTile = kShRows * 128;       // one [128 rows, 64 bf16] tile
constexpr int kShMaskTile = kShQ * kShRows;     // attend bytes of one block [32][128]
constexpr int kShMergeRow = 68;              // floats per merged O row (pad: conflict-free float4 stores)
constexpr int kShMergeBytes = 4 * kShQ * kShMergeRow * 4 + 4 * kShQ * 2 * 4;

// Two shapes of the kernel.  The full one (one CTA per SM: S and P
// double-buffered, 512 TMEM columns, a 5-stage ring) serves launches of up to
// two waves; the compact one (two CTAs per SM: one S and one P buffer, 256
// TMEM columns, a 2-stage ring) serves larger launches, where the second
// CTA's softmax fills the gaps in the first one's chain.
template <bool kCompact>
struct ShCfg {
  static constexpr int kStages = kCompact ? 2 : 5;
  static constexpr int kSB = kCompact ? 1 : 2;  // S buffers
  static constexpr int kPB = kCompact ? 1 : 2;  // P buffers
  static constexpr uint32_t kColS = 0;
  static constexpr uint32_t kColP = 128 * kSB;
  static constexpr uint32_t kColO = kColP + 64 * kPB;
  static constexpr uint32_t kTmemCols = kCompact ? 256 : 512;
  static constexpr int kBarOff = (1 + 2 * kStages) * kShTile + kStages * kShMaskTile;
  static constexpr int kSmem = kBarOff + 256 + 1024;  // + barriers, + alignment slack
  static_assert(kShMergeBytes <= 2 * kStages * kShTile, "the merge overlays the K and V rings");
  static_assert(kColO + 64 <= kTmemCols, "TMEM columns");
};
constexpr float kShLazy = 8.f;
constexpr int kErrShortWait = 0x4155;

struct AttnShortArgs {
  CUtensorMap tq;    // Q   [B, Sq, H*64], box 64 x Sq
  CUtensorMap tk1;   // K1  [B, S1, H*64], box 64 x min(128, S1)
  CUtensorMap tv1;
  CUtensorMap tk2;   // K2  [B, S2, H*64], box 64 x min(128, S2)
  CUtensorMap tv2;
  CUtensorMap tm;    // attend bytes [Sq, S1+S2], box 128 x Sq (mask_tma)
  const uint8_t* mask2d;
  long long mask_rs;
  const uint8_t* key_mask;
  long long key_mask_bs;
  __nv_bfloat16* out;
  long long out_bs, out_ts;
  int Sq, S1, S2;
  int box1, box2;    // rows per K / V box of each source
  int mask_tma;      // attend tiles arrive with the K / V stages
  int kv1_const;
  float scale_log2;
  int* status;
};

// Bit i: byte i of the 32 attend bytes in (u0, u1) is nonzero.  All-ones bytes
// (a bool mask that hides nothing here) take one AND chain.
__device__ __forceinline__ uint32_t word_bits(const uint4& u0, const uint4& u1) {
  const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
  if ((w[0] & w[1] & w[2] & w[3] & w[4] & w[5] & w[6] & w[7] & 0x01010101u) == 0x01010101u) return 0xffffffffu;
  uint32_t bits = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) bits |= (((w[i] >> (8 * k)) & 0xffu) != 0u ? 1u : 0u) << (4 * i + k);
  return bits;
}

// Bits i < nv of the attend bytes starting at p (nonzero = attend), byte loads.
__device__ __forceinline__ uint32_t attend_bits(const uint8_t* p, int nv) {
  uint32_t bits = 0;
  for (int i = 0; i < nv && i < 32; ++i) bits |= (p[i] != 0 ? 1u : 0u) << i;
  return bits;
}

template <bool kCompact>
__global__ void __launch_bounds__(256, kCompact ? 2 : 1) attention_short_tc_kernel(const __grid_constant__ AttnShortArgs a) {
  using Cfg = ShCfg<kCompact>;
  constexpr int kSB = Cfg::kSB, kPB = Cfg::kPB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = sm;
  uint8_t* sK = sm + kShTile;                      // stage s at + s kShTile
  uint8_t* sV = sm + (1 + Cfg::kStages) * kShTile;
  uint8_t* sMk = sm + (1 + 2 * Cfg::kStages) * kShTile;  // stage s at + s kShMaskTile
  // the quarter merge overlays the K and V rings: no copy is in flight and no
  // MMA reads them once the last P.V is complete
  float* so = reinterpret_cast<float*>(sK);                                    // [4][32][kShMergeRow]
  float* sml = so + 4 * kShQ * kShMergeRow;                                     // [4][32] (m, l)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Cfg::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                    // [Cfg::kStages]
  uint64_t* kv_empty = bars + 1 + Cfg::kStages;       // [Cfg::kStages]
  uint64_t* s_full = bars + 1 + 2 * Cfg::kStages;     // [kSB] S buffer
  uint64_t* p_full = bars + 3 + 2 * Cfg::kStages;     // [kPB] P buffer, 4 softmax warps each
  uint64_t* pv_done = bars + 5 + 2 * Cfg::kStages;    // [kPB] P buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7 + 2 * Cfg::kStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* fail_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, b = blockIdx.y;
  const int nb1 = (a.S1 + kShRows - 1) / kShRows;
  const int nb = nb1 + (a.S2 + kShRows - 1) / kShRows;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < Cfg::kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    *abort_flag = 0;
    *fail_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&a.tq);
    if (a.S1 > 0) {
      tma_prefetch_desc(&a.tk1);
      tma_prefetch_desc(&a.tv1);
    }
    if (a.S2 > 0) {
      tma_prefetch_desc(&a.tk2);
      tma_prefetch_desc(&a.tv2);
    }
    if (a.mask_tma) tma_prefetch_desc(&a.tm);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  // Rows a box does not cover are read by the MMAs too: zero the Q copies when
  // there are fewer than 32 queries, and each stage whose first block comes
  // from a source shorter than 128 keys (masked keys need finite V rows).
  {
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    if (a.Sq < kShQ)
      for (int i = threadIdx.x; i < kShTile / 16; i += blockDim.x) reinterpret_cast<uint4*>(sQ)[i] = z;
    const int first_short[2] = {a.box1 < kShRows && nb1 > 0 ? 0 : -1, a.box2 < kShRows && nb > nb1 ? nb1 : -1};
    for (int f = 0; f < 2; ++f) {
      const int j = first_short[f];
      if (j < 0 || j >= Cfg::kStages) continue;
      for (int i = threadIdx.x; i < kShTile / 16; i += blockDim.x) {
        reinterpret_cast<uint4*>(sK + j * kShTile)[i] = z;
        reinterpret_cast<uint4*>(sV + j * kShTile)[i] = z;
      }
    }
    fence_async_smem();  // generic-proxy stores before the TMA writes and MMA reads
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_kv = policy_evict_first();  // every K/V tile is read by this CTA only
      const uint64_t pol_q = policy_evict_last();
      auto load_block = [&](int j) {
        const int s = j % Cfg::kStages;
        mbar_arrive_expect_tx(&kv_full[s], 2 * 128 * (j < nb1 ? a.box1 : a.box2) + (a.mask_tma ? a.Sq * kShRows : 0));
        if (a.mask_tma)
          tma_load_2d(sMk + s * kShMaskTile, &a.tm, &kv_full[s], j < nb1 ? j * kShRows : a.S1 + (j - nb1) * kShRows,
                      0, pol_q);
        if (j < nb1) {
          tma_load_3d(sK + s * kShTile, &a.tk1, &kv_full[s], h * kShHd, j * kShRows, b, pol_kv);
          tma_load_3d(sV + s * kShTile, &a.tv1, &kv_full[s], h * kShHd, j * kShRows, b, pol_kv);
        } else {
          tma_load_3d(sK + s * kShTile, &a.tk2, &kv_full[s], h * kShHd, (j - nb1) * kShRows, b, pol_kv);
          tma_load_3d(sV + s * kShTile, &a.tv2, &kv_full[s], h * kShHd, (j - nb1) * kShRows, b, pol_kv);
        }
      };
      int issued = 0;
      // cache blocks stream in before the programmatic-launch wait when no
      // earlier kernel of the chain writes them
      if (a.kv1_const)
        for (; issued < Cfg::kStages && issued < nb1; ++issued) load_block(issued);
      pdl_wait();
      mbar_arrive_expect_tx(q_full, 4 * a.Sq * 128);
      for (int r = 0; r < 4; ++r) tma_load_3d(sQ + r * kShQ * 128, &a.tq, q_full, h * kShHd, 0, b, pol_q);
      for (int j = issued; j < nb; ++j) {
        const int s = j % Cfg::kStages;
        if (*abort_flag) break;
        if (j >= Cfg::kStages &&
            !mbar_wait(&kv_empty[s], static_cast<uint32_t>(j / Cfg::kStages - 1) & 1, a.status, kErrShortWait)) {
          *abort_flag = 1;
          break;
        }
        load_block(j);
        issued = j + 1;
      }
      // every issued copy has landed before the CTA can exit
      mbar_wait(q_full, 0, a.status, kErrShortWait);
      for (int j = max(0, issued - Cfg::kStages); j < issued; ++j)
        mbar_wait(&kv_full[j % Cfg::kStages], static_cast<uint32_t>(j / Cfg::kStages) & 1, a.status, kErrShortWait);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_bf16(kShRows, kShRows);
      const uint32_t idesc_pv = umma_idesc_bf16_bmn(kShRows, kShHd);
      bool ok = mbar_wait(q_full, 0, a.status, kErrShortWait);
      auto issue_s = [&](int j) -> bool {
        const int s = j % Cfg::kStages;
        if (!mbar_wait(&kv_full[s], static_cast<uint32_t>(j / Cfg::kStages) & 1, a.status, kErrShortWait)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kShHd / 16; ++kk)
          umma_bf16_ss(tmem_base + Cfg::kColS + 128 * (j % kSB), umma_desc_sw128(sQ) + 2 * kk,
                       umma_desc_sw128(sK + s * kShTile) + 2 * kk, idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[j % kSB]);
        return true;
      };
      if (ok && nb > 0) ok = issue_s(0);
      if (kSB > 1 && ok && nb > 1) ok = issue_s(1);
      for (int j = 0; ok && j < nb; ++j) {
        if (*abort_flag ||
            !mbar_wait(&p_full[j % kPB], static_cast<uint32_t>(j / kPB) & 1, a.status, kErrShortWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int s = j % Cfg::kStages;
#pragma unroll
        for (int kk = 0; kk < kShRows / 16; ++kk)
          umma_bf16_ts(tmem_base + Cfg::kColO, tmem_base + Cfg::kColP + 64 * (j % kPB) + 8 * kk,
                       umma_desc_sw128_mn(sV + s * kShTile + kk * 16 * 128), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&pv_done[j % kPB]);
        umma_commit(&kv_empty[s]);  // K_j (read by S(j)) and V_j consumed
        if (j + kSB < nb) ok = issue_s(j + kSB);  // S buffer j % kSB was read by softmax(j)
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp >= 4) {
    pdl_wait();  // the output rows are read by the previous layer's launches
    const int wq = warp - 4;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(wq * 32) << 16);
    {
      const uint32_t z[16] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
      for (int c = 0; c < 4 * kPB; ++c) tmem_st16(lane_addr + Cfg::kColP + 16 * c, z);
      tmem_wait_st();
    }
    const int q = lane;
    const bool row_ok = q < a.Sq;
    const uint8_t* km = a.key_mask != nullptr ? a.key_mask + static_cast<long long>(b) * a.key_mask_bs : nullptr;
    const uint8_t* mrow = (a.mask2d != nullptr && row_ok) ? a.mask2d + static_cast<long long>(q) * a.mask_rs : nullptr;
    // keys [kg0, kg0 + nv) of the concatenated key list are this warp's in block j
    auto block_keys = [&](int j, int& kg0, int& nv) {
      const bool src1 = j < nb1;
      const int kb = (src1 ? j : j - nb1) * kShRows + 32 * wq;
      nv = max(0, min(32, (src1 ? a.S1 : a.S2) - kb));
      kg0 = (src1 ? 0 : a.S1) + kb;
    };
    // the attend words (32 bytes of this row, when aligned) and this lane's key-mask
    // byte of block j, loaded one block ahead of their use
    uint4 mw0 = make_uint4(0u, 0u, 0u, 0u), mw1 = mw0;
    int kmv = 0;
    auto prefetch = [&](int j) {
      int kg0, nv;
      block_keys(j, kg0, nv);
      if (mrow != nullptr && !a.mask_tma && nv >= 32 && (reinterpret_cast<uintptr_t>(mrow + kg0) & 15) == 0) {
        mw0 = __ldg(reinterpret_cast<const uint4*>(mrow + kg0));
        mw1 = __ldg(reinterpret_cast<const uint4*>(mrow + kg0 + 16));
      }
      kmv = (km != nullptr && lane < nv) ? km[kg0 + lane] : 0;
    };
    if (nb > 0) prefetch(0);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nb && ok; ++j) {
      // warp-uniform outcome of every wait: the TMEM loads and stores are warp-collective
      bool got = mbar_wait(&s_full[j % kSB], static_cast<uint32_t>(j / kSB) & 1, a.status, kErrShortWait);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[32];
      tmem_ld32(lane_addr + Cfg::kColS + 128 * (j % kSB) + 32 * wq, sv);
      int kg0, nv;
      block_keys(j, kg0, nv);
      uint32_t bits = nv >= 32 ? 0xffffffffu : ((1u << nv) - 1u);
      if (km != nullptr) bits &= __ballot_sync(0xffffffffu, kmv != 0);
      if (!row_ok) {
        bits = 0u;
      } else if (a.mask_tma) {
        // the block's attend tile landed with its K / V (kv_full of the stage)
        const int s = j % Cfg::kStages;
        got = mbar_wait(&kv_full[s], static_cast<uint32_t>(j / Cfg::kStages) & 1, a.status, kErrShortWait);
        const uint4* t4 = reinterpret_cast<const uint4*>(sMk + s * kShMaskTile + q * kShRows + 32 * wq);
        bits = got ? bits & word_bits(t4[0], t4[1]) : 0u;
      } else if (mrow != nullptr) {
        bits &= (nv >= 32 && (reinterpret_cast<uintptr_t>(mrow + kg0) & 15) == 0) ? word_bits(mw0, mw1)
                                                                                : attend_bits(mrow + kg0, nv);
      }
      if (j + 1 < nb) prefetch(j + 1);
      tmem_wait_ld();
      // one warp per SM sub-partition runs this: keep the dependency chains short
      // (tree maximum, four partial sums) and skip the per-key selects when every
      // key of the slice is visible to every row of the warp (a second softmax
      // warp per quarter sharing the running maximum measured slower: the
      // per-block exchange cost more than the halved element work)
      const bool full = __all_sync(0xffffffffu, bits == 0xffffffffu);
      if (!full) {
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[i] = ((bits >> i) & 1u) ? sv[i] : -INFINITY;
      }
      float t16[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) t16[i] = fmaxf(sv[i], sv[i + 16]);
#pragma unroll
      for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int i = 0; i < w; ++i) t16[i] = fmaxf(t16[i], t16[i + w]);
      float mx = t16[0];
      mx = mx == -INFINITY ? mx : mx * a.scale_log2;  // scale_log2 > 0
      float alpha = 1.f;
      if (mx > m + kShLazy || (m == -INFINITY && mx > -INFINITY)) {
        alpha = m == -INFINITY ? 0.f : exp2f(m - mx);
        m = mx;
      }
      const float base = m == -INFINITY ? 0.f : m;
      float psa[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float p0 = exp2f(fmaf(sv[i], a.scale_log2, -base));  // exp2(-inf) = 0 for hidden keys
        const float p1 = exp2f(fmaf(sv[i + 1], a.scale_log2, -base));
        psa[(i >> 1) & 3] += p0 + p1;
        pk[i / 2] = pack2_bf16(p0, p1);
      }
      const float ps = (psa[0] + psa[1]) + (psa[2] + psa[3]);
      // P buffer j % kPB was last read by P(j-kPB).V(j-kPB)
      got = j < kPB || mbar_wait(&pv_done[j % kPB], static_cast<uint32_t>(j / kPB - 1) & 1, a.status, kErrShortWait);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      if (j > 0 && !__all_sync(0xffffffffu, alpha == 1.f)) {
        // rescale O once P(j-1).V(j-1) (and with it every earlier P.V) is complete
        got = mbar_wait(&pv_done[(j - 1) % kPB], static_cast<uint32_t>((j - 1) / kPB) & 1, a.status, kErrShortWait);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        {
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            float ov[32];
            tmem_ld32(lane_addr + Cfg::kColO + 32 * c, ov);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= alpha;
            tmem_st32(lane_addr + Cfg::kColO + 32 * c, ov);
          }
        }
      }
      tc_fence_after();
      tmem_st16(lane_addr + Cfg::kColP + 64 * (j % kPB) + 16 * wq, pk);
      l = l * alpha + ps;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j % kPB]);
    }
    if (!ok) *abort_flag = 1;
    const bool fin = ok && nb > 0 &&
                     mbar_wait(&pv_done[(nb - 1) % kPB], static_cast<uint32_t>((nb - 1) / kPB) & 1, a.status, kErrShortWait);
    if (__all_sync(0xffffffffu, fin)) {
      tc_fence_after();
      float* orow = so + (wq * kShQ + q) * kShMergeRow;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float ov[32];
        tmem_ld32(lane_addr + Cfg::kColO + 32 * c, ov);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i)
          reinterpret_cast<float4*>(orow + 32 * c)[i] = make_float4(ov[4 * i], ov[4 * i + 1], ov[4 * i + 2], ov[4 * i + 3]);
      }
      sml[(wq * kShQ + q) * 2] = m;
      sml[(wq * kShQ + q) * 2 + 1] = l;
    } else if (lane == 0) {
      *fail_flag = 1;
    }
    // merge the four quarters: every softmax warp reaches this barrier once
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (*fail_flag == 0) {
      const int t = threadIdx.x - 128;
      const int r = t >> 2, d0 = (t & 3) * 16;
      if (r < a.Sq) {
        float mq[4], M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          mq[w] = sml[(w * kShQ + r) * 2];
          M = fmaxf(M, mq[w]);
        }
        float wt[4], L = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          wt[w] = mq[w] == -INFINITY ? 0.f : exp2f(mq[w] - M);
          L += wt[w] * sml[(w * kShQ + r) * 2 + 1];
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        float acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float* src = so + (w * kShQ + r) * kShMergeRow + d0;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 v = reinterpret_cast<const float4*>(src)[i];
            acc[4 * i] += wt[w] * v.x;
            acc[4 * i + 1] += wt[w] * v.y;
            acc[4 * i + 2] += wt[w] * v.z;
            acc[4 * i + 3] += wt[w] * v.w;
          }
        }
        __nv_bfloat16* dst = a.out + static_cast<long long>(b) * a.out_bs + static_cast<long long>(r) * a.out_ts +
                             h * kShHd + d0;
        reinterpret_cast<uint4*>(dst)[0] =
            make_uint4(pack2_bf16(acc[0] * inv, acc[1] * inv), pack2_bf16(acc[2] * inv, acc[3] * inv),
                       pack2_bf16(acc[4] * inv, acc[5] * inv), pack2_bf16(acc[6] * inv, acc[7] * inv));
        reinterpret_cast<uint4*>(dst)[1] =
            make_uint4(pack2_bf16(acc[8] * inv, acc[9] * inv), pack2_bf16(acc[10] * inv, acc[11] * inv),
                       pack2_bf16(acc[12] * inv, acc[13] * inv), pack2_bf16(acc[14] * inv, acc[15] * inv));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

// Builds the launch's tensor maps; false (nothing launched) when the shape or
// the layout is outside what the kernel takes.  At batch x heads below about
// one wave of CTAs (128) the split-KV attention_kernel keeps more SMs busy.
static bool prepare_attention_short_tc(const AttnArgs& a, int B, int head_dim, AttnShortArgs* s) {
  if (head_dim != kShHd || a.Sq < 1 || a.Sq > kShQ || a.first_frame_tokens != 0 || a.S1 < 0 || a.S2 < 0 ||
      a.S1 + a.S2 <= 0 || static_cast<long long>(B) * a.H < 128)
    return false;
  if (!aligned16(a.q) || !aligned16(a.out) || ((a.q_ts | a.q_bs | a.out_ts | a.out_bs) & 7) != 0) return false;
  const uint64_t cols = static_cast<uint64_t>(a.H) * kShHd;
  memset(s, 0, sizeof(*s));
  // boxes no taller than the tensor (the encoder rejects taller ones)
  s->box1 = a.S1 < kShRows ? a.S1 : kShRows;
  s->box2 = a.S2 < kShRows ? a.S2 : kShRows;
  if (!make_tmap_bf16_3d(&s->tq, a.q, B, a.Sq, cols, a.q_ts, a.q_bs, a.Sq)) return false;
  if (a.S1 > 0) {
    if (!aligned16(a.k1) || !aligned16(a.v1) || ((a.kv1_ts | a.kv1_bs) & 7) != 0 ||
        !make_tmap_bf16_3d(&s->tk1, a.k1, B, a.S1, cols, a.kv1_ts, a.kv1_bs, s->box1) ||
        !make_tmap_bf16_3d(&s->tv1, a.v1, B, a.S1, cols, a.kv1_ts, a.kv1_bs, s->box1))
      return false;
  }
  if (a.S2 > 0) {
    if (!aligned16(a.k2) || !aligned16(a.v2) || ((a.kv2_ts | a.kv2_bs) & 7) != 0 ||
        !make_tmap_bf16_3d(&s->tk2, a.k2, B, a.S2, cols, a.kv2_ts, a.kv2_bs, s->box2) ||
        !make_tmap_bf16_3d(&s->tv2, a.v2, B, a.S2, cols, a.kv2_ts, a.kv2_bs, s->box2))
      return false;
  }
  // attend tiles by TMA: 16-byte rows and block offsets (source 2 starts at S1)
  s->mask_tma = a.mask2d != nullptr && aligned16(a.mask2d) && a.mask_rs % 16 == 0 && (a.S2 == 0 || a.S1 % 16 == 0) &&
                make_tmap_u8_2d(&s->tm, a.mask2d, a.Sq, a.S1 + a.S2, a.mask_rs, kShRows, a.Sq);
  s->mask2d = a.mask2d;
  s->mask_rs = a.mask_rs;
  s->key_mask = a.key_mask;
  s->key_mask_bs = a.key_mask_bs;
  s->out = a.out;
  s->out_bs = a.out_bs;
  s->out_ts = a.out_ts;
  s->Sq = a.Sq;
  s->S1 = a.S1;
  s->S2 = a.S2;
  s->kv1_const = a.kv1_const;
  s->scale_log2 = a.scale_log2;
  s->status = a.status;
  return true;
}

template <bool kCompact>
static cudaError_t launch_short_cfg(const AttnShortArgs& s, int B, int H, cudaStream_t st, bool pdl) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(attention_short_tc_kernel<kCompact>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, ShCfg<kCompact>::kSmem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  cudaLaunchAttribute attr_l[1];
  attr_l[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr_l[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(H, B);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = ShCfg<kCompact>::kSmem;
  cfg.stream = st;
  cfg.attrs = attr_l;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attention_short_tc_kernel<kCompact>, s);
}

cudaError_t launch_attention_auto(const AttnArgs& a, int B, int head_dim, cudaStream_t st, bool pdl) {
  AttnShortArgs s;
  if (!prepare_attention_short_tc(a, B, head_dim, &s)) return launch_attention(a, B, head_dim, st, pdl);
  // beyond two waves of one CTA per SM, two CTAs share each SM
  return static_cast<long long>(B) * a.H > 2 * 148 ? launch_short_cfg<true>(s, B, a.H, st, pdl)
                                                    : launch_short_cfg<false>(s, B, a.H, st, pdl);
}

bool attention_short_tc_taken(const AttnArgs& a, int B, int head_dim) {
  AttnShortArgs s;
  return prepare_attention_short_tc(a, B, head_dim, &s);
}

}  // namespace fam
