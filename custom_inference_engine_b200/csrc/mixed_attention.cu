// Varlen mixed attention (chunked prefill + decode rows) on 5th-generation
// tensor cores (tcgen05 + TMEM) for sm_100a.
//
// Replaces mixed_gqa_attention_kernel (kernels/prefill_attention.py:10-198)
// behind the host contract of attn/core.py:69-111.
//
// One CTA owns one query tile of one (sequence, kv head): 18 consecutive
// tokens x the 7 query heads that share the kv head = 126 rows of the
// tcgen05 M = 128 tile (the reference pads 7 heads to 8 and uses 16 tokens,
// 112 useful rows of 128). The tile is a single TMA box over q viewed as
// (token, kv head, head-in-group, dim), so row r = token * 7 + head.
//
// Warp roles (192 threads):
//   warp 0      TMA producer: the Q tile once, then per 128-key block the
//               8 K pages and 8 V pages of this kv head (2 KiB boxes through
//               the block table) into a 3-stage ring;
//   warp 1      TMEM owner and single-thread MMA issuer:
//               S_j = Q K_j^T (M128 N128 K16 x4) into one of two S buffers,
//               then PV_{j-1} = P_{j-1} V_{j-1} (M128 N64 K16 x8) into one of
//               two PV buffers, so block j's QK^T overlaps block j-1's softmax;
//   warps 2-5   softmax: thread = TMEM lane = tile row. Reads S_j, applies
//               scale, causal limit and online max, writes fp16 P_j to shared
//               memory in the 128B-swizzled K-major layout the MMA reads, then
//               folds PV_{j-1} into fp32 registers: O = O * alpha + PV, the
//               same update as the reference (acc * alpha + dot(P, V)).
// All waits are bounded; on a timeout the kernel records
// CIE_DEVERR_WAIT_TIMEOUT, drains its own copies and MMAs, frees TMEM and
// returns.
#include <math_constants.h>

#include "cie_common.cuh"
#include "cie_host.h"

namespace cie {
namespace mixed {

constexpr int kD = 64;
constexpr int kPage = 16;
constexpr int kGroup = 7;
constexpr int kTileTokens = 18;
constexpr int kRows = kTileTokens * kGroup;  // 126 useful rows of M = 128
constexpr int kM = 128;
constexpr int kBlockKeys = 128;
constexpr int kPagesPerBlock = kBlockKeys / kPage;  // 8
constexpr int kStages = 3;
constexpr int kThreads = 192;

constexpr int kQBytes = kM * kD * 2;             // 16 KiB
constexpr int kQLoadBytes = kRows * kD * 2;      // 16128 bytes delivered by the box
constexpr int kKVTileBytes = kBlockKeys * kD * 2;  // 16 KiB per K or V block
constexpr int kStageBytes = 2 * kKVTileBytes;
constexpr int kPBytes = kM * kBlockKeys * 2;     // 32 KiB
constexpr int kPageBoxBytes = kPage * kD * 2;    // 2 KiB

constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + kQBytes;
constexpr int kOffP = kOffKV + kStages * kStageBytes;
constexpr int kOffBar = kOffP + 2 * kPBytes;
// barriers: kv_full[3], kv_empty[3], q_full, s_full[2], s_free[2], p_full[2],
// pv_full[2], pv_free[2], mma_done; then the TMEM base address
constexpr int kNumBars = 2 * kStages + 1 + 2 * 5 + 1;
constexpr int kOffTmemPtr = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = 1024 + kOffTmemPtr + 16;

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;     // two 128-column S buffers
constexpr uint32_t kColPV = 256;  // two 64-column PV buffers

constexpr uint32_t kIdescS = idesc_f16_f32(kM, kBlockKeys, false);
constexpr uint32_t kIdescPV = idesc_f16_f32(kM, kD, true);

struct Params {
  const int64_t* cu_seqlens;
  const int64_t* kv_lens;
  const int64_t* slot_ids;
  const int64_t* block_table;
  __half* o;
  int64_t total_tokens;
  int64_t max_seqlen;
  int64_t n_pages;
  int64_t n_slots;
  int64_t bt_stride;
  int num_q_heads;
};

struct Bars {
  uint32_t base;
  __device__ uint32_t kv_full(int s) const { return base + 8u * s; }
  __device__ uint32_t kv_empty(int s) const { return base + 8u * (kStages + s); }
  __device__ uint32_t q_full() const { return base + 8u * (2 * kStages); }
  __device__ uint32_t s_full(int b) const { return base + 8u * (2 * kStages + 1 + b); }
  __device__ uint32_t s_free(int b) const { return base + 8u * (2 * kStages + 3 + b); }
  __device__ uint32_t p_full(int b) const { return base + 8u * (2 * kStages + 5 + b); }
  __device__ uint32_t pv_full(int b) const { return base + 8u * (2 * kStages + 7 + b); }
  __device__ uint32_t pv_free(int b) const { return base + 8u * (2 * kStages + 9 + b); }
  __device__ uint32_t mma_done() const { return base + 8u * (2 * kStages + 11); }
};

__global__ void __launch_bounds__(kThreads, 1)
    mixed_attention_kernel(const __grid_constant__ CUtensorMap tm_q,
                           const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase + kOffQ;
  const uint32_t sKV = sbase + kOffKV;
  const uint32_t sP = sbase + kOffP;
  const Bars bars{sbase + kOffBar};
  uint32_t* tmem_ptr_smem = reinterpret_cast<uint32_t*>(smem + kOffTmemPtr);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;

  // ---- sequence bounds (uniform across the CTA) -----------------------------
  const int64_t start = p.cu_seqlens[b];
  const int64_t end = p.cu_seqlens[b + 1];
  if (start < 0 || end < start || end > p.total_tokens) {
    if (threadIdx.x == 0) raise_error(CIE_DEVERR_BAD_SEQLENS);
    return;
  }
  const int64_t L64 = end - start;
  if (tile == 0 && L64 > p.max_seqlen && threadIdx.x == 0) raise_error(CIE_DEVERR_BAD_SEQLENS);
  const int tok0 = tile * kTileTokens;
  if (tok0 >= L64) return;
  const int L = static_cast<int>(L64);
  const int64_t slot = p.slot_ids[b];
  if (slot < 0 || slot >= p.n_slots) {
    if (threadIdx.x == 0) raise_error(CIE_DEVERR_BAD_SLOT);
    return;
  }
  int64_t kv_len = p.kv_lens[b];
  if (kv_len < 0) kv_len = 0;
  const int tile_tokens = min(L - tok0, kTileTokens);
  int64_t n_keys64 = kv_len + tok0 + tile_tokens;  // keys visible to the tile's last row
  if ((kv_len + L + kPage - 1) / kPage > p.bt_stride) {
    if (threadIdx.x == 0) raise_error(CIE_DEVERR_BAD_LENGTH);
    return;
  }
  const int n_keys = static_cast<int>(n_keys64);
  const int n_blocks = (n_keys + kBlockKeys - 1) / kBlockKeys;
  const int n_valid_pages = (n_keys + kPage - 1) / kPage;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bars.kv_full(s), 1);
      mbar_init(bars.kv_empty(s), 1);
    }
    mbar_init(bars.q_full(), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(bars.s_full(i), 1);
      mbar_init(bars.s_free(i), 128);
      mbar_init(bars.p_full(i), 128);
      mbar_init(bars.pv_full(i), 1);
      mbar_init(bars.pv_free(i), 128);
    }
    mbar_init(bars.mma_done(), 1);
    fence_mbar_init();
  }
  // Q rows 126 and 127 are never loaded: zero them so the tensor core only
  // ever sees finite values there.
  if (threadIdx.x < 16) {
    const uint32_t addr = sQ + kRows * 128 + threadIdx.x * 16;
    asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
  }
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_ptr_smem), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_ptr_smem;

  if (warp == 0) {
    // ============================ producer ====================================
    int issued = 0;
    bool ok = true;
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(bars.q_full(), kQLoadBytes);
      tma_load_4d(sQ, &tm_q, bars.q_full(), 0, 0, h, static_cast<int>(start) + tok0);
    }
    const int64_t* bt_row = p.block_table + slot * p.bt_stride;
    for (int j = 0; j < n_blocks; ++j) {
      const int s = j % kStages;
      const uint32_t use = static_cast<uint32_t>(j / kStages);
      if (lane == 0) {
        if (j >= kStages && !mbar_wait(bars.kv_empty(s), (use & 1u) ^ 1u, CIE_DEVERR_WAIT_TIMEOUT))
          ok = false;
        if (ok) mbar_arrive_expect_tx(bars.kv_full(s), kStageBytes);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      if (lane < kPagesPerBlock) {
        const int lp = j * kPagesPerBlock + lane;
        int page = 0;
        if (lp < n_valid_pages) {
          int64_t pid = bt_row[lp];
          if (pid < 0 || pid >= p.n_pages) {
            raise_error(CIE_DEVERR_BAD_PAGE);
            pid = 0;
          }
          page = static_cast<int>(pid);
        }
        const uint32_t dst = sKV + s * kStageBytes + lane * kPageBoxBytes;
        tma_load_4d(dst, &tm_k, bars.kv_full(s), 0, 0, h, page);
        tma_load_4d(dst + kKVTileBytes, &tm_v, bars.kv_full(s), 0, 0, h, page);
      }
      __syncwarp();
      ++issued;
    }
    if (lane == 0) {
      mbar_wait(bars.q_full(), 0, CIE_DEVERR_WAIT_TIMEOUT);
      for (int j = max(0, issued - kStages); j < issued; ++j)
        mbar_wait(bars.kv_full(j % kStages), static_cast<uint32_t>(j / kStages) & 1u,
                  CIE_DEVERR_WAIT_TIMEOUT);
    }
  } else if (warp == 1) {
    // ============================ MMA issuer ==================================
    if (lane == 0) {
      bool ok = mbar_wait(bars.q_full(), 0, CIE_DEVERR_WAIT_TIMEOUT);
      const uint64_t dq = smem_desc(sQ, 16, 1024);
      auto issue_pv = [&](int i) -> bool {
        const int pb = i & 1;
        const uint32_t use = static_cast<uint32_t>(i >> 1);
        if (!mbar_wait(bars.p_full(pb), use & 1u, CIE_DEVERR_WAIT_TIMEOUT)) return false;
        if (i >= 2 && !mbar_wait(bars.pv_free(pb), (use & 1u) ^ 1u, CIE_DEVERR_WAIT_TIMEOUT))
          return false;
        tc_fence_after();
        const int s = i % kStages;
        const uint32_t v_tile = sKV + s * kStageBytes + kKVTileBytes;
        const uint32_t p_tile = sP + pb * kPBytes;
#pragma unroll
        for (int kk = 0; kk < kBlockKeys / 16; ++kk) {
          const uint64_t da = smem_desc(p_tile + (kk >> 2) * (kM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t db = smem_desc(v_tile + kk * 2048, kKVTileBytes, 1024);
          tc_mma_f16(tmem + kColPV + pb * kD, da, db, kIdescPV, kk > 0 ? 1u : 0u);
        }
        tc_commit(bars.pv_full(pb));
        tc_commit(bars.kv_empty(s));
        return true;
      };
      for (int j = 0; ok && j < n_blocks; ++j) {
        const int s = j % kStages;
        const int sb = j & 1;
        if (!mbar_wait(bars.kv_full(s), static_cast<uint32_t>(j / kStages) & 1u,
                       CIE_DEVERR_WAIT_TIMEOUT)) {
          ok = false;
          break;
        }
        if (j >= 2 && !mbar_wait(bars.s_free(sb), (static_cast<uint32_t>(j >> 1) & 1u) ^ 1u,
                                 CIE_DEVERR_WAIT_TIMEOUT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_tile = sKV + s * kStageBytes;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          const uint64_t da = smem_desc(sQ + k * 32, 16, 1024);
          const uint64_t db = smem_desc(k_tile + k * 32, 16, 1024);
          tc_mma_f16(tmem + kColS + sb * kBlockKeys, da, db, kIdescS, k > 0 ? 1u : 0u);
        }
        (void)dq;
        tc_commit(bars.s_full(sb));
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && n_blocks > 0) issue_pv(n_blocks - 1);
      // drain: every MMA this thread issued has completed before TMEM is freed
      tc_commit(bars.mma_done());
      mbar_wait(bars.mma_done(), 0, CIE_DEVERR_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ============================ softmax =====================================
    const int quad = warp & 3;              // TMEM lane quadrant of this warp
    const int row = quad * 32 + lane;       // tile row == TMEM lane
    const int tok_in_tile = row / kGroup;
    const int head_in_group = row - tok_in_tile * kGroup;
    const bool row_valid = row < kRows && tok_in_tile < tile_tokens;
    // inclusive causal limit of this row; padded rows use the tile's first
    // row limit so that every value they produce stays finite
    const int limit = static_cast<int>(kv_len) + tok0 + (row_valid ? tok_in_tile : 0);
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    constexpr float kScale = 0.125f;  // head_dim ** -0.5 for D = 64

    float m_run = -CUDART_INF_F;
    float l_run = 0.f;
    float alpha_prev = 1.f;
    float o_acc[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) o_acc[d] = 0.f;

    auto fold_pv = [&](int i, float alpha) -> bool {
      const int pb = i & 1;
      if (!mbar_wait(bars.pv_full(pb), static_cast<uint32_t>(i >> 1) & 1u, CIE_DEVERR_WAIT_TIMEOUT))
        return false;
      tc_fence_after();
      uint32_t r0[32], r1[32];
      tmem_ld_32x32b_x32(tmem + lane_addr + kColPV + pb * kD, r0);
      tmem_ld_32x32b_x32(tmem + lane_addr + kColPV + pb * kD + 32, r1);
      tc_wait_ld();
      tc_fence_before();
      mbar_arrive(bars.pv_free(pb));
#pragma unroll
      for (int d = 0; d < 32; ++d) {
        o_acc[d] = o_acc[d] * alpha + __uint_as_float(r0[d]);
        o_acc[32 + d] = o_acc[32 + d] * alpha + __uint_as_float(r1[d]);
      }
      return true;
    };

    bool ok = true;
    for (int j = 0; j < n_blocks; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(bars.s_full(sb), static_cast<uint32_t>(j >> 1) & 1u, CIE_DEVERR_WAIT_TIMEOUT)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[kBlockKeys];
#pragma unroll
      for (int c = 0; c < kBlockKeys / 32; ++c)
        tmem_ld_32x32b_x32(tmem + lane_addr + kColS + sb * kBlockKeys + c * 32,
                           *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tc_wait_ld();
      tc_fence_before();
      mbar_arrive(bars.s_free(sb));

      const int lim = limit - j * kBlockKeys;  // last visible column of this block
      float mx = -CUDART_INF_F;
      if (lim >= kBlockKeys - 1) {
#pragma unroll
        for (int c = 0; c < kBlockKeys; ++c) {
          const float x = __uint_as_float(sr[c]) * kScale;
          sr[c] = __float_as_uint(x);
          mx = fmaxf(mx, x);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kBlockKeys; ++c) {
          const float x = c <= lim ? __uint_as_float(sr[c]) * kScale : -CUDART_INF_F;
          sr[c] = __float_as_uint(x);
          mx = fmaxf(mx, x);
        }
      }
      const float m_new = fmaxf(m_run, mx);  // finite: key 0 is visible to every row
      const float alpha = ex2((m_run - m_new) * kLog2e);
      const float mneg = m_new * kLog2e;
      float ls0 = 0.f, ls1 = 0.f, ls2 = 0.f, ls3 = 0.f;
      const uint32_t p_tile = sP + sb * kPBytes;
#pragma unroll
      for (int c8 = 0; c8 < kBlockKeys / 8; ++c8) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          pv[e] = ex2(fmaf(__uint_as_float(sr[c8 * 8 + e]), kLog2e, -mneg));
        ls0 += pv[0] + pv[4];
        ls1 += pv[1] + pv[5];
        ls2 += pv[2] + pv[6];
        ls3 += pv[3] + pv[7];
        const uint32_t w0 = pack_half2(pv[0], pv[1]);
        const uint32_t w1 = pack_half2(pv[2], pv[3]);
        const uint32_t w2 = pack_half2(pv[4], pv[5]);
        const uint32_t w3 = pack_half2(pv[6], pv[7]);
        // K-major, 128B swizzle: keys [64a, 64a+64) of all rows form atom column a
        const uint32_t addr = p_tile + (c8 >> 3) * (kM * 128) + sw128(row, c8 & 7);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w0), "r"(w1),
                     "r"(w2), "r"(w3)
                     : "memory");
      }
      l_run = l_run * alpha + ((ls0 + ls1) + (ls2 + ls3));
      m_run = m_new;

      // V rows past the last key of the tile hold stale pool data: zero them
      // (each softmax thread owns one V row of the block) so that
      // 0 * (non-finite) cannot reach the accumulator.
      if (j == n_blocks - 1 && j * kBlockKeys + row >= n_keys) {
        const uint32_t vrow = sKV + (j % kStages) * kStageBytes + kKVTileBytes;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(vrow + sw128(row, c)),
                       "r"(0)
                       : "memory");
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(bars.p_full(sb));

      if (j >= 1 && !fold_pv(j - 1, alpha_prev)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    if (ok && n_blocks > 0) ok = fold_pv(n_blocks - 1, alpha_prev);

    if (ok && row_valid) {
      const float inv = 1.f / l_run;
      const int64_t tok = start + tok0 + tok_in_tile;
      __half* dst = p.o + (tok * p.num_q_heads + h * kGroup + head_in_group) * kD;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 w;
        w.x = pack_half2(o_acc[c * 8 + 0] * inv, o_acc[c * 8 + 1] * inv);
        w.y = pack_half2(o_acc[c * 8 + 2] * inv, o_acc[c * 8 + 3] * inv);
        w.z = pack_half2(o_acc[c * 8 + 4] * inv, o_acc[c * 8 + 5] * inv);
        w.w = pack_half2(o_acc[c * 8 + 6] * inv, o_acc[c * 8 + 7] * inv);
        reinterpret_cast<uint4*>(dst)[c] = w;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace mixed
}  // namespace cie

extern "C" int cie_mixed_attention(const void* q, const void* k, const void* v,
                                   int64_t max_seqlen, const int64_t* cu_seqlens,
                                   const int64_t* kv_lens, const int64_t* slot_ids,
                                   const int64_t* block_table, void* o, int batch,
                                   int64_t total_tokens, int num_q_heads, int num_kv_heads,
                                   int head_dim, int page_size, int64_t n_pages, int64_t n_slots,
                                   int64_t bt_stride, int64_t kv_page_stride,
                                   int64_t kv_head_stride, cie_stream_t stream) {
  using namespace cie;
  using namespace cie::mixed;
  if (batch < 0 || total_tokens < 0 || max_seqlen < 0)
    return fail(CIE_ERR_INVALID_ARGUMENT, "negative batch / total_tokens / max_seqlen");
  if (batch == 0 || total_tokens == 0 || max_seqlen == 0) return CIE_OK;
  if (!q || !k || !v || !cu_seqlens || !kv_lens || !slot_ids || !block_table || !o)
    return fail(CIE_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (head_dim != kD || page_size != kPage)
    return fail(CIE_ERR_UNSUPPORTED, "head_dim %d / page_size %d (supported: 64 / 16)", head_dim,
                page_size);
  if (num_kv_heads < 1 || num_q_heads != num_kv_heads * kGroup)
    return fail(CIE_ERR_UNSUPPORTED, "num_q_heads %d must be 7 * num_kv_heads (%d)", num_q_heads,
                num_kv_heads);
  if (n_pages < 1 || n_slots < 1 || bt_stride < 1)
    return fail(CIE_ERR_INVALID_ARGUMENT, "n_pages / n_slots / bt_stride must be >= 1");
  if (n_pages >= (int64_t(1) << 31) || total_tokens >= (int64_t(1) << 31) ||
      bt_stride * kPage >= (int64_t(1) << 31))
    return fail(CIE_ERR_OVERFLOW, "n_pages / total_tokens / keys per slot must fit int32");
  if (batch > 65535 || num_kv_heads > 65535)
    return fail(CIE_ERR_UNSUPPORTED, "batch %d / kv heads %d", batch, num_kv_heads);
  if (kv_head_stride < page_size * head_dim || kv_page_stride < kv_head_stride * num_kv_heads)
    return fail(CIE_ERR_INVALID_ARGUMENT, "overlapping K/V strides");
  if ((kv_page_stride % 8) || (kv_head_stride % 8) || !aligned16(k) || !aligned16(v) ||
      !aligned16(q) || !aligned16(o))
    return fail(CIE_ERR_ALIGNMENT, "q/o/k/v must be 16-byte aligned with 16-byte strides");
  const int64_t n_tiles = (max_seqlen + kTileTokens - 1) / kTileTokens;
  if (n_tiles > 0x7fffffff) return fail(CIE_ERR_OVERFLOW, "max_seqlen too large");

  CUtensorMap tm_q, tm_k, tm_v;
  {
    const uint64_t dims[4] = {kD, kGroup, static_cast<uint64_t>(num_kv_heads),
                              static_cast<uint64_t>(total_tokens)};
    const uint64_t strides[3] = {kD * 2, kGroup * kD * 2,
                                 static_cast<uint64_t>(num_q_heads) * kD * 2};
    const uint32_t box[4] = {kD, kGroup, 1, kTileTokens};
    int st = encode_tensor_map(&tm_q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(q),
                               dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != CIE_OK) return st;
  }
  {
    const uint64_t dims[4] = {kD, kPage, static_cast<uint64_t>(num_kv_heads),
                              static_cast<uint64_t>(n_pages)};
    const uint64_t strides[3] = {kD * 2, static_cast<uint64_t>(kv_head_stride) * 2,
                                 static_cast<uint64_t>(kv_page_stride) * 2};
    const uint32_t box[4] = {kD, kPage, 1, 1};
    int st = encode_tensor_map(&tm_k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(k), dims,
                               strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != CIE_OK) return st;
    st = encode_tensor_map(&tm_v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(v), dims,
                           strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != CIE_OK) return st;
  }
  int st = ensure_smem_attribute(reinterpret_cast<const void*>(&mixed_attention_kernel), kSmemBytes,
                                 8);
  if (st != CIE_OK) return st;

  Params p;
  p.cu_seqlens = cu_seqlens;
  p.kv_lens = kv_lens;
  p.slot_ids = slot_ids;
  p.block_table = block_table;
  p.o = static_cast<__half*>(o);
  p.total_tokens = total_tokens;
  p.max_seqlen = max_seqlen;
  p.n_pages = n_pages;
  p.n_slots = n_slots;
  p.bt_stride = bt_stride;
  p.num_q_heads = num_q_heads;
  dim3 grid(static_cast<unsigned>(n_tiles), num_kv_heads, batch);
  mixed_attention_kernel<<<grid, kThreads, kSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(
      tm_q, tm_k, tm_v, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "mixed launch: %s", cudaGetErrorString(e));
  return CIE_OK;
}
