// Split-KV paged GQA decode attention for sm_100a.
//
// Replaces the reference's decode_gqa_attention_kernel_load / _merge
// (kernels/decode_attention.py:12-272) behind the same host contract
// (attn/core.py:13-66).
//
// Design (B200-first):
//  * one CTA per (split, sequence) covers ALL kv heads of that sequence, so a
//    page is fetched as one 4 KiB TMA box per pool (both heads of
//    (page, :, 16, 64) are contiguous) into a deep ring of 128B-swizzled
//    shared-memory stages; a single producer warp reads the int64 block table
//    32 entries at a time and keeps every stage in flight;
//  * compute is tiny next to the bytes moved, so each consumer warp uses
//    warp-level MMA with the GQA group on the MMA's N side: S^T = K . Q^T
//    (M = 16 keys of a page, N = 8 >= 7 query heads, K = 64 dims) and
//    O^T += V^T . P^T; P^T is turned into the next B fragment with
//    movmatrix, so nothing goes back through shared memory;
//  * two consumer warps per kv head take alternate pages and are merged at
//    the end; with more than one split per sequence each CTA writes an
//    (m, l, acc) partial and a small merge kernel combines them.
// Numerics follow the reference: fp16 dot with fp32 accumulation, scale
// after the dot, fp32 online softmax, probabilities rounded to fp16 before
// P.V, one fp16 rounding of the output.
#include <math_constants.h>

#include "cie_common.cuh"
#include "cie_host.h"

namespace cie {
namespace decode {

constexpr int kD = 64;
constexpr int kPage = 16;
constexpr int kGroup = 7;
constexpr int kHeadTileBytes = kPage * kD * 2;  // 2 KiB: one head of one page

template <int HKV>
struct Cfg {
  static constexpr int kConsumerWarps = 2 * HKV;
  static constexpr int kThreads = 32 * (1 + kConsumerWarps);
  static constexpr int kStageBytes = 2 * HKV * kHeadTileBytes;  // K + V
  static constexpr int kStages = HKV == 1 ? 16 : (HKV == 2 ? 12 : 6);
  static constexpr int kRingBytes = kStages * kStageBytes;
  // merge scratch per kv head: m[8], l[8], acc[64][8] fp32
  static constexpr int kScratchFloats = 8 + 8 + kD * 8;
  static constexpr int kScratchBytes = HKV * kScratchFloats * 4;
  static constexpr int kBarBytes = 2 * kStages * 8;
  static constexpr int kSmemBytes = 1024 + kRingBytes + kScratchBytes + kBarBytes;
};

struct Params {
  const __half* q;            // (B, H_q, D)
  const int64_t* lens;        // (B,)
  const int64_t* slot_ids;    // (B,)
  BlockTable block_table;     // (n_slots, bt_stride)
  __half* o;                  // (B, H_q, D)
  float* ws_acc;              // (B, S, H_q, D)
  float* ws_ml;               // (B, S, H_q, 2)
  int batch;
  int num_splits;
  int64_t n_pages;
  int64_t n_slots;
  int64_t bt_stride;
  // Fused rotary embedding + KV write (cie_rope_kv_decode_attention), when qkv
  // is set: q comes from the fused QKV projection and is rotated in
  // registers; lens is then per SLOT (the length before this token), the
  // token sits at position lens[slot] and attends to lens[slot] + 1 keys; its
  // rotated k and its v are written to the pool and into the shared-memory
  // copy of their page.
  const __half* qkv;          // (B, (H_q + 2 H_kv) * D), row stride qkv_tok
  int64_t qkv_tok;
  const __half* cos;          // (B, D), row stride cs_tok
  const __half* sin;
  int64_t cs_tok;
  __half* k_cache;            // the pools, for the new row
  __half* v_cache;
  int64_t page_stride, head_stride;
};

// x * c + rot * s on 8 fp16 values, each operation rounded to fp16 (no fused
// multiply-add): transformers' apply_rotary_pos_emb step by step.
__device__ __forceinline__ uint4 rope8(uint4 x, uint4 rot, uint4 c, uint4 sn) {
  uint4 r;
  const __half2* xh = reinterpret_cast<const __half2*>(&x);
  const __half2* rh = reinterpret_cast<const __half2*>(&rot);
  const __half2* ch = reinterpret_cast<const __half2*>(&c);
  const __half2* sh = reinterpret_cast<const __half2*>(&sn);
  __half2* oh = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int e = 0; e < 4; ++e) oh[e] = __hadd2_rn(__hmul2_rn(xh[e], ch[e]), __hmul2_rn(rh[e], sh[e]));
  return r;
}

__device__ __forceinline__ uint4 neg8(uint4 x) {
  const __half2* xh = reinterpret_cast<const __half2*>(&x);
  uint4 r;
  __half2* oh = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int e = 0; e < 4; ++e) oh[e] = __hneg2(xh[e]);
  return r;
}

__device__ __forceinline__ uint4 ldg16(const __half* ptr) {
  return __ldg(reinterpret_cast<const uint4*>(ptr));
}

// Fewest pages a split is given: below this the fixed cost of a CTA (start-up,
// first TMA round trip, its partial) outweighs the bytes it streams.
constexpr int kMinPagesPerSplit = 4;

// Pages of sequence b that the kernels visit; 0 for an invalid slot. A length
// beyond the block-table row is clamped to it.
__device__ __forceinline__ int seq_pages(const int64_t* lens, const int64_t* slot_ids, int b,
                                         int64_t n_slots, int64_t bt_stride, int lens_per_slot) {
  const int64_t slot = slot_ids[b];
  if (slot < 0 || slot >= n_slots) return 0;
  // per sequence: keys visible to the query; per slot: the slot's length
  // before the query token, which is then written and attended to as well
  int64_t L = lens_per_slot ? lens[slot] + 1 : lens[b];
  if (L < 0) L = 0;
  const int64_t np = (L + kPage - 1) / kPage;
  return static_cast<int>(np > bt_stride ? bt_stride : np);
}

// Contiguous pages per split (the same partition in the split and merge kernels).
__device__ __forceinline__ int split_pages(int n_seq_pages, int S) {
  return max((n_seq_pages + S - 1) / S, kMinPagesPerSplit);
}

__device__ __forceinline__ float shfl_max_group(float x) {
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 4));
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 8));
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 16));
  return x;
}
__device__ __forceinline__ float shfl_sum_group(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  x += __shfl_xor_sync(0xffffffffu, x, 8);
  x += __shfl_xor_sync(0xffffffffu, x, 16);
  return x;
}

template <int HKV>
__global__ void __launch_bounds__(Cfg<HKV>::kThreads)
    decode_split_kernel(const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const Params p) {
  using C = Cfg<HKV>;
  constexpr int H_Q = HKV * kGroup;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* scratch = reinterpret_cast<float*>(smem + C::kRingBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kRingBytes + C::kScratchBytes);
  const uint32_t ring_u32 = smem_u32(ring);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8u * C::kStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int b = blockIdx.y;
  const int S = p.num_splits;

  // Launched as a programmatic dependent of the previous kernel in the stream:
  // the barriers and the tensor-map prefetch need none of its results, every
  // read of an input comes after griddepcontrol.wait.
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, HKV);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- per-sequence page range of this split -------------------------------
  int64_t slot = p.slot_ids[b];
  bool bad = false;
  if (slot < 0 || slot >= p.n_slots) {
    if (threadIdx.x == 0) raise_error(CIE_DEVERR_BAD_SLOT);
    bad = true;
  }
  int64_t L = p.qkv == nullptr ? p.lens[b] : (bad ? 0 : p.lens[slot] + 1);
  if (L < 0) L = 0;
  bool clamped = false;
  if (!bad && (L + kPage - 1) / kPage > p.bt_stride) {
    if (threadIdx.x == 0) raise_error(CIE_DEVERR_BAD_LENGTH);
    L = p.bt_stride * kPage;
    clamped = true;
  }
  if (bad) L = 0;
  const int n_seq_pages = static_cast<int>((L + kPage - 1) / kPage);
  const int pps = split_pages(n_seq_pages, S);
  const int page_begin = split * pps;
  const int n = max(0, min(page_begin + pps, n_seq_pages) - page_begin);
  const int Li = static_cast<int>(L);

  if (threadIdx.x == 0) {
    // let the merge kernel (launched with programmatic stream serialization)
    // get scheduled while this grid streams; it waits for our completion
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  }
  __syncthreads();

  if (warp == 0) {
    // ======================= producer warp ==================================
    const int64_t bt_row = slot * p.bt_stride + page_begin;
    auto page_id = [&](int j) -> int {  // block-table entry j of this split, checked
      if (j >= n) return 0;
      int64_t pid = p.block_table.at(bt_row + j);
      if (pid < 0 || pid >= p.n_pages) {
        raise_error(CIE_DEVERR_BAD_PAGE);
        pid = 0;
      }
      return static_cast<int>(pid);
    };
    bool abort = false;
    int issued = 0;
    int next_page = page_id(lane);
    for (int base = 0; base < n && !abort; base += 32) {
      const int page = next_page;
      // fetch the next 32 entries now; they are needed only after this batch
      next_page = page_id(base + 32 + lane);
      const int cnt = min(32, n - base);
      for (int t = 0; t < cnt; ++t) {
        const int pg = __shfl_sync(0xffffffffu, page, t);
        if (lane == 0) {
          const int i = base + t;
          const int s = i % C::kStages;
          const uint32_t use = static_cast<uint32_t>(i / C::kStages);
          if (i >= C::kStages && !mbar_wait(empty0 + 8u * s, (use & 1u) ^ 1u, CIE_DEVERR_WAIT_TIMEOUT))
            abort = true;
          if (!abort) {
            const uint32_t dst = ring_u32 + s * C::kStageBytes;
            mbar_arrive_expect_tx(full0 + 8u * s, C::kStageBytes);
            tma_load_4d(dst, &tm_k, full0 + 8u * s, 0, 0, 0, pg);
            tma_load_4d(dst + HKV * kHeadTileBytes, &tm_v, full0 + 8u * s, 0, 0, 0, pg);
            ++issued;
          }
        }
        abort = __shfl_sync(0xffffffffu, abort ? 1 : 0, 0) != 0;
        if (abort) break;
      }
    }
    // Never leave the CTA with bulk copies in flight: wait (bounded) for the
    // last load issued into every stage.
    if (lane == 0) {
      for (int i = max(0, issued - C::kStages); i < issued; ++i) {
        const int s = i % C::kStages;
        mbar_wait(full0 + 8u * s, static_cast<uint32_t>(i / C::kStages) & 1u,
                  CIE_DEVERR_WAIT_TIMEOUT);
      }
    }
    return;
  }

  // ========================= consumer warps ===================================
  const int cw = warp - 1;
  const int h = cw % HKV;        // kv head
  const int par = cw / HKV;      // page parity handled by this warp
  const int g = lane >> 2;       // fragment row group: query head within the group
  const int t4 = lane & 3;

  // Q^T as the B operand: b0 = Q[g][16ks + 2t4 .. +1], b1 = Q[g][16ks + 8 + 2t4 .. +1]
  uint32_t bq[4][2];
  if (p.qkv == nullptr) {
    const bool valid = g < kGroup;
    const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
        p.q + (static_cast<int64_t>(b) * H_Q + h * kGroup + (valid ? g : 0)) * kD);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      bq[ks][0] = valid ? qrow[(ks * 16 + 2 * t4) >> 1] : 0u;
      bq[ks][1] = valid ? qrow[(ks * 16 + 8 + 2 * t4) >> 1] : 0u;
    }
  } else {
    // rotate_half(x)[e] = -x[e + 32] (e < 32), x[e - 32] (e >= 32)
    const bool valid = g < kGroup && !bad;
    const __half2* qrow = reinterpret_cast<const __half2*>(
        p.qkv + static_cast<int64_t>(b) * p.qkv_tok + (h * kGroup + (valid ? g : 0)) * kD);
    const __half2* cs = reinterpret_cast<const __half2*>(p.cos + static_cast<int64_t>(b) * p.cs_tok);
    const __half2* sn = reinterpret_cast<const __half2*>(p.sin + static_cast<int64_t>(b) * p.cs_tok);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int e = ks * 16 + hf * 8 + 2 * t4;  // even: (e, e + 1) in one half
        const __half2 x = qrow[e >> 1];
        const __half2 rot = e < 32 ? __hneg2(qrow[(e + 32) >> 1]) : qrow[(e - 32) >> 1];
        const __half2 r = __hadd2_rn(__hmul2_rn(x, cs[e >> 1]), __hmul2_rn(rot, sn[e >> 1]));
        bq[ks][hf] = valid ? *reinterpret_cast<const uint32_t*>(&r) : 0u;
      }
    }
  }
  // fused mode: the page (index in this split) holding the new token, and its row
  const int new_i = (p.qkv != nullptr && Li > 0 && !clamped) ? (Li - 1) / kPage - page_begin : -1;
  const int new_row = (Li - 1) & (kPage - 1);

  constexpr float kScale = 0.125f;  // head_dim ** -0.5 for D = 64
  float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F;  // heads 2*t4, 2*t4+1
  float l0 = 0.f, l1 = 0.f;                      // per-thread partial sums
  float acc[4][4];
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[mt][e] = 0.f;

  for (int i = par; i < n; i += 2) {
    const int s = i % C::kStages;
    const uint32_t use = static_cast<uint32_t>(i / C::kStages);
    // ldmatrix / mma / movmatrix below are warp-collective: leave together
    if (!__all_sync(0xffffffffu, mbar_wait(full0 + 8u * s, use & 1u, CIE_DEVERR_WAIT_TIMEOUT)))
      break;
    // Head h's 16 rows start at a multiple of 1 KiB inside the stage, so the
    // 128B-swizzle phase of row r is r mod 8.
    const uint32_t kt = ring_u32 + s * C::kStageBytes + h * kHeadTileBytes;
    const uint32_t vt = kt + HKV * kHeadTileBytes;
    if (i == new_i) {
      // the new token: rotated k and v of kv head h into this page's row, in
      // shared memory (for this attention) and in the pool (for later steps);
      // lanes 0-7 own k chunks, lanes 8-15 v chunks of 8 elements
      if (lane < 16) {
        const int c = lane & 7;
        const __half* src = p.qkv + static_cast<int64_t>(b) * p.qkv_tok +
                            ((lane < 8 ? H_Q : H_Q + HKV) + h) * kD;
        uint4 val = ldg16(src + c * 8);
        if (lane < 8) {
          const __half* cs = p.cos + static_cast<int64_t>(b) * p.cs_tok + c * 8;
          const __half* sn = p.sin + static_cast<int64_t>(b) * p.cs_tok + c * 8;
          const uint4 partner = ldg16(src + (c ^ 4) * 8);
          val = rope8(val, c < 4 ? neg8(partner) : partner, ldg16(cs), ldg16(sn));
        }
        const uint32_t saddr = (lane < 8 ? kt : vt) + sw128(new_row, c);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(saddr), "r"(val.x),
                     "r"(val.y), "r"(val.z), "r"(val.w)
                     : "memory");
        int64_t pg = p.block_table.at(slot * p.bt_stride + (Li - 1) / kPage);
        if (pg >= 0 && pg < p.n_pages) {
          __half* dst = (lane < 8 ? p.k_cache : p.v_cache) + pg * p.page_stride +
                        h * p.head_stride + new_row * kD + c * 8;
          *reinterpret_cast<uint4*>(dst) = val;
        }
      }
      fence_proxy_async_smem();  // the stage is refilled by TMA later
      __syncwarp();
    }

    // S^T (16 keys x 8 heads) = K (16 x 64) . Q^T (64 x 8)
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(kt + sw128(lane & 15, ks * 2 + (lane >> 4)), a0, a1, a2, a3);
      mma_16816(sc, a0, a1, a2, a3, bq[ks][0], bq[ks][1]);
    }
    const int key0 = (page_begin + i) * kPage + g;
    const int key1 = key0 + 8;
    const float s0 = key0 < Li ? sc[0] * kScale : -CUDART_INF_F;
    const float s1 = key0 < Li ? sc[1] * kScale : -CUDART_INF_F;
    const float s2 = key1 < Li ? sc[2] * kScale : -CUDART_INF_F;
    const float s3 = key1 < Li ? sc[3] * kScale : -CUDART_INF_F;
    const float mx0 = shfl_max_group(fmaxf(s0, s2));
    const float mx1 = shfl_max_group(fmaxf(s1, s3));
    const float mn0 = fmaxf(m0, mx0);
    const float mn1 = fmaxf(m1, mx1);
    // every visited page holds at least one visible key, so mn* is finite
    const float al0 = ex2((m0 - mn0) * kLog2e);
    const float al1 = ex2((m1 - mn1) * kLog2e);
    const float p0 = ex2((s0 - mn0) * kLog2e);
    const float p1 = ex2((s1 - mn1) * kLog2e);
    const float p2 = ex2((s2 - mn0) * kLog2e);
    const float p3 = ex2((s3 - mn1) * kLog2e);
    l0 = l0 * al0 + (p0 + p2);
    l1 = l1 * al1 + (p1 + p3);
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      acc[mt][0] *= al0;
      acc[mt][1] *= al1;
      acc[mt][2] *= al0;
      acc[mt][3] *= al1;
    }
    const uint32_t pb0 = movmatrix_trans(pack_half2(p0, p1));
    const uint32_t pb1 = movmatrix_trans(pack_half2(p2, p3));

    // Rows past the sequence end hold stale pool data; zero them so that
    // 0 * (non-finite) cannot reach the accumulator (the reference loads
    // them masked with other=0).
    const int valid_rows = Li - (page_begin + i) * kPage;
    if (valid_rows < kPage) {
      for (int e = lane; e < (kPage - valid_rows) * 8; e += 32) {
        const int r = valid_rows + (e >> 3);
        const uint32_t addr = vt + sw128(r, e & 7);
        asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
      }
      __syncwarp();
    }

    // O^T (64 dims x 8 heads) += V^T (64 x 16 keys) . P^T (16 x 8)
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      uint32_t a0, a1, a2, a3;
      const int key = (lane & 7) + ((lane >> 4) << 3);
      ldmatrix_x4_trans(vt + sw128(key, mt * 2 + ((lane >> 3) & 1)), a0, a1, a2, a3);
      mma_16816(acc[mt], a0, a1, a2, a3, pb0, pb1);
    }
    if (valid_rows < kPage) fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8u * s);
  }

  l0 = shfl_sum_group(l0);
  l1 = shfl_sum_group(l1);

  // ---- merge the two page-parity warps of kv head h -------------------------
  float* sc_h = scratch + h * C::kScratchFloats;  // m[8] | l[8] | acc[64][8]
  if (par == 1) {
    if (g == 0) {
      sc_h[2 * t4] = m0;
      sc_h[2 * t4 + 1] = m1;
      sc_h[8 + 2 * t4] = l0;
      sc_h[8 + 2 * t4 + 1] = l1;
    }
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      const int d0 = mt * 16 + g;
      sc_h[16 + d0 * 8 + 2 * t4] = acc[mt][0];
      sc_h[16 + d0 * 8 + 2 * t4 + 1] = acc[mt][1];
      sc_h[16 + (d0 + 8) * 8 + 2 * t4] = acc[mt][2];
      sc_h[16 + (d0 + 8) * 8 + 2 * t4 + 1] = acc[mt][3];
    }
  }
  // named barrier per kv head: its two consumer warps (64 threads)
  asm volatile("bar.sync %0, 64;" ::"r"(1 + h) : "memory");
  if (par == 1) return;

  {
    const float mb0 = sc_h[2 * t4], mb1 = sc_h[2 * t4 + 1];
    const float lb0 = sc_h[8 + 2 * t4], lb1 = sc_h[8 + 2 * t4 + 1];
    const float M0 = fmaxf(m0, mb0), M1 = fmaxf(m1, mb1);
    const float wa0 = M0 == -CUDART_INF_F ? 0.f : ex2((m0 - M0) * kLog2e);
    const float wb0 = M0 == -CUDART_INF_F ? 0.f : ex2((mb0 - M0) * kLog2e);
    const float wa1 = M1 == -CUDART_INF_F ? 0.f : ex2((m1 - M1) * kLog2e);
    const float wb1 = M1 == -CUDART_INF_F ? 0.f : ex2((mb1 - M1) * kLog2e);
    l0 = l0 * wa0 + lb0 * wb0;
    l1 = l1 * wa1 + lb1 * wb1;
    m0 = M0;
    m1 = M1;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      const int d0 = mt * 16 + g;
      acc[mt][0] = acc[mt][0] * wa0 + sc_h[16 + d0 * 8 + 2 * t4] * wb0;
      acc[mt][1] = acc[mt][1] * wa1 + sc_h[16 + d0 * 8 + 2 * t4 + 1] * wb1;
      acc[mt][2] = acc[mt][2] * wa0 + sc_h[16 + (d0 + 8) * 8 + 2 * t4] * wb0;
      acc[mt][3] = acc[mt][3] * wa1 + sc_h[16 + (d0 + 8) * 8 + 2 * t4 + 1] * wb1;
    }
  }
  __syncwarp();

  const int hq0 = h * kGroup + 2 * t4;  // global q head of acc[.][0] / acc[.][2]
  if (S == 1) {
    // final output: acc / l; a row that saw no key (L == 0) is zero
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
    const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
    // stage fp16 rows in the (now free) scratch area, then write 16-byte chunks
    __half* stage = reinterpret_cast<__half*>(sc_h);  // [7][64]
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      const int d0 = mt * 16 + g;
      if (2 * t4 < kGroup) {
        stage[(2 * t4) * kD + d0] = __float2half_rn(acc[mt][0] * inv0);
        stage[(2 * t4) * kD + d0 + 8] = __float2half_rn(acc[mt][2] * inv0);
      }
      if (2 * t4 + 1 < kGroup) {
        stage[(2 * t4 + 1) * kD + d0] = __float2half_rn(acc[mt][1] * inv1);
        stage[(2 * t4 + 1) * kD + d0 + 8] = __float2half_rn(acc[mt][3] * inv1);
      }
    }
    __syncwarp();
    const uint4* src = reinterpret_cast<const uint4*>(stage);
    uint4* dst = reinterpret_cast<uint4*>(p.o + (static_cast<int64_t>(b) * H_Q + h * kGroup) * kD);
    for (int e = lane; e < kGroup * kD / 8; e += 32) dst[e] = src[e];
  } else if (n > 0) {  // the merge reads only splits that saw pages
    const int64_t base = (static_cast<int64_t>(b) * S + split) * H_Q;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int hq = hq0 + hh;
      if (2 * t4 + hh >= kGroup) continue;
      float* a = p.ws_acc + (base + hq) * kD;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        a[mt * 16 + g] = acc[mt][hh];
        a[mt * 16 + g + 8] = acc[mt][2 + hh];
      }
      if (g == 0) {
        p.ws_ml[(base + hq) * 2 + 0] = hh ? m1 : m0;
        p.ws_ml[(base + hq) * 2 + 1] = hh ? l1 : l0;
      }
    }
  }
}

// Combines the split partials of one (query head, sequence):
// O = sum_s w_s acc_s / sum_s w_s l_s, w_s = exp(m_s - max m), over the splits
// that saw pages; a sequence with no key at all gets a zero row (reference
// merge, kernels/decode_attention.py:243-264). 8 warps each fold every 8th
// split (lane = two output columns), then warp 0 folds the 8 warp results.
// Launched with programmatic stream serialization: griddepcontrol.wait holds
// it until the split kernel has finished and its writes are visible (the
// sequence's page count, from inputs the split kernel does not write, is read
// before).
__global__ void __launch_bounds__(256)
    decode_merge_kernel(const float* __restrict__ ws_acc, const float* __restrict__ ws_ml,
                        __half* __restrict__ o, const int64_t* __restrict__ lens,
                        const int64_t* __restrict__ slot_ids, int64_t n_slots,
                        int64_t bt_stride, int num_splits, int num_q_heads, int lens_per_slot) {
  __shared__ float s_m[8], s_l[8];
  __shared__ float2 s_acc[8][32];
  const int hq = blockIdx.x;
  const int b = blockIdx.y;
  const int S = num_splits;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // the split kernel does not write lengths or slots: read them while it runs
  const int np = seq_pages(lens, slot_ids, b, n_slots, bt_stride, lens_per_slot);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int pps = split_pages(np, S);
  const int active = np == 0 ? 0 : (np + pps - 1) / pps;

  float M = -CUDART_INF_F, l = 0.f;
  float2 acc = make_float2(0.f, 0.f);
  for (int s = warp; s < active; s += 8) {
    const int64_t r = (static_cast<int64_t>(b) * S + s) * num_q_heads + hq;
    const float m = ws_ml[r * 2];   // finite: every active split saw a key
    const float ls = ws_ml[r * 2 + 1];
    const float2 a = *reinterpret_cast<const float2*>(ws_acc + r * kD + 2 * lane);
    const float Mn = fmaxf(M, m);
    const float wo = ex2((M - Mn) * kLog2e);
    const float wn = ex2((m - Mn) * kLog2e);
    l = l * wo + ls * wn;
    acc.x = acc.x * wo + a.x * wn;
    acc.y = acc.y * wo + a.y * wn;
    M = Mn;
  }
  if (lane == 0) {
    s_m[warp] = M;
    s_l[warp] = l;
  }
  s_acc[warp][lane] = acc;
  __syncthreads();
  if (warp != 0) return;
  float Mt = -CUDART_INF_F;
#pragma unroll
  for (int w = 0; w < 8; ++w) Mt = fmaxf(Mt, s_m[w]);
  float den = 0.f;
  float2 num = make_float2(0.f, 0.f);
  if (Mt != -CUDART_INF_F) {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float wt = s_m[w] == -CUDART_INF_F ? 0.f : ex2((s_m[w] - Mt) * kLog2e);
      den += wt * s_l[w];
      num.x += wt * s_acc[w][lane].x;
      num.y += wt * s_acc[w][lane].y;
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  *reinterpret_cast<__half2*>(o + (static_cast<int64_t>(b) * num_q_heads + hq) * kD + 2 * lane) =
      __floats2half2_rn(num.x * inv, num.y * inv);
}

// Split counts up to this use decode_merge_small_kernel.
constexpr int kSmallMergeSplits = 8;

// The same combination for S <= kSmallMergeSplits with one CTA per sequence and
// one warp per query head (lane = two output columns): the warp reads the
// sequence's active partials at once and folds them in split order. This is
// the arithmetic and order of decode_merge_kernel for such S (there each split
// sits in a warp of its own and warp 0 folds them in warp order); the grid is
// B CTAs instead of H_q x B CTAs of 8 warps, most of which have nothing to
// fold when S is small.
__global__ void __launch_bounds__(1024)
    decode_merge_small_kernel(const float* __restrict__ ws_acc, const float* __restrict__ ws_ml,
                              __half* __restrict__ o, const int64_t* __restrict__ lens,
                              const int64_t* __restrict__ slot_ids, int64_t n_slots,
                              int64_t bt_stride, int num_splits, int num_q_heads,
                              int lens_per_slot) {
  const int hq = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  const int S = num_splits;
  // the split kernel does not write lengths or slots: read them while it runs
  const int np = seq_pages(lens, slot_ids, b, n_slots, bt_stride, lens_per_slot);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int pps = split_pages(np, S);
  const int active = np == 0 ? 0 : (np + pps - 1) / pps;

  float m[kSmallMergeSplits], ls[kSmallMergeSplits];
  float2 a[kSmallMergeSplits];
#pragma unroll
  for (int s = 0; s < kSmallMergeSplits; ++s) {
    if (s < active) {
      const int64_t r = (static_cast<int64_t>(b) * S + s) * num_q_heads + hq;
      m[s] = ws_ml[r * 2];   // finite: every active split saw a key
      ls[s] = ws_ml[r * 2 + 1];
      a[s] = *reinterpret_cast<const float2*>(ws_acc + r * kD + 2 * lane);
    } else {
      m[s] = -CUDART_INF_F;
      ls[s] = 0.f;
      a[s] = make_float2(0.f, 0.f);
    }
  }
  float Mt = -CUDART_INF_F;
#pragma unroll
  for (int s = 0; s < kSmallMergeSplits; ++s) Mt = fmaxf(Mt, m[s]);
  float den = 0.f;
  float2 num = make_float2(0.f, 0.f);
  if (Mt != -CUDART_INF_F) {
#pragma unroll
    for (int s = 0; s < kSmallMergeSplits; ++s) {
      const float wt = m[s] == -CUDART_INF_F ? 0.f : ex2((m[s] - Mt) * kLog2e);
      den += wt * ls[s];
      num.x += wt * a[s].x;
      num.y += wt * a[s].y;
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  *reinterpret_cast<__half2*>(o + (static_cast<int64_t>(b) * num_q_heads + hq) * kD + 2 * lane) =
      __floats2half2_rn(num.x * inv, num.y * inv);
}

// Arguments of the fused rotary embedding + KV write (see Params).
struct FusedRope {
  const void* qkv;
  int64_t qkv_tok;
  const void* cos;
  const void* sin;
  int64_t cs_tok;
};

template <int HKV>
int launch(const void* q, const void* k, const void* v, const int64_t* lens,
           const int64_t* slot_ids, BlockTable block_table, void* o, float* ws, int batch,
           int64_t n_pages, int64_t n_slots, int64_t bt_stride, int64_t page_stride,
           int64_t head_stride, int S, cudaStream_t stream, const FusedRope* rope = nullptr) {
  using C = Cfg<HKV>;
  CUtensorMap tm_k, tm_v;
  const uint64_t dims[4] = {kD, kPage, HKV, static_cast<uint64_t>(n_pages)};
  const uint64_t strides[3] = {kD * 2, static_cast<uint64_t>(head_stride) * 2,
                               static_cast<uint64_t>(page_stride) * 2};
  const uint32_t box[4] = {kD, kPage, HKV, 1};
  int st = encode_tensor_map(&tm_k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(k), dims,
                             strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != CIE_OK) return st;
  st = encode_tensor_map(&tm_v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(v), dims,
                         strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != CIE_OK) return st;
  st = ensure_smem_attribute(reinterpret_cast<const void*>(&decode_split_kernel<HKV>), C::kSmemBytes,
                             HKV);
  if (st != CIE_OK) return st;

  Params p;
  p.q = static_cast<const __half*>(q);
  p.lens = lens;
  p.slot_ids = slot_ids;
  p.block_table = block_table;
  p.o = static_cast<__half*>(o);
  const int H_Q = HKV * kGroup;
  p.ws_acc = ws;
  p.ws_ml = ws == nullptr ? nullptr : ws + static_cast<int64_t>(batch) * S * H_Q * kD;
  p.batch = batch;
  p.num_splits = S;
  p.n_pages = n_pages;
  p.n_slots = n_slots;
  p.bt_stride = bt_stride;
  p.qkv = nullptr;
  p.qkv_tok = 0;
  p.cos = p.sin = nullptr;
  p.cs_tok = 0;
  p.k_cache = p.v_cache = nullptr;
  p.page_stride = page_stride;
  p.head_stride = head_stride;
  if (rope != nullptr) {
    p.qkv = static_cast<const __half*>(rope->qkv);
    p.qkv_tok = rope->qkv_tok;
    p.cos = static_cast<const __half*>(rope->cos);
    p.sin = static_cast<const __half*>(rope->sin);
    p.cs_tok = rope->cs_tok;
    p.k_cache = static_cast<__half*>(const_cast<void*>(k));
    p.v_cache = static_cast<__half*>(const_cast<void*>(v));
  }
  // a programmatic dependent of the previous kernel in the stream: scheduled
  // as that kernel drains, it waits (griddepcontrol.wait) before reading inputs
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t scfg = {};
  scfg.gridDim = dim3(S, batch);
  scfg.blockDim = dim3(C::kThreads);
  scfg.dynamicSmemBytes = C::kSmemBytes;
  scfg.stream = stream;
  scfg.attrs = pdl;
  scfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&scfg, decode_split_kernel<HKV>, tm_k, tm_v, p);
  if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
  if (S > 1) {
    const bool small = S <= kSmallMergeSplits;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = small ? dim3(batch) : dim3(H_Q, batch);
    cfg.blockDim = dim3(small ? 32 * H_Q : 256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, small ? decode_merge_small_kernel : decode_merge_kernel,
                           static_cast<const float*>(p.ws_acc),
                           static_cast<const float*>(p.ws_ml), p.o, lens, slot_ids, n_slots,
                           bt_stride, S, H_Q, rope != nullptr ? 1 : 0);
    if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "merge launch: %s", cudaGetErrorString(e));
  }
  return CIE_OK;
}

}  // namespace decode
}  // namespace cie

extern "C" {

int cie_decode_default_splits(int batch, int device) {
  int sms = 148;
  if (device >= 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && n > 0)
      sms = n;
  }
  if (batch <= 0) return 1;
  // two resident CTAs per SM; one wave of (split, sequence) CTAs, at most 64
  // splits: past that the merge of the partials costs more than the extra
  // parallelism gives (B = 1 x 16384: 12.1 us at 64 splits, 16.0 us at 256).
  // A count less than 5/4 of a power of two is rounded down to it: 37 -> 32,
  // 18 -> 16 and 9 -> 8 splits were 1-7 % faster at kv_len 2048-32768 on
  // B200, while rounding 3, 6, 12 or 24 down to 2, 4, 8 or 16 was slower.
  int s = (2 * sms) / batch;
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  int p2 = 1;
  while (p2 * 2 <= s) p2 *= 2;
  if (4 * s < 5 * p2) s = p2;
  return s;
}

size_t cie_decode_workspace_bytes(int batch, int num_q_heads, int head_dim, int num_splits) {
  if (batch <= 0 || num_splits <= 1 || num_q_heads <= 0 || head_dim <= 0) return 0;
  const size_t rows = static_cast<size_t>(batch) * num_splits * num_q_heads;
  return rows * (static_cast<size_t>(head_dim) + 2) * sizeof(float);
}

}  // extern "C"

namespace cie {
namespace decode {

// Argument checks shared by every decode entry point (everything but the
// workspace); q is null exactly when `rope` is given. On success *splits is
// the split count the call will use (0 when batch == 0: nothing to do).
int check_args(const void* q, const void* k, const void* v, const int64_t* lens,
               const int64_t* slot_ids, const void* block_table, const void* o, int batch,
               int num_q_heads, int num_kv_heads, int head_dim, int page_size, int64_t n_pages,
               int64_t n_slots, int64_t bt_stride, int64_t kv_page_stride,
               int64_t kv_head_stride, int num_splits, const FusedRope* rope, int* splits) {
  *splits = 0;
  if (batch < 0) return fail(CIE_ERR_INVALID_ARGUMENT, "batch < 0");
  if (batch == 0) return CIE_OK;
  if ((!q && !rope) || !k || !v || !lens || !slot_ids || !block_table || !o)
    return fail(CIE_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (head_dim != kD || page_size != kPage)
    return fail(CIE_ERR_UNSUPPORTED, "head_dim %d / page_size %d (supported: 64 / 16)", head_dim,
                page_size);
  if (num_kv_heads != 1 && num_kv_heads != 2 && num_kv_heads != 4)
    return fail(CIE_ERR_UNSUPPORTED, "num_kv_heads %d (supported: 1, 2, 4)", num_kv_heads);
  if (num_q_heads != num_kv_heads * kGroup)
    return fail(CIE_ERR_UNSUPPORTED, "num_q_heads %d must be 7 * num_kv_heads", num_q_heads);
  if (n_pages < 1 || n_slots < 1 || bt_stride < 1)
    return fail(CIE_ERR_INVALID_ARGUMENT, "n_pages / n_slots / bt_stride must be >= 1");
  if (n_pages >= (int64_t(1) << 31))
    return fail(CIE_ERR_OVERFLOW, "n_pages %lld does not fit int32", (long long)n_pages);
  if (batch > 65535) return fail(CIE_ERR_UNSUPPORTED, "batch %d > 65535", batch);
  if (kv_head_stride < page_size * head_dim || kv_page_stride < kv_head_stride * num_kv_heads)
    return fail(CIE_ERR_INVALID_ARGUMENT, "overlapping K/V strides (page %lld, head %lld)",
                (long long)kv_page_stride, (long long)kv_head_stride);
  if ((kv_page_stride % 8) || (kv_head_stride % 8) || !aligned16(k) || !aligned16(v) ||
      (q && !aligned16(q)) || !aligned16(o))
    return fail(CIE_ERR_ALIGNMENT, "q/o/k/v must be 16-byte aligned with 16-byte strides");
  if (rope) {
    if (!rope->qkv || !rope->cos || !rope->sin)
      return fail(CIE_ERR_INVALID_ARGUMENT, "null qkv / cos / sin");
    if (rope->qkv_tok < static_cast<int64_t>(num_q_heads + 2 * num_kv_heads) * head_dim ||
        rope->cs_tok < head_dim)
      return fail(CIE_ERR_INVALID_ARGUMENT, "qkv / cos / sin rows overlap");
    if ((rope->qkv_tok % 8) || (rope->cs_tok % 8) || !aligned16(rope->qkv) ||
        !aligned16(rope->cos) || !aligned16(rope->sin))
      return fail(CIE_ERR_ALIGNMENT, "qkv / cos / sin rows must start on 16-byte boundaries");
  }
  const int S = num_splits > 0 ? num_splits : cie_decode_default_splits(batch, current_device());
  if (S > 4096) return fail(CIE_ERR_INVALID_ARGUMENT, "num_splits %d > 4096", S);
  *splits = S;
  return CIE_OK;
}

// Argument checks and dispatch of the decode entry points.
int entry(const void* q, const void* k, const void* v, const int64_t* lens,
          const int64_t* slot_ids, BlockTable block_table, void* o, void* workspace,
          size_t workspace_bytes, int batch, int num_q_heads, int num_kv_heads, int head_dim,
          int page_size, int64_t n_pages, int64_t n_slots, int64_t bt_stride,
          int64_t kv_page_stride, int64_t kv_head_stride, int num_splits, cie_stream_t stream,
          const FusedRope* rope) {
  int S = 0;
  const int st = check_args(q, k, v, lens, slot_ids, block_table.ptr, o, batch, num_q_heads,
                            num_kv_heads, head_dim, page_size, n_pages, n_slots, bt_stride,
                            kv_page_stride, kv_head_stride, num_splits, rope, &S);
  if (st != CIE_OK || S == 0) return st;
  float* ws = nullptr;
  if (S > 1) {
    const size_t need = cie_decode_workspace_bytes(batch, num_q_heads, head_dim, S);
    if (workspace == nullptr || workspace_bytes < need)
      return fail(CIE_ERR_WORKSPACE, "split path needs %zu workspace bytes, got %zu", need,
                  workspace == nullptr ? size_t(0) : workspace_bytes);
    if (!aligned16(workspace)) return fail(CIE_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
    ws = static_cast<float*>(workspace);
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (num_kv_heads) {
    case 1:
      return launch<1>(q, k, v, lens, slot_ids, block_table, o, ws, batch, n_pages, n_slots,
                       bt_stride, kv_page_stride, kv_head_stride, S, s, rope);
    case 2:
      return launch<2>(q, k, v, lens, slot_ids, block_table, o, ws, batch, n_pages, n_slots,
                       bt_stride, kv_page_stride, kv_head_stride, S, s, rope);
    default:
      return launch<4>(q, k, v, lens, slot_ids, block_table, o, ws, batch, n_pages, n_slots,
                       bt_stride, kv_page_stride, kv_head_stride, S, s, rope);
  }
}

}  // namespace decode
}  // namespace cie

extern "C" {

int cie_decode_attention(const void* q, const void* k, const void* v, const int64_t* lens,
                         const int64_t* slot_ids, const int64_t* block_table, void* o,
                         void* workspace, size_t workspace_bytes, int batch, int num_q_heads,
                         int num_kv_heads, int head_dim, int page_size, int64_t n_pages,
                         int64_t n_slots, int64_t bt_stride, int64_t kv_page_stride,
                         int64_t kv_head_stride, int num_splits, cie_stream_t stream) {
  return cie::decode::entry(q, k, v, lens, slot_ids, cie::BlockTable{block_table, 1}, o,
                            workspace, workspace_bytes, batch, num_q_heads, num_kv_heads,
                            head_dim, page_size, n_pages, n_slots, bt_stride, kv_page_stride,
                            kv_head_stride, num_splits, stream, nullptr);
}

int cie_decode_attention_bt32(const void* q, const void* k, const void* v, const int64_t* lens,
                              const int64_t* slot_ids, const int32_t* block_table, void* o,
                              void* workspace, size_t workspace_bytes, int batch, int num_q_heads,
                              int num_kv_heads, int head_dim, int page_size, int64_t n_pages,
                              int64_t n_slots, int64_t bt_stride, int64_t kv_page_stride,
                              int64_t kv_head_stride, int num_splits, cie_stream_t stream) {
  return cie::decode::entry(q, k, v, lens, slot_ids, cie::BlockTable{block_table, 0}, o,
                            workspace, workspace_bytes, batch, num_q_heads, num_kv_heads,
                            head_dim, page_size, n_pages, n_slots, bt_stride, kv_page_stride,
                            kv_head_stride, num_splits, stream, nullptr);
}

static int rope_kv_decode_attention(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                                    const void* sin, int64_t cs_tok_stride, void* k_cache,
                                    void* v_cache, const int64_t* lens, const int64_t* slot_ids,
                                    cie::BlockTable block_table, void* o, void* workspace,
                                    size_t workspace_bytes, int batch, int num_q_heads,
                                    int num_kv_heads, int head_dim, int page_size, int64_t n_pages,
                                    int64_t n_slots, int64_t bt_stride, int64_t cache_page_stride,
                                    int64_t cache_head_stride, int num_splits,
                                    cie_stream_t stream) {
  const cie::decode::FusedRope rope{qkv, qkv_tok_stride, cos, sin, cs_tok_stride};
  return cie::decode::entry(nullptr, k_cache, v_cache, lens, slot_ids, block_table, o, workspace,
                            workspace_bytes, batch, num_q_heads, num_kv_heads, head_dim,
                            page_size, n_pages, n_slots, bt_stride, cache_page_stride,
                            cache_head_stride, num_splits, stream, &rope);
}

int cie_rope_kv_decode_attention(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                                 const void* sin, int64_t cs_tok_stride, void* k_cache,
                                 void* v_cache, const int64_t* lens, const int64_t* slot_ids,
                                 const int64_t* block_table, void* o, void* workspace,
                                 size_t workspace_bytes, int batch, int num_q_heads,
                                 int num_kv_heads, int head_dim, int page_size, int64_t n_pages,
                                 int64_t n_slots, int64_t bt_stride, int64_t cache_page_stride,
                                 int64_t cache_head_stride, int num_splits, cie_stream_t stream) {
  return rope_kv_decode_attention(qkv, qkv_tok_stride, cos, sin, cs_tok_stride, k_cache, v_cache,
                                  lens, slot_ids, cie::BlockTable{block_table, 1}, o, workspace,
                                  workspace_bytes, batch, num_q_heads, num_kv_heads, head_dim,
                                  page_size, n_pages, n_slots, bt_stride, cache_page_stride,
                                  cache_head_stride, num_splits, stream);
}

int cie_rope_kv_decode_attention_bt32(
    const void* qkv, int64_t qkv_tok_stride, const void* cos, const void* sin,
    int64_t cs_tok_stride, void* k_cache, void* v_cache, const int64_t* lens,
    const int64_t* slot_ids, const int32_t* block_table, void* o, void* workspace,
    size_t workspace_bytes, int batch, int num_q_heads, int num_kv_heads, int head_dim,
    int page_size, int64_t n_pages, int64_t n_slots, int64_t bt_stride, int64_t cache_page_stride,
    int64_t cache_head_stride, int num_splits, cie_stream_t stream) {
  return rope_kv_decode_attention(qkv, qkv_tok_stride, cos, sin, cs_tok_stride, k_cache, v_cache,
                                  lens, slot_ids, cie::BlockTable{block_table, 0}, o, workspace,
                                  workspace_bytes, batch, num_q_heads, num_kv_heads, head_dim,
                                  page_size, n_pages, n_slots, bt_stride, cache_page_stride,
                                  cache_head_stride, num_splits, stream);
}

}  // extern "C"
