// Varlen mixed attention (chunked prefill + decode rows) on 5th-generation
// tensor cores (tcgen05 + TMEM) for sm_100a.
//
// Replaces mixed_gqa_attention_kernel (kernels/prefill_attention.py:10-198)
// behind the host contract of attn/core.py:69-111.
//
// Work unit: one CTA = TWO consecutive query tiles (A, B) of one
// (sequence, kv head) x one contiguous range of 128-key blocks. A tile is 18
// tokens x the 7 query heads that share the kv head = 126 rows of the
// tcgen05 M = 128 tile (the reference pads 7 heads to 8 and uses 16 tokens,
// 112 useful rows of 128); it is one TMA box over q viewed as
// (token, kv head, head-in-group, dim), row r = token * 7 + head. Both tiles
// consume the same K/V blocks, loaded once. When a tile pair's keys are split
// over several CTAs, each writes an fp32 partial (m, l, unnormalised O) per
// row and a merge kernel combines them; a pair that is not split writes O.
//
// Tensor memory (512 columns) per tile x: S = Q K^T at 256x (128 fp32
// columns), P at 256x + 128 (128 fp16 keys packed two per column) and the
// O accumulator at 256x + 192 (64 columns). P never touches shared memory:
// the softmax writes it with tcgen05.st and O += P V reads it as the
// TMEM-resident A operand, with V from shared memory.
//
// Warp roles (384 threads, three warpgroups):
//   warp 0       TMA producer: both Q tiles, then per key block the 8 K and
//                8 V pages of this kv head (2 KiB boxes through the block
//                table) into a 5-stage ring.
//   warps 1, 2   MMA issuers of tile A and tile B (the whole warp runs the
//                loop, one elected lane issues; warp 1 also owns TMEM):
//                S_x(j) = Q_x K_j^T as soon as K_j is in and
//                tile x's softmax has read S_x(j-1), then O_x += P_x(j-1)
//                V_{j-1} once P_x(j-1) is published. S_x(j+1) is computed while
//                the softmax of tile x still works on block j, and neither
//                tile's MMAs wait behind the other's issue.
//   warp 3       idle: warpgroup 0 hands most of its registers to the softmax
//                warpgroups (setmaxnreg).
//   warps 4-7    softmax of tile A, warps 8-11 of tile B, one thread per row
//                (warp w owns TMEM lanes [32 (w % 4), +32)). Per block: the
//                row maximum first, then the exponentials into registers
//                (the two tiles take turns at this phase, block by block);
//                only then the wait for the previous P V (which must have
//                consumed P and updated O). The reference max moves only
//                when the block maximum exceeds it by more than 2^8 (then O
//                and l are rescaled): P stays <= 256, exact in fp16, and O / l
//                is the reference's softmax (acc * alpha + dot(P, V),
//                kernels/prefill_attention.py:157-184) up to rounding. Warps
//                whose 32 rows are all padding (short chunks, decode rows) do
//                nothing; barrier arrival counts cover the working warps only.
// CTAs run most-expensive first: blockIdx.y walks the tile pairs from the
// last (most keys) to the first.
// All waits are bounded; on a timeout the kernel records
// CIE_DEVERR_WAIT_TIMEOUT, drains its own copies and MMAs, frees TMEM and
// returns. tcgen05.ld / st / wait are warp-collective, so every decision that
// guards one is warp-uniform.
#include <math_constants.h>

#include "cie_common.cuh"
#include "cie_host.h"

namespace cie {
namespace mixed {

constexpr int kD = 64;
constexpr int kPage = 16;
constexpr int kGroup = 7;
constexpr int kTileTokens = 18;
constexpr int kPairTokens = 2 * kTileTokens;
constexpr int kRows = kTileTokens * kGroup;  // 126 useful rows of M = 128
constexpr int kM = 128;
constexpr int kBlockKeys = 128;
constexpr int kPagesPerBlock = kBlockKeys / kPage;  // 8
constexpr int kStages = 5;
constexpr int kMinBlocksPerSplit = 2;
constexpr int kMaxSplits = 16;      // num_splits >= 1: key ranges per tile pair at most
constexpr int kMaxPieces = 16;      // automatic plan: key ranges per tile pair at most
// Automatic plan: pieces of at most 1 / slots of the work, slots = 3/2 x SMs
// (1, 5/4 and 2 x SMs measured: level, level and 8 % slower on 512-token
// chunks; 3/2 is 2 % faster there and level on config 3).
constexpr int kSlotsNum = 3;
constexpr int kSlotsDen = 2;
__host__ __device__ constexpr long long plan_slots(long long n_sm) {
  return (n_sm * kSlotsNum + kSlotsDen - 1) / kSlotsDen;
}
constexpr int kPlanThreads = 1024;  // the planning kernel is one CTA
constexpr int kPlanMaxBatch = 2048;
constexpr int kSizeBuckets = kPlanThreads;  // pieces ordered by key blocks, largest first
constexpr int kTileThreads = 128;                   // softmax threads per tile, one per row
constexpr int kThreads = 128 + 2 * kTileThreads;    // warpgroup 0 + one per tile
// Register split after launch (launch: 384 x 168): warpgroup 0 drops to 56,
// the softmax warpgroups rise to 224 (128 x 56 + 256 x 224 = 384 x 168).
constexpr uint32_t kCtrlRegs = 56;
constexpr uint32_t kSoftmaxRegs = 224;
constexpr float kRescaleLog2 = 8.f;                 // move the max when it grows by > 2^8

constexpr int kQBytes = kM * kD * 2;               // 16 KiB
constexpr int kQLoadBytes = kRows * kD * 2;        // 16128 bytes delivered by one box
constexpr int kKVTileBytes = kBlockKeys * kD * 2;  // 16 KiB per K or V block
constexpr int kStageBytes = 2 * kKVTileBytes;
constexpr int kPageBoxBytes = kPage * kD * 2;      // 2 KiB

constexpr int kOffQ = 0;                                   // Q_A, Q_B
constexpr int kOffKV = kOffQ + 2 * kQBytes;
constexpr int kOffBar = kOffKV + kStages * kStageBytes;
// barriers: kv_full[5], kv_empty[5], q_full, mma_done[2], then per tile:
// s_full, s_free, p_full, pv_done, turn
constexpr int kTileBars = 5;
constexpr int kNumBars = 2 * kStages + 3 + 2 * kTileBars;
constexpr int kOffTmemPtr = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = 1024 + kOffTmemPtr + 16;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;
constexpr uint32_t kColP = 128;
constexpr uint32_t kColO = 192;

constexpr uint32_t kIdescS = idesc_f16_f32(kM, kBlockKeys, false);
constexpr uint32_t kIdescPV = idesc_f16_f32(kM, kD, true);

// Partial record of one piece of a tile pair: per row, the unnormalised O[64],
// m (log2 units: max of score * scale * log2(e)) and l, stored column-major as
// [kPartCols][kRecRows] float2 -- column cc < kD / 2 holds (O[2cc], O[2cc+1]),
// column kD / 2 holds (m, l). Tile x's row r sits at x * kM + r, so a warp's
// 32 rows of one column are 256 contiguous, aligned bytes for both the
// writing and the merging CTA.
constexpr int kPartCols = kD / 2 + 1;
constexpr int kPartFloats = 2 * kPartCols;
constexpr int kRecRows = 2 * kM;

// The work plan, in the caller's workspace. A work item is one CTA: a tile
// pair of one (sequence, kv head) and a contiguous range of its key blocks.
// Items are stored largest range first, two int4 each:
//   {b, pair | kv_head << 16, first block, blocks}, {record, split, piece, pieces}.
// A pair cut into `pieces` ranges owns records [record, record + pieces) and
// the counter counters[split]; its last piece to finish merges the others.
struct Plan {
  int* header;         // [0] items
  int4* items;
  unsigned* counters;  // per split pair: pieces finished
  float* records;      // [record][kPartCols][kRecRows] float2
  int max_items, max_split, max_rec;
};

struct Params {
  const int64_t* cu_seqlens;
  const int64_t* kv_lens;
  const int64_t* slot_ids;
  BlockTable block_table;
  __half* o;
  Plan plan;
  int64_t total_tokens;
  int64_t max_seqlen;
  int64_t n_pages;
  int64_t n_slots;
  int64_t bt_stride;
  int batch;
  int num_q_heads;
  int num_kv_heads;
  int num_splits;  // <= 0: automatic plan
  int n_sm;
};

struct Bars {
  uint32_t base;
  __device__ uint32_t kv_full(int s) const { return base + 8u * s; }
  __device__ uint32_t kv_empty(int s) const { return base + 8u * (kStages + s); }
  __device__ uint32_t q_full() const { return base + 8u * (2 * kStages); }
  __device__ uint32_t mma_done(int x) const { return base + 8u * (2 * kStages + 1 + x); }
  __device__ uint32_t tile(int x, int i) const {
    return base + 8u * (2 * kStages + 3 + x * kTileBars + i);
  }
  __device__ uint32_t s_full(int x) const { return tile(x, 0); }
  __device__ uint32_t s_free(int x) const { return tile(x, 1); }
  __device__ uint32_t p_full(int x) const { return tile(x, 2); }
  __device__ uint32_t pv_done(int x) const { return tile(x, 3); }
  // tile x may start the maximum and exponentials of its next block
  __device__ uint32_t turn(int x) const { return tile(x, 4); }
};

// 32 lanes x N consecutive 32-bit TMEM columns (load and store).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}


// three-input maximum (one instruction on sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair of values on the FMA pipe, to unload the 16/clk/SM MUFU that
// ex2.approx uses. Cody-Waite split x = n + f with n = rint(x) (adding
// 1.5 * 2^23 rounds to an integer), f in [-0.5, 0.5]; 2^f by a degree-3
// polynomial fitted for minimax relative error on that interval (7.5e-5,
// below half an fp16 ulp); 2^n added into the exponent field. x is clamped at
// -100 (keeps the exponent in range; 2^-100 is 0 in fp16).
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  x.x = fmaxf(x.x, -100.f);
  x.y = fmaxf(x.y, -100.f);
  const float2 t = __fadd2_rn(x, make_float2(12582912.f, 12582912.f));
  const float2 n = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = __fadd2_rn(x, make_float2(-n.x, -n.y));
  float2 q = __ffma2_rn(make_float2(0.05517132f, 0.05517132f), f,
                        make_float2(0.24261054f, 0.24261054f));
  q = __ffma2_rn(q, f, make_float2(0.69326097f, 0.69326097f));
  q = __ffma2_rn(q, f, make_float2(0.9999281f, 0.9999281f));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}
// Of every 8 column pairs (16 columns), the pairs whose bit is set go through
// exp2_fma2 (a quarter of the exponentials), the rest through ex2.approx.
constexpr unsigned kPolyPairs = 0x88u;

// ---- the work decomposition, shared with the merge kernel -------------------

struct SeqInfo {
  int L;       // chunk length
  int kv_len;  // cached keys before the chunk
  bool valid;
};

// Sequence b's chunk; invalid (and, with `report`, a device error) when its
// row range, slot or length is out of bounds.
__device__ __forceinline__ SeqInfo seq_info(const Params& p, int b, bool report) {
  SeqInfo si{0, 0, false};
  // all four loads issued before any of them is tested
  const int64_t start = p.cu_seqlens[b];
  const int64_t end = p.cu_seqlens[b + 1];
  const int64_t slot = p.slot_ids[b];
  int64_t kv_len = p.kv_lens[b];
  if (start < 0 || end < start || end > p.total_tokens) {
    if (report) raise_error(CIE_DEVERR_BAD_SEQLENS);
    return si;
  }
  const int64_t L64 = end - start;
  if (L64 > p.max_seqlen) {
    if (report) raise_error(CIE_DEVERR_BAD_SEQLENS);
    return si;
  }
  if (L64 == 0) return si;
  if (slot < 0 || slot >= p.n_slots) {
    if (report) raise_error(CIE_DEVERR_BAD_SLOT);
    return si;
  }
  if (kv_len < 0) kv_len = 0;
  if ((kv_len + L64 + kPage - 1) / kPage > p.bt_stride) {
    if (report) raise_error(CIE_DEVERR_BAD_LENGTH);
    return si;
  }
  si.L = static_cast<int>(L64);
  si.kv_len = static_cast<int>(kv_len);
  si.valid = true;
  return si;
}

// key blocks the last row of tile pair `pair` needs
__device__ __forceinline__ int pair_blocks(int L, int kv_len, int pair) {
  const int end = min(L, (pair + 1) * kPairTokens);
  return (kv_len + end + kBlockKeys - 1) / kBlockKeys;
}

struct PairInfo {
  int L;            // chunk length of the sequence
  int tok0;         // first token of the pair inside the chunk
  int pair_tokens;  // tokens of the pair (1..36)
  int kv_len;
  int n_blocks;     // key blocks the pair's last row needs
  bool valid;
};

__device__ __forceinline__ PairInfo pair_info(const Params& p, int b, int pair) {
  PairInfo pi{};
  pi.valid = false;
  const SeqInfo si = seq_info(p, b, false);
  if (!si.valid) return pi;
  const int tok0 = pair * kPairTokens;
  if (tok0 >= si.L) return pi;
  pi.L = si.L;
  pi.tok0 = tok0;
  pi.pair_tokens = min(pi.L - tok0, kPairTokens);
  pi.kv_len = si.kv_len;
  pi.n_blocks = pair_blocks(si.L, si.kv_len, pair);
  pi.valid = true;
  return pi;
}

// Exclusive prefix sum over the kPlanThreads threads of a CTA; `total`
// receives the sum. Every thread must call it.
__device__ __forceinline__ int plan_excl_scan(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[w] = x;
  __syncthreads();
  if (w == 0) {
    int t = lane < kPlanThreads / 32 ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    s_warp[lane] = t;
  }
  __syncthreads();
  const int before = (w > 0 ? s_warp[w - 1] : 0) + x - v;
  total = s_warp[kPlanThreads / 32 - 1];
  __syncthreads();
  return before;
}

// The work plan (one CTA). Units are (sequence, tile pair, kv head); a unit of
// nb key blocks becomes k pieces of balanced key ranges: with num_splits >= 1
// k = ceil(nb / max(ceil(nb / num_splits), 2)); automatically, ranges of at
// most C = max(2, ceil(total blocks / plan_slots(SMs))) blocks, k <= kMaxPieces.
// Pieces are written largest first (a counting sort on their block count), so
// the longest CTAs start first and the short ones fill the tail. Sequences
// whose rows, slot or length are out of bounds raise a device error here and
// get no work.
//
// With `rope_ctas` > 0 (cie_rope_kv_mixed_attention) the grid has that many more
// CTAs, which apply the rotary embedding to the pass's q and k rows and write
// k and v to their pages (rope::rope_kv_item, the work of
// cie_rope_kv_mixed_update) while CTA 0 plans; the attention grid waits for the
// whole grid, so it reads the rotated q and the written pages.
__global__ void __launch_bounds__(kPlanThreads)
    mixed_plan_kernel(const Params p, const rope::Args ra, int rope_ctas) {
  __shared__ int s_pfx[kPlanMaxBatch + 1];  // tile pairs before sequence b
  __shared__ int s_len[kPlanMaxBatch];
  __shared__ int s_kv[kPlanMaxBatch];
  __shared__ int s_bkt[kSizeBuckets];
  __shared__ int s_warp[32];
  __shared__ unsigned long long s_blocks;
  __shared__ int s_cnt[3];  // items, split pairs, records
  // the attention grid may be scheduled now; it waits for this grid to finish
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (blockIdx.x > 0) {
    const int64_t n = rope::work_items(ra);
    for (int64_t idx = static_cast<int64_t>(blockIdx.x - 1) * kPlanThreads + threadIdx.x; idx < n;
         idx += static_cast<int64_t>(rope_ctas) * kPlanThreads)
      rope::rope_kv_item(ra, idx);
    return;
  }
  const int tid = threadIdx.x;
  const int B = p.batch;
  const int H = p.num_kv_heads;
  if (tid == 0) {
    s_blocks = 0;
    s_cnt[0] = s_cnt[1] = s_cnt[2] = 0;
  }
  for (int i = tid; i < kSizeBuckets; i += kPlanThreads) s_bkt[i] = 0;
  int carry = 0;
  for (int base = 0; base < B; base += kPlanThreads) {
    const int b = base + tid;
    SeqInfo si{0, 0, false};
    if (b < B) si = seq_info(p, b, true);
    const int P = si.valid ? (si.L + kPairTokens - 1) / kPairTokens : 0;
    int tot;
    const int before = plan_excl_scan(P, s_warp, tot);
    if (b < B) {
      s_pfx[b] = carry + before;
      s_len[b] = si.L;
      s_kv[b] = si.kv_len;
    }
    carry += tot;
  }
  if (tid == 0) s_pfx[B] = carry;
  __syncthreads();
  const int n_units = carry * H;
  // unit g: pair g / H (sequences in order, pairs in order), kv head g % H
  auto unit = [&](int g, int& b, int& pair, int& h) {
    h = g % H;
    const int gp = g / H;
    int lo = 0, hi = B - 1;  // the last b with s_pfx[b] <= gp owns pair gp
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_pfx[mid] <= gp) lo = mid;
      else hi = mid - 1;
    }
    b = lo;
    pair = gp - s_pfx[lo];
    return pair_blocks(s_len[lo], s_kv[lo], pair);
  };
  unsigned long long mine = 0;
  for (int g = tid; g < n_units; g += kPlanThreads) {
    int b, pair, h;
    mine += static_cast<unsigned long long>(unit(g, b, pair, h));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
  if ((tid & 31) == 0 && mine != 0) atomicAdd(&s_blocks, mine);
  __syncthreads();
  const long long total_blocks = static_cast<long long>(s_blocks);
  const long long slots = plan_slots(p.n_sm);
  const long long C = max(static_cast<long long>(kMinBlocksPerSplit), (total_blocks + slots - 1) / slots);
  auto pieces_of = [&](int nb) {
    if (p.num_splits <= 0) return static_cast<int>(min(static_cast<long long>(kMaxPieces), (nb + C - 1) / C));
    const int bps = max((nb + p.num_splits - 1) / p.num_splits, kMinBlocksPerSplit);
    return (nb + bps - 1) / bps;
  };
  auto bucket = [](int blocks) { return min(blocks, kSizeBuckets - 1); };
  for (int g = tid; g < n_units; g += kPlanThreads) {
    int b, pair, h;
    const int nb = unit(g, b, pair, h);
    const int k = pieces_of(nb);
    for (int i = 0; i < k; ++i)
      atomicAdd(&s_bkt[bucket(nb * (i + 1) / k - nb * i / k)], 1);
  }
  __syncthreads();
  {  // bucket cursors: items of larger ranges first
    const int bk = kSizeBuckets - 1 - tid;
    const int c = s_bkt[bk];
    int tot;
    const int before = plan_excl_scan(c, s_warp, tot);
    s_bkt[bk] = before;
    if (tid == 0) s_cnt[0] = tot;
  }
  __syncthreads();
  for (int g = tid; g < n_units; g += kPlanThreads) {
    int b, pair, h;
    const int nb = unit(g, b, pair, h);
    const int k = pieces_of(nb);
    int split = -1, rec = -1;
    bool dead = false;
    if (k > 1) {
      split = atomicAdd(&s_cnt[1], 1);
      rec = atomicAdd(&s_cnt[2], k);
      if (split < p.plan.max_split && rec + k <= p.plan.max_rec) {
        p.plan.counters[split] = 0u;
      } else {  // outside the host's bounds (cannot happen): no work, an error
        raise_error(CIE_DEVERR_BAD_LENGTH);
        dead = true;
      }
    }
    for (int i = 0; i < k; ++i) {
      const int lo = nb * i / k;
      const int n = nb * (i + 1) / k - lo;
      const int pos = atomicAdd(&s_bkt[bucket(n)], 1);
      if (pos >= p.plan.max_items) {
        raise_error(CIE_DEVERR_BAD_LENGTH);
        continue;
      }
      p.plan.items[2 * pos] = make_int4(b, pair | (h << 16), lo, dead ? 0 : n);
      p.plan.items[2 * pos + 1] = make_int4(rec, split, i, k);
    }
  }
  __syncthreads();
  if (tid == 0) p.plan.header[0] = min(s_cnt[0], p.plan.max_items);
}

// Combines the records of one row of a split tile pair (every piece's
// record, this CTA's included, is written before the last piece gets here):
// O = sum_q w_q acc_q / sum_q w_q l_q with w_q = 2^(m_q - max m), m in log2
// units. Out of line, so that its registers do not weigh on the softmax loop.
// `rec0` points at the row's (O[0], O[1]) entry of the pair's first record.
__device__ __noinline__ void merge_row(const float2* rec0, int n_pieces, __half* dst) {
  constexpr int64_t kStride = static_cast<int64_t>(kRecRows) * kPartCols;
  constexpr int kML = (kD / 2) * kRecRows;
  float M = -CUDART_INF_F;
  for (int q = 0; q < n_pieces; ++q) M = fmaxf(M, __ldcg(rec0 + q * kStride + kML).x);
  float acc[kD];
#pragma unroll
  for (int d = 0; d < kD; ++d) acc[d] = 0.f;
  float den = 0.f;
  for (int q = 0; q < n_pieces; ++q) {
    const float2* rec = rec0 + q * kStride;
    const float2 ml = __ldcg(rec + kML);
    if (ml.x == -CUDART_INF_F) continue;  // no visible key in this piece's range
    const float w = ex2(ml.x - M);
    den += w * ml.y;
#pragma unroll
    for (int cc = 0; cc < kD / 2; ++cc) {
      const float2 a = __ldcg(rec + cc * kRecRows);
      acc[2 * cc] += w * a.x;
      acc[2 * cc + 1] += w * a.y;
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
#pragma unroll
  for (int cc = 0; cc < kD / 8; ++cc) {
    uint4 w;
    w.x = pack_half2(acc[cc * 8 + 0] * inv, acc[cc * 8 + 1] * inv);
    w.y = pack_half2(acc[cc * 8 + 2] * inv, acc[cc * 8 + 3] * inv);
    w.z = pack_half2(acc[cc * 8 + 4] * inv, acc[cc * 8 + 5] * inv);
    w.w = pack_half2(acc[cc * 8 + 6] * inv, acc[cc * 8 + 7] * inv);
    reinterpret_cast<uint4*>(dst)[cc] = w;
  }
}

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
  const Bars bars{sbase + kOffBar};
  uint32_t* tmem_ptr_smem = reinterpret_cast<uint32_t*>(smem + kOffTmemPtr);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + kOffTmemPtr + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // the plan is written by the planning grid, which this launch depends on
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (static_cast<int>(blockIdx.x) >= p.plan.header[0]) return;
  const int4 item = p.plan.items[2 * blockIdx.x];
  const int4 item_m = p.plan.items[2 * blockIdx.x + 1];
  const int b = item.x;
  const int pair = item.y & 0xffff;
  const int h = static_cast<int>(static_cast<unsigned>(item.y) >> 16);
  const int blk0 = item.z;      // first key block of this CTA
  const int n_blocks = item.w;  // key blocks of this CTA
  if (n_blocks <= 0) return;
  const PairInfo pi = pair_info(p, b, pair);
  if (!pi.valid) return;
  const int64_t start = p.cu_seqlens[b];
  const int64_t slot = p.slot_ids[b];
  const int n_keys = pi.kv_len + pi.tok0 + pi.pair_tokens;  // keys of the pair's last row
  const int n_valid_pages = (n_keys + kPage - 1) / kPage;
  const bool direct = item_m.w == 1;                        // write O, no partial
  const int n_tiles = pi.pair_tokens > kTileTokens ? 2 : 1;
  // lane quadrants of tile x whose rows [0, 7 * tokens) hold any real token
  auto quads_of = [&](int x) {
    const int tt = x < n_tiles ? min(pi.pair_tokens - x * kTileTokens, kTileTokens) : 0;
    return (tt * kGroup + 31) / 32;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bars.kv_full(s), 1);
      mbar_init(bars.kv_empty(s), n_tiles);  // one release per tile
    }
    mbar_init(bars.q_full(), 1);
    mbar_init(bars.mma_done(0), 1);
    mbar_init(bars.mma_done(1), 1);
    for (int x = 0; x < 2; ++x) {
      const uint32_t quad_threads = 32u * static_cast<uint32_t>(max(quads_of(x), 1));
      mbar_init(bars.s_full(x), 1);
      mbar_init(bars.s_free(x), quad_threads);
      mbar_init(bars.p_full(x), quad_threads);
      mbar_init(bars.pv_done(x), 1);
      mbar_init(bars.turn(x), 32u * static_cast<uint32_t>(max(quads_of(1 - x), 1)));
    }
    fence_mbar_init();
  }
  // Rows 126 and 127 of each Q tile are never loaded, and tile B's box is
  // skipped when the pair has one tile: zero what TMA will not write so the
  // tensor core only ever sees finite values.
  if (threadIdx.x < 32) {
    const int x = threadIdx.x >> 4;
    const uint32_t addr = sQ + x * kQBytes + kRows * 128 + (threadIdx.x & 15) * 16;
    asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
  }
  if (n_tiles == 1) {
    for (int e = threadIdx.x; e < kQBytes / 16; e += kThreads)
      asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(sQ + kQBytes + e * 16),
                   "r"(0)
                   : "memory");
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

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kCtrlRegs));
    if (warp == 0) {
      // ============================ producer ==================================
      int issued = 0;
      bool ok = true;
      if (lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
        mbar_arrive_expect_tx(bars.q_full(), n_tiles * kQLoadBytes);
        tma_load_4d(sQ, &tm_q, bars.q_full(), 0, 0, h, static_cast<int>(start) + pi.tok0);
        if (n_tiles == 2)
          tma_load_4d(sQ + kQBytes, &tm_q, bars.q_full(), 0, 0, h,
                      static_cast<int>(start) + pi.tok0 + kTileTokens);
      }
      const int64_t bt_row = slot * p.bt_stride;
      for (int j = 0; j < n_blocks; ++j) {
        const int s = j % kStages;
        const uint32_t use = static_cast<uint32_t>(j / kStages);
        int page = 0;  // page ids of this block, read before waiting for the stage
        if (lane < kPagesPerBlock) {
          const int lp = (blk0 + j) * kPagesPerBlock + lane;
          if (lp < n_valid_pages) {
            int64_t pid = p.block_table.at(bt_row + lp);
            if (pid < 0 || pid >= p.n_pages) {
              raise_error(CIE_DEVERR_BAD_PAGE);
              pid = 0;
            }
            page = static_cast<int>(pid);
          }
        }
        if (lane == 0) {
          if (j >= kStages &&
              !mbar_wait(bars.kv_empty(s), (use & 1u) ^ 1u, CIE_DEVERR_WAIT_TIMEOUT))
            ok = false;
          if (ok) mbar_arrive_expect_tx(bars.kv_full(s), kStageBytes);
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        if (lane < kPagesPerBlock) {
          const uint32_t dst = sKV + s * kStageBytes + lane * kPageBoxBytes;
          tma_load_4d(dst, &tm_k, bars.kv_full(s), 0, 0, h, page);
          tma_load_4d(dst + kKVTileBytes, &tm_v, bars.kv_full(s), 0, 0, h, page);
        }
        __syncwarp();
        ++issued;
      }
      // never leave the CTA with copies in flight
      if (lane == 0) {
        mbar_wait(bars.q_full(), 0, CIE_DEVERR_WAIT_TIMEOUT);
        for (int j = max(0, issued - kStages); j < issued; ++j)
          mbar_wait(bars.kv_full(j % kStages), static_cast<uint32_t>(j / kStages) & 1u,
                    CIE_DEVERR_WAIT_TIMEOUT);
      }
    } else if (warp <= 2) {
      // ======================= MMA issuers (warp 1: tile A, warp 2: tile B) ===
      // One warp per tile, in order: S(j) = Q K_j^T as soon as K_j is in and
      // the softmax has read S(j-1), then O += P(j-1) V_{j-1} once P(j-1) is
      // published. A tile's QK^T is never queued behind the other tile's P.V
      // issue, and S(j) goes ahead of PV(j-1), which the softmax needs later.
      // The whole warp runs the loop and one elected lane issues each MMA and
      // commit (the warp shares its SM sub-partition with two softmax warps,
      // which would starve a single-lane issuing branch).
      const int x = warp - 1;
      if (x < n_tiles) {
        bool ok = __all_sync(0xffffffffu, mbar_wait(bars.q_full(), 0, CIE_DEVERR_WAIT_TIMEOUT));
        auto wait = [&](uint32_t bar, uint32_t parity) {
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar, parity, CIE_DEVERR_WAIT_TIMEOUT));
          return ok;
        };
        auto issue_pv = [&](int j) {  // O_x (+)= P_x(j) V_j, P from TMEM
          if (!wait(bars.p_full(x), static_cast<uint32_t>(j) & 1u)) return;
          tc_fence_after();
          const uint32_t v_tile = sKV + (j % kStages) * kStageBytes + kKVTileBytes;
#pragma unroll
          for (int kk = 0; kk < kBlockKeys / 16; ++kk) {
            // 16 keys = 8 P columns; V: 16 keys = two 8-row swizzle atoms of 1 KiB
            const uint64_t db = smem_desc(v_tile + kk * 2048, kKVTileBytes, 1024);
            tc_mma_f16_ts_elect(tmem + x * 256 + kColO, tmem + x * 256 + kColP + kk * 8, db,
                                kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit_elect(bars.pv_done(x));
          tc_commit_elect(bars.kv_empty(j % kStages));  // this tile is done with K_j and V_j
        };
        for (int j = 0; j < n_blocks && ok; ++j) {
          if (!wait(bars.kv_full(j % kStages), static_cast<uint32_t>(j / kStages) & 1u)) break;
          if (j > 0 && !wait(bars.s_free(x), static_cast<uint32_t>(j - 1) & 1u)) break;
          tc_fence_after();
          const uint32_t k_tile = sKV + (j % kStages) * kStageBytes;
#pragma unroll
          for (int k = 0; k < kD / 16; ++k) {  // S_x(j) = Q_x K_j^T
            const uint64_t da = smem_desc(sQ + x * kQBytes + k * 32, 16, 1024);
            const uint64_t db = smem_desc(k_tile + k * 32, 16, 1024);
            tc_mma_f16_elect(tmem + x * 256 + kColS, da, db, kIdescS, k > 0 ? 1u : 0u);
          }
          tc_commit_elect(bars.s_full(x));
          if (j > 0) issue_pv(j - 1);
        }
        if (ok && n_blocks > 0) issue_pv(n_blocks - 1);
        // drain: every MMA this warp issued has completed before TMEM is freed
        tc_commit_elect(bars.mma_done(x));
        mbar_wait(bars.mma_done(x), 0, CIE_DEVERR_WAIT_TIMEOUT);
      }
      __syncwarp();
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ============================ softmax =====================================
    const int x = (warp >> 2) - 1;          // tile
    const int quad = warp & 3;              // TMEM lane quadrant of this warp
    const int row = quad * 32 + lane;       // tile row == TMEM lane
    const int n_quads = quads_of(x);
    if (quad < n_quads) {
      const int tile_tok0 = pi.tok0 + x * kTileTokens;
      const int tile_tokens = min(pi.L - tile_tok0, kTileTokens);
      const int tok_in_tile = row / kGroup;
      const int head_in_group = row - tok_in_tile * kGroup;
      const bool row_valid = row < kRows && tok_in_tile < tile_tokens;
      // inclusive causal limit (absolute key index) of this row; padding rows
      // use the tile's first row limit so that every value stays finite
      const int limit = pi.kv_len + tile_tok0 + (row_valid ? tok_in_tile : 0);
      const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
      const uint32_t t_s = tmem + lane_addr + x * 256 + kColS;
      const uint32_t t_p = tmem + lane_addr + x * 256 + kColP;
      const uint32_t t_o = tmem + lane_addr + x * 256 + kColO;
      // scores in log2 units: u = (q . k) * head_dim^-0.5 * log2(e)
      constexpr float kC = 0.125f * kLog2e;
      const float2 c2 = make_float2(kC, kC);

      float m_ref = -CUDART_INF_F;  // log2-unit max the P values are taken against
      float l_run = 0.f;
      bool ok = true;
      for (int j = 0; j < n_blocks; ++j) {
        const uint32_t par = static_cast<uint32_t>(j) & 1u;
        if (!__all_sync(0xffffffffu, mbar_wait(bars.s_full(x), par, CIE_DEVERR_WAIT_TIMEOUT))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[kBlockKeys];
#pragma unroll
        for (int c = 0; c < kBlockKeys; c += 32)
          tmem_ld_32x32b_x32(t_s + c, *reinterpret_cast<uint32_t(*)[32]>(&sr[c]));
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(bars.s_free(x));
        // With two tiles, their maxima and exponentials take turns (A0, B0, A1,
        // B1, ...): the two softmax warps of an SM sub-partition otherwise run
        // in step and both sit out the ~0.45 us per block spent outside the
        // exponentials; taking turns, one tile's waits overlap the other's
        // exponentials (512-token chunks 97.3 -> 95.1 us, config 3 95.4 -> 93.2).
        // Strict alternation keeps every waiter one phase behind its barrier.
        if (n_tiles == 2 && (x == 1 || j > 0)) {
          const uint32_t tp = static_cast<uint32_t>(x == 1 ? j : j - 1) & 1u;
          if (!__all_sync(0xffffffffu, mbar_wait(bars.turn(x), tp, CIE_DEVERR_WAIT_TIMEOUT))) {
            ok = false;
            break;
          }
        }

        // raw row maximum of this block; masked columns become -inf
        const int lim = limit - (blk0 + j) * kBlockKeys;
        if (lim < kBlockKeys - 1) {
#pragma unroll
          for (int c = 0; c < kBlockKeys; ++c)
            if (c > lim) sr[c] = __float_as_uint(-CUDART_INF_F);
        }
        float mx4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          mx4[e] = fmax3(__uint_as_float(sr[2 * e]), __uint_as_float(sr[2 * e + 1]),
                         -CUDART_INF_F);
#pragma unroll
        for (int c = 8; c < kBlockKeys; c += 8)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            mx4[e] = fmax3(mx4[e], __uint_as_float(sr[c + 2 * e]),
                           __uint_as_float(sr[c + 2 * e + 1]));
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * kC;

        const bool need = mx > m_ref + kRescaleLog2;
        const float alpha = (need && m_ref != -CUDART_INF_F) ? ex2(m_ref - mx) : 1.f;
        if (need) m_ref = mx;
        // no visible key yet: every column is -inf and p = 0
        const float mneg = m_ref == -CUDART_INF_F ? 0.f : -m_ref;
        const float2 mneg2 = make_float2(mneg, mneg);
        float2 lsum0 = make_float2(0.f, 0.f), lsum1 = make_float2(0.f, 0.f);
        uint32_t pw[kBlockKeys / 2];
#pragma unroll
        for (int c8 = 0; c8 < kBlockKeys / 8; ++c8) {
          float pv[8];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const float2 t = __ffma2_rn(make_float2(__uint_as_float(sr[c8 * 8 + e]),
                                                    __uint_as_float(sr[c8 * 8 + e + 1])),
                                        c2, mneg2);
            if ((kPolyPairs >> ((c8 & 1) * 4 + e / 2)) & 1u) {
              const float2 r = exp2_fma2(t);
              pv[e] = r.x;
              pv[e + 1] = r.y;
            } else {
              pv[e] = ex2(t.x);
              pv[e + 1] = ex2(t.y);
            }
          }
          lsum0 = __fadd2_rn(lsum0, __fadd2_rn(make_float2(pv[0], pv[1]), make_float2(pv[4], pv[5])));
          lsum1 = __fadd2_rn(lsum1, __fadd2_rn(make_float2(pv[2], pv[3]), make_float2(pv[6], pv[7])));
          pw[c8 * 4 + 0] = pack_half2(pv[0], pv[1]);
          pw[c8 * 4 + 1] = pack_half2(pv[2], pv[3]);
          pw[c8 * 4 + 2] = pack_half2(pv[4], pv[5]);
          pw[c8 * 4 + 3] = pack_half2(pv[6], pv[7]);
        }
        l_run = l_run * alpha + ((lsum0.x + lsum0.y) + (lsum1.x + lsum1.y));
        if (n_tiles == 2) mbar_arrive(bars.turn(1 - x));  // the other tile's turn

        // PV(j-1) must have consumed P(j-1) and finished updating O
        if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(bars.pv_done(x), par ^ 1u,
                                                         CIE_DEVERR_WAIT_TIMEOUT))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // TMEM round trip of O by the whole warp when any of its rows moved
        // its max; the other rows multiply by 1. O holds nothing before the
        // first PV of this CTA (j == 0).
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < kD; c += 16) {  // 16 columns at a time: few live registers
            uint32_t o[16];
            tmem_ld_32x32b_x16(t_o + c, o);
            tc_wait_ld();
#pragma unroll
            for (int d = 0; d < 16; ++d) o[d] = __float_as_uint(__uint_as_float(o[d]) * alpha);
            tmem_st_32x32b_x16(t_o + c, o);
          }
        }
        tmem_st_32x32b_x32(t_p, pw);
        tmem_st_32x32b_x32(t_p + 32, pw + 32);

        // V rows past the pair's last key hold stale pool data: zero them so
        // that 0 * (non-finite) cannot reach an accumulator. Each tile's
        // working threads write the (same) zeros before their own p_full
        // arrival, because the two tiles' PVs are issued independently.
        if (blk0 + j == pi.n_blocks - 1) {
          const int first = n_keys - (blk0 + j) * kBlockKeys;
          const int rows = kBlockKeys - first;
          if (rows > 0) {
            const uint32_t vtile = sKV + (j % kStages) * kStageBytes + kKVTileBytes;
            const int nthr = 32 * n_quads;
            for (int e = quad * 32 + lane; e < rows * 8; e += nthr) {
              asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(
                               vtile + sw128(first + (e >> 3), e & 7)),
                           "r"(0)
                           : "memory");
            }
            fence_proxy_async_smem();
          }
        }
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(bars.p_full(x));
      }
      // last PV of this tile
      if (ok && n_blocks > 0)
        ok = __all_sync(0xffffffffu, mbar_wait(bars.pv_done(x),
                                               static_cast<uint32_t>(n_blocks - 1) & 1u,
                                               CIE_DEVERR_WAIT_TIMEOUT));
      tc_fence_after();
      uint32_t ob[kD];
      tmem_ld_32x32b_x32(t_o, *reinterpret_cast<uint32_t(*)[32]>(&ob[0]));
      tmem_ld_32x32b_x32(t_o + 32, *reinterpret_cast<uint32_t(*)[32]>(&ob[32]));
      tc_wait_ld();
      const int64_t tok = start + tile_tok0 + tok_in_tile;
      const int hq = h * kGroup + head_in_group;
      auto store_o = [&](float inv) {
        __half* dst = p.o + (tok * p.num_q_heads + hq) * kD;
#pragma unroll
        for (int cc = 0; cc < kD / 8; ++cc) {
          uint4 w;
          w.x = pack_half2(__uint_as_float(ob[cc * 8 + 0]) * inv,
                           __uint_as_float(ob[cc * 8 + 1]) * inv);
          w.y = pack_half2(__uint_as_float(ob[cc * 8 + 2]) * inv,
                           __uint_as_float(ob[cc * 8 + 3]) * inv);
          w.z = pack_half2(__uint_as_float(ob[cc * 8 + 4]) * inv,
                           __uint_as_float(ob[cc * 8 + 5]) * inv);
          w.w = pack_half2(__uint_as_float(ob[cc * 8 + 6]) * inv,
                           __uint_as_float(ob[cc * 8 + 7]) * inv);
          reinterpret_cast<uint4*>(dst)[cc] = w;
        }
      };
      if (direct) {
        if (ok && row_valid) store_o(1.f / l_run);
      } else {
        // This piece's partial (m = -inf when its key range had no visible
        // key for the row). The last piece of the pair to finish combines
        // all of them: O = sum_q w_q acc_q / sum_q w_q l_q, w_q = 2^(m_q - max m).
        // the item's split fields, read again here rather than kept live
        // through the softmax loop
        int4 im;
        asm volatile("ld.global.cg.v4.s32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(im.x), "=r"(im.y), "=r"(im.z), "=r"(im.w)
                     : "l"(p.plan.items + 2 * blockIdx.x + 1));
        const int rec0 = im.x, split = im.y, piece = im.z, n_pieces = im.w;
        if (row_valid) {
          float2* rec = reinterpret_cast<float2*>(p.plan.records) +
                        static_cast<int64_t>(rec0 + piece) * kRecRows * kPartCols + x * kM + row;
#pragma unroll
          for (int cc = 0; cc < kD / 2; ++cc)
            rec[cc * kRecRows] =
                make_float2(__uint_as_float(ob[cc * 2 + 0]), __uint_as_float(ob[cc * 2 + 1]));
          // a piece whose pipeline wait gave up (ok == false; the device
          // error bit is set) publishes an empty range, which the merge skips,
          // instead of whatever its accumulators hold
          rec[(kD / 2) * kRecRows] =
              ok ? make_float2(m_ref, l_run) : make_float2(-CUDART_INF_F, 0.f);
        }
        __threadfence();
        // every working softmax thread of both tiles has published its rows
        const uint32_t n_thr = 32u * static_cast<uint32_t>(quads_of(0) + quads_of(1));
        asm volatile("bar.sync 1, %0;" ::"r"(n_thr) : "memory");
        if (warp == 4 && lane == 0)
          *last_flag = atomicAdd(p.plan.counters + split, 1u) ==
                               static_cast<unsigned>(n_pieces - 1)
                           ? 1
                           : 0;
        asm volatile("bar.sync 1, %0;" ::"r"(n_thr) : "memory");
        if (*last_flag != 0 && row_valid && ok) {
          __threadfence();
          merge_row(reinterpret_cast<const float2*>(p.plan.records) +
                        static_cast<int64_t>(rec0) * kRecRows * kPartCols + x * kM + row,
                    n_pieces, p.o + (tok * p.num_q_heads + hq) * kD);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// Workspace layout: the plan header, the items, the split counters and the
// partial records, each section 256-byte aligned. The bounds hold for any
// lengths: a sequence has at most ceil(L / 36) <= L / 36 + 1 tile pairs; with
// num_splits = S every pair is cut into at most S pieces; automatically a
// pair of nb blocks gets at most nb / C + 1 pieces and only pairs longer than
// C (fewer than total / C <= plan_slots(SMs) of them) are cut, so the pieces of
// cut pairs number at most 2 * plan_slots(SMs).
struct PlanSizes {
  int64_t items, split, rec;
  size_t off_items, off_counters, off_records, bytes;
};

inline size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

inline PlanSizes plan_sizes(int batch, int64_t total_tokens, int num_kv_heads, int num_splits,
                            int n_sm) {
  PlanSizes ps{};
  const int64_t units =
      static_cast<int64_t>(num_kv_heads) * ((total_tokens + kPairTokens - 1) / kPairTokens + batch);
  if (num_splits >= 1) {
    ps.items = num_splits * units;
    ps.split = num_splits > 1 ? units : 0;
    ps.rec = num_splits > 1 ? num_splits * units : 0;
  } else {
    const int64_t slots = plan_slots(n_sm);
    ps.items = units + slots;
    ps.split = slots;
    ps.rec = 2 * slots;
  }
  ps.off_items = 256;
  ps.off_counters = ps.off_items + round256(static_cast<size_t>(ps.items) * 2 * sizeof(int4));
  ps.off_records = ps.off_counters + round256(static_cast<size_t>(ps.split) * sizeof(unsigned));
  ps.bytes = ps.off_records +
             static_cast<size_t>(ps.rec) * kRecRows * kPartFloats * sizeof(float);
  return ps;
}

inline int device_sms(int device) {
  int n = 0;
  if (device >= 0 &&
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && n > 0)
    return n;
  return 148;
}

}  // namespace mixed
}  // namespace cie

extern "C" {

size_t cie_mixed_workspace_bytes(int batch, int64_t total_tokens, int num_kv_heads,
                                 int num_splits, int device) {
  using namespace cie::mixed;
  if (batch < 0 || total_tokens < 0 || num_kv_heads < 1) return 0;
  return plan_sizes(batch, total_tokens, num_kv_heads, num_splits, device_sms(device)).bytes;
}

}  // extern "C"

namespace cie {
namespace mixed {

// Argument checks, tensor maps and the two launches of cie_mixed_attention
// (and of its int32-block-table variant). With `rope` (cie_rope_kv_mixed_attention)
// q is ignored: the planning grid's extra CTAs rotate the pass's q into the
// workspace tail and write its k / v rows to their pages first.
int entry(const void* q, const void* k, const void* v, int64_t max_seqlen,
          const int64_t* cu_seqlens, const int64_t* kv_lens, const int64_t* slot_ids,
          BlockTable block_table, void* o, void* workspace, size_t workspace_bytes, int batch,
          int64_t total_tokens, int num_q_heads, int num_kv_heads, int head_dim, int page_size,
          int64_t n_pages, int64_t n_slots, int64_t bt_stride, int64_t kv_page_stride,
          int64_t kv_head_stride, int num_splits, cie_stream_t stream,
          const rope::Args* rope = nullptr) {
  if (batch < 0 || total_tokens < 0 || max_seqlen < 0)
    return fail(CIE_ERR_INVALID_ARGUMENT, "negative batch / total_tokens / max_seqlen");
  if (rope != nullptr && total_tokens > 0 && (batch == 0 || max_seqlen == 0)) {
    // no attention to compute, but the pass's rows still go to their pages
    rope::Args ra = *rope;
    ra.q_out = static_cast<__half*>(workspace);
    if (workspace == nullptr ||
        workspace_bytes < static_cast<size_t>(total_tokens) * num_q_heads * kD * 2)
      return fail(CIE_ERR_WORKSPACE, "the rotated q needs workspace");
    return rope::launch(ra, head_dim, stream);
  }
  if (batch == 0 || total_tokens == 0 || max_seqlen == 0) return CIE_OK;
  if ((!q && !rope) || !k || !v || !cu_seqlens || !kv_lens || !slot_ids || !block_table.ptr || !o)
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
  const int64_t n_pairs = (max_seqlen + kPairTokens - 1) / kPairTokens;
  if (n_pairs > 65535)
    return fail(CIE_ERR_UNSUPPORTED, "max_seqlen %lld needs more than 65535 query tile pairs",
                (long long)max_seqlen);
  if (static_cast<int64_t>(batch) * num_kv_heads > 0x7fffffff)
    return fail(CIE_ERR_OVERFLOW, "batch x kv heads does not fit the grid");
  if (kv_head_stride < page_size * head_dim || kv_page_stride < kv_head_stride * num_kv_heads)
    return fail(CIE_ERR_INVALID_ARGUMENT, "overlapping K/V strides");
  if ((kv_page_stride % 8) || (kv_head_stride % 8) || !aligned16(k) || !aligned16(v) ||
      !aligned16(q) || !aligned16(o))
    return fail(CIE_ERR_ALIGNMENT, "q/o/k/v must be 16-byte aligned with 16-byte strides");
  if (num_splits > kMaxSplits)
    return fail(CIE_ERR_INVALID_ARGUMENT, "num_splits %d > %d", num_splits, kMaxSplits);
  if (batch > kPlanMaxBatch)
    return fail(CIE_ERR_UNSUPPORTED, "batch %d > %d sequences", batch, kPlanMaxBatch);
  if (num_kv_heads > 32767) return fail(CIE_ERR_UNSUPPORTED, "num_kv_heads %d", num_kv_heads);
  const int n_sm = sm_count();
  const PlanSizes ps = plan_sizes(batch, total_tokens, num_kv_heads, num_splits, n_sm);
  if (ps.items > 0x7fffffff) return fail(CIE_ERR_OVERFLOW, "too many work items");
  size_t need = ps.bytes;
  rope::Args ra{};
  int rope_ctas = 0;
  if (rope != nullptr) {
    const size_t q_off = round256(ps.bytes);
    need = q_off + static_cast<size_t>(total_tokens) * num_q_heads * kD * 2;
    ra = *rope;
    ra.q_out = workspace ? reinterpret_cast<__half*>(static_cast<uint8_t*>(workspace) + q_off)
                         : nullptr;
    ra.k_cache = static_cast<__half*>(const_cast<void*>(k));
    ra.v_cache = static_cast<__half*>(const_cast<void*>(v));
    ra.page_stride = kv_page_stride;
    ra.head_stride = kv_head_stride;
    ra.num_tokens = total_tokens;
    ra.hq = num_q_heads;
    ra.hkv = num_kv_heads;
    ra.page_size = page_size;
    ra.n_pages = n_pages;
    q = ra.q_out;
  }
  if (workspace == nullptr || workspace_bytes < need)
    return fail(CIE_ERR_WORKSPACE, "mixed attention needs %zu workspace bytes, got %zu", need,
                workspace == nullptr ? size_t(0) : workspace_bytes);
  if (rope != nullptr) {
    const int st = rope::check(ra, head_dim);
    if (st != CIE_OK) return st;
    const int64_t blocks = (rope::work_items(ra) + kPlanThreads - 1) / kPlanThreads;
    rope_ctas = static_cast<int>(blocks < 4 * n_sm ? blocks : 4 * n_sm);
  }
  if (!aligned16(workspace)) return fail(CIE_ERR_ALIGNMENT, "workspace must be 16-byte aligned");

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
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.plan.header = reinterpret_cast<int*>(ws);
  p.plan.items = reinterpret_cast<int4*>(ws + ps.off_items);
  p.plan.counters = reinterpret_cast<unsigned*>(ws + ps.off_counters);
  p.plan.records = reinterpret_cast<float*>(ws + ps.off_records);
  p.plan.max_items = static_cast<int>(ps.items);
  p.plan.max_split = static_cast<int>(ps.split);
  p.plan.max_rec = static_cast<int>(ps.rec);
  p.total_tokens = total_tokens;
  p.max_seqlen = max_seqlen;
  p.n_pages = n_pages;
  p.n_slots = n_slots;
  p.bt_stride = bt_stride;
  p.batch = batch;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.num_splits = num_splits;
  p.n_sm = n_sm;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  mixed_plan_kernel<<<1 + rope_ctas, kPlanThreads, 0, s>>>(p, ra, rope_ctas);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "mixed plan launch: %s", cudaGetErrorString(e));
  // one CTA per item (the plan holds at most ps.items; the rest return at
  // once); scheduled while the plan is made, waiting for it in griddepcontrol.wait
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ps.items));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, mixed_attention_kernel, tm_q, tm_k, tm_v, p);
  if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "mixed launch: %s", cudaGetErrorString(e));
  return CIE_OK;
}

}  // namespace mixed
}  // namespace cie

extern "C" {

int cie_mixed_attention(const void* q, const void* k, const void* v, int64_t max_seqlen,
                        const int64_t* cu_seqlens, const int64_t* kv_lens,
                        const int64_t* slot_ids, const int64_t* block_table, void* o,
                        void* workspace, size_t workspace_bytes, int batch,
                        int64_t total_tokens, int num_q_heads, int num_kv_heads, int head_dim,
                        int page_size, int64_t n_pages, int64_t n_slots, int64_t bt_stride,
                        int64_t kv_page_stride, int64_t kv_head_stride, int num_splits,
                        cie_stream_t stream) {
  return cie::mixed::entry(q, k, v, max_seqlen, cu_seqlens, kv_lens, slot_ids,
                           cie::BlockTable{block_table, 1}, o, workspace, workspace_bytes, batch,
                           total_tokens, num_q_heads, num_kv_heads, head_dim, page_size, n_pages,
                           n_slots, bt_stride, kv_page_stride, kv_head_stride, num_splits, stream);
}

int cie_mixed_attention_bt32(const void* q, const void* k, const void* v, int64_t max_seqlen,
                             const int64_t* cu_seqlens, const int64_t* kv_lens,
                             const int64_t* slot_ids, const int32_t* block_table, void* o,
                             void* workspace, size_t workspace_bytes, int batch,
                             int64_t total_tokens, int num_q_heads, int num_kv_heads,
                             int head_dim, int page_size, int64_t n_pages, int64_t n_slots,
                             int64_t bt_stride, int64_t kv_page_stride, int64_t kv_head_stride,
                             int num_splits, cie_stream_t stream) {
  return cie::mixed::entry(q, k, v, max_seqlen, cu_seqlens, kv_lens, slot_ids,
                           cie::BlockTable{block_table, 0}, o, workspace, workspace_bytes, batch,
                           total_tokens, num_q_heads, num_kv_heads, head_dim, page_size, n_pages,
                           n_slots, bt_stride, kv_page_stride, kv_head_stride, num_splits, stream);
}

// cie_rope_kv_mixed_attention and its int32-block-table twin.
static int rope_kv_mixed_attention(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                                   const void* sin, int64_t cs_tok_stride, void* k_cache,
                                   void* v_cache, const int64_t* pages, const int64_t* offsets,
                                   int64_t max_seqlen, const int64_t* cu_seqlens,
                                   const int64_t* kv_lens, const int64_t* slot_ids,
                                   cie::BlockTable block_table, void* o, void* workspace,
                                   size_t workspace_bytes, int batch, int64_t total_tokens,
                                   int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                                   int64_t n_pages, int64_t n_slots, int64_t bt_stride,
                                   int64_t cache_page_stride, int64_t cache_head_stride,
                                   int num_splits, cie_stream_t stream) {
  using namespace cie;
  if (total_tokens > 0 && (!pages || !offsets))
    return fail(CIE_ERR_INVALID_ARGUMENT, "null pages / offsets");
  rope::Args ra{};
  ra.qkv = static_cast<const __half*>(qkv);
  ra.qkv_tok = qkv_tok_stride;
  ra.cos = static_cast<const __half*>(cos);
  ra.sin = static_cast<const __half*>(sin);
  ra.cs_tok = cs_tok_stride;
  ra.k_cache = static_cast<__half*>(k_cache);
  ra.v_cache = static_cast<__half*>(v_cache);
  ra.page_stride = cache_page_stride;
  ra.head_stride = cache_head_stride;
  ra.pages = pages;
  ra.offsets = offsets;
  ra.num_tokens = total_tokens;
  ra.hq = num_q_heads;
  ra.hkv = num_kv_heads;
  ra.page_size = page_size;
  ra.n_pages = n_pages;
  return mixed::entry(nullptr, k_cache, v_cache, max_seqlen, cu_seqlens, kv_lens, slot_ids,
                      block_table, o, workspace, workspace_bytes, batch, total_tokens,
                      num_q_heads, num_kv_heads, head_dim, page_size, n_pages, n_slots, bt_stride,
                      cache_page_stride, cache_head_stride, num_splits, stream, &ra);
}

size_t cie_rope_kv_mixed_workspace_bytes(int batch, int64_t total_tokens, int num_q_heads,
                                         int num_kv_heads, int num_splits, int device) {
  using namespace cie::mixed;
  if (batch < 0 || total_tokens < 0 || num_kv_heads < 1 || num_q_heads < 1) return 0;
  const size_t q_bytes = static_cast<size_t>(total_tokens) * num_q_heads * kD * 2;
  return round256(cie_mixed_workspace_bytes(batch, total_tokens, num_kv_heads, num_splits,
                                            device)) +
         q_bytes;
}

int cie_rope_kv_mixed_attention(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                                const void* sin, int64_t cs_tok_stride, void* k_cache,
                                void* v_cache, const int64_t* pages, const int64_t* offsets,
                                int64_t max_seqlen, const int64_t* cu_seqlens,
                                const int64_t* kv_lens, const int64_t* slot_ids,
                                const int64_t* block_table, void* o, void* workspace,
                                size_t workspace_bytes, int batch, int64_t total_tokens,
                                int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                                int64_t n_pages, int64_t n_slots, int64_t bt_stride,
                                int64_t cache_page_stride, int64_t cache_head_stride,
                                int num_splits, cie_stream_t stream) {
  return rope_kv_mixed_attention(qkv, qkv_tok_stride, cos, sin, cs_tok_stride, k_cache, v_cache,
                                 pages, offsets, max_seqlen, cu_seqlens, kv_lens, slot_ids,
                                 cie::BlockTable{block_table, 1}, o, workspace, workspace_bytes,
                                 batch, total_tokens, num_q_heads, num_kv_heads, head_dim,
                                 page_size, n_pages, n_slots, bt_stride, cache_page_stride,
                                 cache_head_stride, num_splits, stream);
}

int cie_rope_kv_mixed_attention_bt32(
    const void* qkv, int64_t qkv_tok_stride, const void* cos, const void* sin,
    int64_t cs_tok_stride, void* k_cache, void* v_cache, const int64_t* pages,
    const int64_t* offsets, int64_t max_seqlen, const int64_t* cu_seqlens, const int64_t* kv_lens,
    const int64_t* slot_ids, const int32_t* block_table, void* o, void* workspace,
    size_t workspace_bytes, int batch, int64_t total_tokens, int num_q_heads, int num_kv_heads,
    int head_dim, int page_size, int64_t n_pages, int64_t n_slots, int64_t bt_stride,
    int64_t cache_page_stride, int64_t cache_head_stride, int num_splits, cie_stream_t stream) {
  return rope_kv_mixed_attention(qkv, qkv_tok_stride, cos, sin, cs_tok_stride, k_cache, v_cache,
                                 pages, offsets, max_seqlen, cu_seqlens, kv_lens, slot_ids,
                                 cie::BlockTable{block_table, 0}, o, workspace, workspace_bytes,
                                 batch, total_tokens, num_q_heads, num_kv_heads, head_dim,
                                 page_size, n_pages, n_slots, bt_stride, cache_page_stride,
                                 cache_head_stride, num_splits, stream);
}

}  // extern "C"
