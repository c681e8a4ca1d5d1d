// Greedy token after the last-token lm_head, in one pass over the weight:
// tokens[b] = argmax_v fp16(hidden[b] . weight[v]) with torch.argmax's
// semantics (first index of the maximum, NaN counting as the largest), and
// optionally the fp16 logits themselves.
//
// Replaces the lm_head GEMM + argmax of the reference's decode and mixed
// modules (scheduler/decode_module.py:103-107, scheduler/mixed_module.py:58-65)
// for the rows whose next token is sampled. The weight (vocab x hidden,
// 151936 x 896 fp16 = 272 MB for Qwen2.5-0.5B) is the only large operand, so
// the kernel is a stream of it at HBM rate: every CTA walks vocab chunks of
// 128 rows (chunk c, c + grid, ...), TMA-loads each chunk 64 columns of K at a
// time (128 x 64 fp16 = 16 KiB boxes, 128-byte swizzle) into a 5-stage ring,
// and the tensor core computes D[128 vocab x N] = W_chunk . H^T with the
// hidden rows (N <= 64 of them, zero-padded to a multiple of 16) resident in
// shared memory and D in TMEM (two buffers, so that the epilogue of chunk i
// overlaps the MMAs of chunk i + 1).
//
// Epilogue (warps 4-7, thread = vocab row = TMEM lane): each of the N logits
// of the row is rounded to fp16 (what a fp16 GEMM returns), optionally stored,
// and turned into a 32-bit key: the fp16 bits mapped to an unsigned order
// (NaN above +inf, -0 equal to +0) in the high half, 0xFFFF - row in the low
// half, so that one redux.sync.max per column gives the warp's largest value
// and, among equal values, its first row. The four warps' keys are combined in
// shared memory and compared with the CTA's best so far (strictly greater
// replaces: chunks are visited in increasing order). Each CTA writes one
// 64-bit key per row (value order << 32 | ~index); a one-warp-per-row kernel,
// launched with programmatic stream serialisation, takes the maximum.
//
// Warp roles (256 threads): warp 0 TMA producer, warp 1 MMA issuer (and TMEM
// owner), warps 2-3 idle, warps 4-7 epilogue. Every wait is bounded; on a
// timeout the kernel records CIE_DEVERR_WAIT_TIMEOUT and returns without
// leaving copies or MMAs in flight.
#include "cie_common.cuh"
#include "cie_host.h"
#include "cie_model_ops.h"

namespace cie {
namespace lmhead {

constexpr int kChunkRows = 128;                 // vocab rows per chunk (MMA M)
constexpr int kKBlock = 64;                     // K columns per TMA box (128 bytes)
constexpr int kStages = 5;
constexpr int kMaxN = 64;                       // hidden rows per launch slice
constexpr int kThreads = 256;
constexpr int kWBoxBytes = kChunkRows * kKBlock * 2;   // 16 KiB
constexpr int kHBlockBytes = kMaxN * kKBlock * 2;      // 8 KiB per K block at N = 64
constexpr int kMaxK = 1024;                            // hidden size bound (smem)
constexpr int kOffRing = 0;
constexpr int kOffH = kOffRing + kStages * kWBoxBytes;
constexpr int kOffRed = kOffH + (kMaxK / kKBlock) * kHBlockBytes;  // [4][kMaxN] keys
constexpr int kOffBar = kOffRed + 4 * kMaxN * 4;
// barriers: full[kStages], empty[kStages], h_full, acc_full[2], acc_empty[2], done
constexpr int kNumBars = 2 * kStages + 1 + 2 + 2 + 1;
constexpr int kOffTmemPtr = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = 1024 + kOffTmemPtr + 16;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
constexpr uint32_t kTmemCols = 2 * kMaxN;

struct Params {
  int64_t* partial;     // [grid][n_pad] 64-bit keys
  __half* logits;       // optional: (rows, vocab) at logits_stride, this slice's rows
  int64_t logits_stride;
  int64_t vocab;
  int rows;             // hidden rows of this slice (<= kMaxN)
  int n_pad;            // rows rounded up to 16
  int k_blocks;         // hidden / 64
  int n_chunks;         // ceil(vocab / 128)
};

struct Bars {
  uint32_t base;
  __device__ uint32_t full(int s) const { return base + 8u * s; }
  __device__ uint32_t empty(int s) const { return base + 8u * (kStages + s); }
  __device__ uint32_t h_full() const { return base + 8u * (2 * kStages); }
  __device__ uint32_t acc_full(int b) const { return base + 8u * (2 * kStages + 1 + b); }
  __device__ uint32_t acc_empty(int b) const { return base + 8u * (2 * kStages + 3 + b); }
  __device__ uint32_t done() const { return base + 8u * (2 * kStages + 5); }
};

// fp16 bits -> unsigned order of torch.argmax: NaN largest, -0 == +0.
__device__ __forceinline__ uint32_t order16(uint32_t h) {
  if ((h & 0x7FFFu) > 0x7C00u) return 0xFFFFu;
  if (h == 0x8000u) h = 0u;
  return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}

__device__ __forceinline__ uint32_t redux_max(uint32_t v) {
  uint32_t r;
  asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__global__ void __launch_bounds__(kThreads, 1)
    lm_head_argmax_kernel(const __grid_constant__ CUtensorMap tm_w,
                          const __grid_constant__ CUtensorMap tm_h, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sRing = sbase + kOffRing;
  const uint32_t sH = sbase + kOffH;
  uint32_t* red = reinterpret_cast<uint32_t*>(smem + kOffRed);
  const Bars bars{sbase + kOffBar};
  uint32_t* tmem_ptr_smem = reinterpret_cast<uint32_t*>(smem + kOffTmemPtr);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the final kernel may be scheduled now; it waits for this grid to finish
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // chunks of this CTA: blockIdx.x, + gridDim.x, ... (increasing vocab order)
  const int my_chunks =
      (p.n_chunks - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
      static_cast<int>(gridDim.x);
  const int h_block_bytes = p.n_pad * kKBlock * 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bars.full(s), 1);
      mbar_init(bars.empty(s), 1);
    }
    mbar_init(bars.h_full(), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(bars.acc_full(b), 1);
      mbar_init(bars.acc_empty(b), 4);  // one arrival per epilogue warp
    }
    mbar_init(bars.done(), 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_ptr_smem), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_ptr_smem;
  const uint32_t idesc = idesc_f16_f32(kChunkRows, p.n_pad, false);

  if (warp == 0) {
    // ============================ producer ====================================
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_h);
      mbar_arrive_expect_tx(bars.h_full(), static_cast<uint32_t>(p.k_blocks * h_block_bytes));
      for (int kb = 0; kb < p.k_blocks; ++kb)
        tma_load_3d(sH + kb * kHBlockBytes, &tm_h, bars.h_full(), kb * kKBlock, 0, 0);
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < my_chunks && ok; ++i) {
        const int v0 = (static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x)) * kChunkRows;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++issued) {
          const int s = issued % kStages;
          const uint32_t use = static_cast<uint32_t>(issued / kStages);
          if (issued >= kStages &&
              !mbar_wait(bars.empty(s), (use & 1u) ^ 1u, CIE_DEVERR_WAIT_TIMEOUT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bars.full(s), kWBoxBytes);
          tma_load_3d(sRing + s * kWBoxBytes, &tm_w, bars.full(s), kb * kKBlock, v0, 0);
        }
      }
      // never leave the CTA with copies in flight
      mbar_wait(bars.h_full(), 0, CIE_DEVERR_WAIT_TIMEOUT);
      for (int j = max(0, issued - kStages); j < issued; ++j)
        mbar_wait(bars.full(j % kStages), static_cast<uint32_t>(j / kStages) & 1u,
                  CIE_DEVERR_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ============================ MMA issuer ==================================
    // The whole warp runs the loop; one elected lane issues each MMA and commit
    // (a single-lane branch issues slowly beside a busy epilogue warp).
    bool ok = __all_sync(0xffffffffu, mbar_wait(bars.h_full(), 0, CIE_DEVERR_WAIT_TIMEOUT));
    int consumed = 0;
    for (int i = 0; i < my_chunks && ok; ++i) {
      const int buf = i & 1;
      if (i >= 2 &&
          !__all_sync(0xffffffffu, mbar_wait(bars.acc_empty(buf),
                                             static_cast<uint32_t>((i >> 1) - 1) & 1u,
                                             CIE_DEVERR_WAIT_TIMEOUT))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + static_cast<uint32_t>(buf * kMaxN);
      for (int kb = 0; kb < p.k_blocks; ++kb, ++consumed) {
        const int s = consumed % kStages;
        if (!__all_sync(0xffffffffu, mbar_wait(bars.full(s),
                                               static_cast<uint32_t>(consumed / kStages) & 1u,
                                               CIE_DEVERR_WAIT_TIMEOUT))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kKBlock / 16; ++k) {
          const uint64_t da = smem_desc(sRing + s * kWBoxBytes + k * 32, 16, 1024);
          const uint64_t db = smem_desc(sH + kb * kHBlockBytes + k * 32, 16, 1024);
          tc_mma_f16_elect(d, da, db, idesc, (kb > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit_elect(bars.empty(s));
      }
      if (ok) tc_commit_elect(bars.acc_full(buf));
    }
    // every MMA issued here has completed before TMEM is freed
    tc_commit_elect(bars.done());
    mbar_wait(bars.done(), 0, CIE_DEVERR_WAIT_TIMEOUT);
    __syncwarp();
  } else if (warp >= 4) {
    // ============================ epilogue ====================================
    const int q = warp & 3;                 // TMEM lane quadrant
    const int row = q * 32 + lane;          // vocab row inside the chunk
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const int et = threadIdx.x - 128;       // 0..127 over the epilogue warps
    uint32_t best_ord = 0;                  // this thread's column (et < rows)
    int64_t best_idx = 0;
    bool have = false;
    bool ok = true;
    // Every epilogue warp reaches both named barriers of every chunk, also
    // after a wait gave up (then it skips its work), so none can be left
    // waiting at a barrier.
    for (int i = 0; i < my_chunks; ++i) {
      const int buf = i & 1;
      const int64_t v0 = (static_cast<int64_t>(blockIdx.x) + static_cast<int64_t>(i) * gridDim.x) *
                         kChunkRows;
      if (ok)
        ok = __all_sync(0xffffffffu, mbar_wait(bars.acc_full(buf), static_cast<uint32_t>(i >> 1) & 1u,
                                               CIE_DEVERR_WAIT_TIMEOUT));
      if (ok) {
        tc_fence_after();
        const bool valid = v0 + row < p.vocab;
        for (int c0 = 0; c0 < p.n_pad; c0 += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(tmem + lane_addr + static_cast<uint32_t>(buf * kMaxN + c0), r);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int n = c0 + e;
            const __half hv = __float2half_rn(__uint_as_float(r[e]));
            const uint32_t bits = __half_as_ushort(hv);
            if (p.logits != nullptr && valid && n < p.rows)
              p.logits[static_cast<int64_t>(n) * p.logits_stride + v0 + row] = hv;
            const uint32_t key =
                valid ? (order16(bits) << 16) | (0xFFFFu - static_cast<uint32_t>(row)) : 0u;
            const uint32_t m = redux_max(key);
            if (lane == 0) red[q * kMaxN + n] = m;
          }
        }
        // this buffer is free for the MMAs of chunk i + 2
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bars.acc_empty(buf));
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (ok && et < p.rows) {
        uint32_t k = red[et];
        k = max(k, red[kMaxN + et]);
        k = max(k, red[2 * kMaxN + et]);
        k = max(k, red[3 * kMaxN + et]);
        const uint32_t ord = k >> 16;
        if (!have || ord > best_ord) {
          best_ord = ord;
          best_idx = v0 + static_cast<int64_t>(0xFFFFu - (k & 0xFFFFu));
          have = true;
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
    }
    if (et < p.n_pad)
      p.partial[static_cast<int64_t>(blockIdx.x) * p.n_pad + et] =
          have ? static_cast<int64_t>((static_cast<uint64_t>(best_ord) << 32) |
                                      (0xFFFFFFFFull - static_cast<uint64_t>(best_idx)))
               : 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// tokens[b] = the index in the largest of the grid's keys for row b (one warp per row).
__global__ void lm_head_final_kernel(const int64_t* __restrict__ partial, int grid, int n_pad,
                                     int64_t* __restrict__ tokens) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.x;
  unsigned long long best = 0;
  for (int g = threadIdx.x; g < grid; g += 32)
    best = max(best, static_cast<unsigned long long>(partial[static_cast<int64_t>(g) * n_pad + b]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  if (threadIdx.x == 0) tokens[b] = static_cast<int64_t>(0xFFFFFFFFull - (best & 0xFFFFFFFFull));
}

inline int grid_for(int64_t vocab, int device) {
  int sms = 148;
  int n = 0;
  if (device >= 0 && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) ==
                         cudaSuccess && n > 0)
    sms = n;
  const int64_t chunks = (vocab + kChunkRows - 1) / kChunkRows;
  return static_cast<int>(chunks < sms ? chunks : sms);
}

}  // namespace lmhead
}  // namespace cie

extern "C" {

size_t cie_lm_head_argmax_workspace_bytes(int batch, int64_t vocab, int device) {
  using namespace cie::lmhead;
  if (batch <= 0 || vocab <= 0) return 0;
  const int slices = (batch + kMaxN - 1) / kMaxN;
  return static_cast<size_t>(slices) * grid_for(vocab, device) * kMaxN * sizeof(int64_t);
}

int cie_lm_head_argmax(const void* hidden, int64_t hidden_stride, const void* weight,
                       int64_t weight_stride, int batch, int hidden_size, int64_t vocab,
                       void* logits, int64_t logits_stride, int64_t* tokens, void* workspace,
                       size_t workspace_bytes, cie_stream_t stream) {
  using namespace cie;
  using namespace cie::lmhead;
  if (batch < 0) return fail(CIE_ERR_INVALID_ARGUMENT, "batch < 0");
  if (batch == 0) return CIE_OK;
  if (!hidden || !weight || !tokens) return fail(CIE_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (vocab < 1 || vocab >= (int64_t(1) << 30))
    return fail(CIE_ERR_UNSUPPORTED, "vocab %lld (1 .. 2^30 - 1)", (long long)vocab);
  if (hidden_size < kKBlock || hidden_size > kMaxK || hidden_size % kKBlock)
    return fail(CIE_ERR_UNSUPPORTED, "hidden_size %d must be a multiple of 64 up to %d",
                hidden_size, kMaxK);
  if (hidden_stride < hidden_size || weight_stride < hidden_size ||
      (logits && logits_stride < vocab))
    return fail(CIE_ERR_INVALID_ARGUMENT, "row strides overlap");
  if (!aligned16(hidden) || !aligned16(weight) || (hidden_stride % 8) || (weight_stride % 8))
    return fail(CIE_ERR_ALIGNMENT, "hidden / weight rows must be 16-byte aligned");
  const int dev = current_device();
  const size_t need = cie_lm_head_argmax_workspace_bytes(batch, vocab, dev);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(CIE_ERR_WORKSPACE, "lm_head argmax needs %zu workspace bytes", need);
  if (!aligned16(workspace)) return fail(CIE_ERR_ALIGNMENT, "workspace must be 16-byte aligned");

  CUtensorMap tm_w;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(hidden_size), static_cast<uint64_t>(vocab), 1};
    const uint64_t strides[2] = {static_cast<uint64_t>(weight_stride) * 2,
                                 static_cast<uint64_t>(weight_stride) * 2 * vocab};
    const uint32_t box[3] = {kKBlock, kChunkRows, 1};
    const int st = encode_tensor_map(&tm_w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                                     const_cast<void*>(weight), dims, strides, box,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != CIE_OK) return st;
  }
  int st = ensure_smem_attribute(reinterpret_cast<const void*>(&lm_head_argmax_kernel), kSmemBytes,
                                 9);
  if (st != CIE_OK) return st;
  const int grid = grid_for(vocab, dev);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int b0 = 0; b0 < batch; b0 += kMaxN) {
    const int rows = min(kMaxN, batch - b0);
    const int n_pad = (rows + 15) / 16 * 16;
    // this slice's hidden rows; rows past the batch read as zeros (TMA bounds)
    CUtensorMap tm_h;
    {
      const __half* h0 = static_cast<const __half*>(hidden) + static_cast<int64_t>(b0) * hidden_stride;
      const uint64_t dims[3] = {static_cast<uint64_t>(hidden_size), static_cast<uint64_t>(rows), 1};
      const uint64_t strides[2] = {static_cast<uint64_t>(hidden_stride) * 2,
                                   static_cast<uint64_t>(hidden_stride) * 2 * rows};
      const uint32_t box[3] = {kKBlock, static_cast<uint32_t>(n_pad), 1};
      st = encode_tensor_map(&tm_h, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(h0),
                             dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
      if (st != CIE_OK) return st;
    }
    Params p;
    p.partial = static_cast<int64_t*>(workspace) +
                static_cast<int64_t>(b0 / kMaxN) * grid * kMaxN;
    p.logits = logits ? static_cast<__half*>(logits) + static_cast<int64_t>(b0) * logits_stride
                      : nullptr;
    p.logits_stride = logits_stride;
    p.vocab = vocab;
    p.rows = rows;
    p.n_pad = n_pad;
    p.k_blocks = hidden_size / kKBlock;
    p.n_chunks = static_cast<int>((vocab + kChunkRows - 1) / kChunkRows);
    lm_head_argmax_kernel<<<grid, kThreads, kSmemBytes, s>>>(tm_w, tm_h, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "lm_head launch: %s", cudaGetErrorString(e));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows);
    cfg.blockDim = dim3(32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, lm_head_final_kernel, static_cast<const int64_t*>(p.partial),
                           grid, n_pad, tokens + b0);
    if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "lm_head final launch: %s", cudaGetErrorString(e));
  }
  return CIE_OK;
}

}  // extern "C"
