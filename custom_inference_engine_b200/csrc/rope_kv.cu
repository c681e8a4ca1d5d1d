// Rotary embedding of q and k fused with the KV-page scatter: one launch per
// layer instead of the reference's RoPE element-wise ops plus the K/V write.
//
// Replaces, inside TritonQwen2Attention.forward (attn/core.py:193-206 of the
// reference): the split of the fused QKV projection, apply_rotary_pos_emb
// (transformers Qwen2: x * cos + rotate_half(x) * sin with rotate_half(x) =
// cat(-x[32:], x[:32])), and KVStorage.decode_update / mixed_update
// (kv_cache/storage.py:62-122). The rotation is computed with the same fp16
// operations in the same order (product, product, sum, each rounded to fp16),
// so q and the written k are bit-identical to the reference's.
//
// Thread = (token, row, c): rows 0..Hq-1 are q heads, Hq..Hq+Hkv-1 k heads,
// then Hkv v heads; c in 0..3 owns the 8-element chunks c and c + 4 of the
// 64-wide row, which are exactly the partners of the rotation.
#include "cie_common.cuh"
#include "cie_host.h"

namespace cie {
namespace rope {

constexpr int kD = 64;
constexpr int kHalfChunks = 4;  // chunk pairs per row

struct Args {
  const __half* qkv;      // (T, (Hq + 2 Hkv) * D), row stride qkv_tok
  int64_t qkv_tok;
  const __half* cos;      // (T, D), row stride cs_tok
  const __half* sin;
  int64_t cs_tok;
  __half* q_out;          // (T, Hq, D) contiguous
  __half* k_cache;        // (n_pages, Hkv, page, D)
  __half* v_cache;
  int64_t page_stride, head_stride;
  // decode addressing (pages == nullptr) or mixed addressing
  const int64_t* lens;
  const int64_t* slot_ids;
  BlockTable block_table;
  const int64_t* pages;
  const int64_t* offsets;
  int64_t num_tokens;
  int hq, hkv, page_size;
  int64_t n_pages, n_slots, bt_stride;
};

__device__ __forceinline__ uint4 ld16(const __half* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// out = x * c + rot * s, every operation rounded to fp16 (rot already negated
// where rotate_half negates)
__device__ __forceinline__ uint4 rope8(uint4 x, uint4 rot, uint4 c, uint4 s) {
  uint4 r;
  const __half2* xh = reinterpret_cast<const __half2*>(&x);
  const __half2* rh = reinterpret_cast<const __half2*>(&rot);
  const __half2* ch = reinterpret_cast<const __half2*>(&c);
  const __half2* sh = reinterpret_cast<const __half2*>(&s);
  __half2* oh = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int e = 0; e < 4; ++e)  // _rn: no contraction into a fused multiply-add
    oh[e] = __hadd2_rn(__hmul2_rn(xh[e], ch[e]), __hmul2_rn(rh[e], sh[e]));
  return r;
}

__device__ __forceinline__ uint4 neg8(uint4 x) {
  uint4 r;
  const __half2* xh = reinterpret_cast<const __half2*>(&x);
  __half2* oh = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int e = 0; e < 4; ++e) oh[e] = __hneg2(xh[e]);
  return r;
}

// Work items of one launch: one per (token, row, chunk pair).
__host__ __device__ __forceinline__ int64_t work_items(const Args& a) {
  return a.num_tokens * (a.hq + 2 * a.hkv) * kHalfChunks;
}

// Work item `idx` (< work_items(a)): the rotation of one chunk pair of a q or k
// row, or the copy of a v row's chunk pair, to its destination.
__device__ __forceinline__ void rope_kv_item(const Args& a, int64_t idx) {
  const int rows = a.hq + 2 * a.hkv;
  const int64_t per_tok = static_cast<int64_t>(rows) * kHalfChunks;
  const int64_t t = idx / per_tok;
  const int row = static_cast<int>((idx % per_tok) / kHalfChunks);
  const int c = static_cast<int>(idx % kHalfChunks);
  const __half* src = a.qkv + t * a.qkv_tok + static_cast<int64_t>(row) * kD;
  const uint4 x1 = ld16(src + c * 8);        // elements [8c, 8c + 8)
  const uint4 x2 = ld16(src + 32 + c * 8);   // elements [32 + 8c, 32 + 8c + 8)

  __half* dst;
  if (row < a.hq) {
    dst = a.q_out + (t * a.hq + row) * kD;
  } else {
    // the slot / page this token's K and V rows go to
    int64_t page, off;
    if (a.pages == nullptr) {
      const int64_t slot = a.slot_ids[t];
      if (slot < 0 || slot >= a.n_slots) {
        if (row == a.hq && c == 0) raise_error(CIE_DEVERR_BAD_SLOT);
        return;
      }
      const int64_t pos = a.lens[slot];
      if (pos < 0 || pos / a.page_size >= a.bt_stride) {
        if (row == a.hq && c == 0) raise_error(CIE_DEVERR_BAD_LENGTH);
        return;
      }
      page = a.block_table.at(slot * a.bt_stride + pos / a.page_size);
      off = pos % a.page_size;
    } else {
      page = a.pages[t];
      off = a.offsets[t];
      if (off < 0 || off >= a.page_size) {
        if (row == a.hq && c == 0) raise_error(CIE_DEVERR_BAD_OFFSET);
        return;
      }
    }
    if (page < 0 || page >= a.n_pages) {
      if (row == a.hq && c == 0) raise_error(CIE_DEVERR_BAD_PAGE);
      return;
    }
    const bool is_v = row >= a.hq + a.hkv;
    const int h = is_v ? row - a.hq - a.hkv : row - a.hq;
    dst = (is_v ? a.v_cache : a.k_cache) + page * a.page_stride + h * a.head_stride + off * kD;
    if (is_v) {  // V is copied as is
      *reinterpret_cast<uint4*>(dst + c * 8) = x1;
      *reinterpret_cast<uint4*>(dst + 32 + c * 8) = x2;
      return;
    }
  }
  const __half* cs = a.cos + t * a.cs_tok;
  const __half* sn = a.sin + t * a.cs_tok;
  // rotate_half: first half gets -x2, second half gets x1
  *reinterpret_cast<uint4*>(dst + c * 8) = rope8(x1, neg8(x2), ld16(cs + c * 8), ld16(sn + c * 8));
  *reinterpret_cast<uint4*>(dst + 32 + c * 8) =
      rope8(x2, x1, ld16(cs + 32 + c * 8), ld16(sn + 32 + c * 8));
}

__global__ void rope_kv_kernel(const Args a) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx < work_items(a)) rope_kv_item(a, idx);
}

// Host-side checks of one launch's arguments (CIE_OK or a status).
int check(const Args& a, int head_dim) {
  if (a.num_tokens < 0) return fail(CIE_ERR_INVALID_ARGUMENT, "negative token count");
  if (a.num_tokens == 0) return CIE_OK;
  if (!a.qkv || !a.cos || !a.sin || !a.q_out || !a.k_cache || !a.v_cache)
    return fail(CIE_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (head_dim != kD) return fail(CIE_ERR_UNSUPPORTED, "head_dim %d (supported: 64)", head_dim);
  if (a.hq < 1 || a.hkv < 1 || a.page_size < 1 || a.n_pages < 1)
    return fail(CIE_ERR_INVALID_ARGUMENT, "heads / page_size / n_pages must be >= 1");
  if (a.head_stride < static_cast<int64_t>(a.page_size) * kD ||
      a.page_stride < a.head_stride * a.hkv)
    return fail(CIE_ERR_INVALID_ARGUMENT, "overlapping cache strides");
  if (a.qkv_tok < static_cast<int64_t>(a.hq + 2 * a.hkv) * kD || a.cs_tok < kD)
    return fail(CIE_ERR_INVALID_ARGUMENT, "qkv / cos / sin rows overlap");
  if ((a.qkv_tok % 8) || (a.cs_tok % 8) || (a.page_stride % 8) || (a.head_stride % 8) ||
      !aligned16(a.qkv) || !aligned16(a.cos) || !aligned16(a.sin) || !aligned16(a.q_out) ||
      !aligned16(a.k_cache) || !aligned16(a.v_cache))
    return fail(CIE_ERR_ALIGNMENT, "all rows must start on 16-byte boundaries");
  return CIE_OK;
}

int launch(Args a, int head_dim, cie_stream_t stream) {
  if (a.num_tokens < 0) return fail(CIE_ERR_INVALID_ARGUMENT, "negative token count");
  if (a.num_tokens == 0) return CIE_OK;
  const int st = check(a, head_dim);
  if (st != CIE_OK) return st;
  const int64_t threads = work_items(a);
  const int block = 256;
  const int64_t grid = (threads + block - 1) / block;
  if (grid > 0x7fffffff) return fail(CIE_ERR_OVERFLOW, "too many tokens");
  rope_kv_kernel<<<static_cast<unsigned>(grid), block, 0,
                   reinterpret_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "rope_kv launch: %s", cudaGetErrorString(e));
  return CIE_OK;
}

}  // namespace rope
}  // namespace cie

extern "C" {

static int rope_kv_decode_update(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                                 const void* sin, int64_t cs_tok_stride, void* q_out,
                                 void* k_cache, void* v_cache, const int64_t* lens,
                                 const int64_t* slot_ids, cie::BlockTable block_table, int batch,
                                 int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                                 int64_t n_pages, int64_t n_slots, int64_t bt_stride,
                                 int64_t cache_page_stride, int64_t cache_head_stride,
                                 cie_stream_t stream) {
  using namespace cie;
  if (batch > 0 && (!lens || !slot_ids || !block_table.ptr))
    return fail(CIE_ERR_INVALID_ARGUMENT, "null lens / slot_ids / block_table");
  if (batch > 0 && (n_slots < 1 || bt_stride < 1))
    return fail(CIE_ERR_INVALID_ARGUMENT, "n_slots / bt_stride must be >= 1");
  rope::Args a{};
  a.qkv = static_cast<const __half*>(qkv);
  a.qkv_tok = qkv_tok_stride;
  a.cos = static_cast<const __half*>(cos);
  a.sin = static_cast<const __half*>(sin);
  a.cs_tok = cs_tok_stride;
  a.q_out = static_cast<__half*>(q_out);
  a.k_cache = static_cast<__half*>(k_cache);
  a.v_cache = static_cast<__half*>(v_cache);
  a.page_stride = cache_page_stride;
  a.head_stride = cache_head_stride;
  a.lens = lens;
  a.slot_ids = slot_ids;
  a.block_table = block_table;
  a.num_tokens = batch;
  a.hq = num_q_heads;
  a.hkv = num_kv_heads;
  a.page_size = page_size;
  a.n_pages = n_pages;
  a.n_slots = n_slots;
  a.bt_stride = bt_stride;
  return rope::launch(a, head_dim, stream);
}

int cie_rope_kv_decode_update(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                              const void* sin, int64_t cs_tok_stride, void* q_out,
                              void* k_cache, void* v_cache, const int64_t* lens,
                              const int64_t* slot_ids, const int64_t* block_table, int batch,
                              int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                              int64_t n_pages, int64_t n_slots, int64_t bt_stride,
                              int64_t cache_page_stride, int64_t cache_head_stride,
                              cie_stream_t stream) {
  return rope_kv_decode_update(qkv, qkv_tok_stride, cos, sin, cs_tok_stride, q_out, k_cache,
                               v_cache, lens, slot_ids, cie::BlockTable{block_table, 1}, batch,
                               num_q_heads, num_kv_heads, head_dim, page_size, n_pages, n_slots,
                               bt_stride, cache_page_stride, cache_head_stride, stream);
}

int cie_rope_kv_decode_update_bt32(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                                   const void* sin, int64_t cs_tok_stride, void* q_out,
                                   void* k_cache, void* v_cache, const int64_t* lens,
                                   const int64_t* slot_ids, const int32_t* block_table, int batch,
                                   int num_q_heads, int num_kv_heads, int head_dim,
                                   int page_size, int64_t n_pages, int64_t n_slots,
                                   int64_t bt_stride, int64_t cache_page_stride,
                                   int64_t cache_head_stride, cie_stream_t stream) {
  return rope_kv_decode_update(qkv, qkv_tok_stride, cos, sin, cs_tok_stride, q_out, k_cache,
                               v_cache, lens, slot_ids, cie::BlockTable{block_table, 0}, batch,
                               num_q_heads, num_kv_heads, head_dim, page_size, n_pages, n_slots,
                               bt_stride, cache_page_stride, cache_head_stride, stream);
}

int cie_rope_kv_mixed_update(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                             const void* sin, int64_t cs_tok_stride, void* q_out, void* k_cache,
                             void* v_cache, const int64_t* pages, const int64_t* offsets,
                             int64_t num_tokens, int num_q_heads, int num_kv_heads, int head_dim,
                             int page_size, int64_t n_pages, int64_t cache_page_stride,
                             int64_t cache_head_stride, cie_stream_t stream) {
  using namespace cie;
  if (num_tokens > 0 && (!pages || !offsets))
    return fail(CIE_ERR_INVALID_ARGUMENT, "null pages / offsets");
  rope::Args a{};
  a.qkv = static_cast<const __half*>(qkv);
  a.qkv_tok = qkv_tok_stride;
  a.cos = static_cast<const __half*>(cos);
  a.sin = static_cast<const __half*>(sin);
  a.cs_tok = cs_tok_stride;
  a.q_out = static_cast<__half*>(q_out);
  a.k_cache = static_cast<__half*>(k_cache);
  a.v_cache = static_cast<__half*>(v_cache);
  a.page_stride = cache_page_stride;
  a.head_stride = cache_head_stride;
  a.pages = pages;
  a.offsets = offsets;
  a.num_tokens = num_tokens;
  a.hq = num_q_heads;
  a.hkv = num_kv_heads;
  a.page_size = page_size;
  a.n_pages = n_pages;
  return rope::launch(a, head_dim, stream);
}

}  // extern "C"
