// KV-page scatter: writes the new tokens' K and V rows into the paged pool.
//
// Replaces KVStorage.decode_update / mixed_update (kv_cache/storage.py:62-122),
// which the reference runs as torch index_put (fused by inductor into its RoPE
// kernel). One thread moves one 16-byte chunk (8 fp16 of a 64-wide row); K and
// V, every kv head and every token go out in a single launch. The copy is
// bit-exact. Source rows may be strided views (the value projection is a
// slice of the fused QKV output, token stride 18 * 64 elements).
#include "cie_common.cuh"
#include "cie_host.h"

namespace cie {
namespace kvupd {

constexpr int kChunkHalves = 8;  // 16 bytes

struct Src {
  const __half* k;
  const __half* v;
  int64_t k_tok, k_head, v_tok, v_head;
};

template <bool kVec>
__device__ __forceinline__ void copy_row_chunk(__half* dst, const __half* src) {
  if (kVec) {
    *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
  } else {
#pragma unroll
    for (int e = 0; e < kChunkHalves; ++e) dst[e] = src[e];
  }
}

// thread -> (token, K|V, kv head, chunk)
template <bool kVec>
__global__ void decode_update_kernel(__half* __restrict__ k_cache, __half* __restrict__ v_cache,
                                     const int64_t* __restrict__ lens,
                                     const int64_t* __restrict__ slot_ids,
                                     BlockTable block_table, Src src, int batch,
                                     int hkv, int head_dim, int page_size, int64_t n_pages,
                                     int64_t n_slots, int64_t bt_stride, int64_t page_stride,
                                     int64_t head_stride) {
  const int chunks = head_dim / kChunkHalves;
  const int64_t total = static_cast<int64_t>(batch) * 2 * hkv * chunks;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int c = static_cast<int>(idx % chunks);
  const int h = static_cast<int>((idx / chunks) % hkv);
  const int which = static_cast<int>((idx / (chunks * hkv)) % 2);
  const int b = static_cast<int>(idx / (chunks * hkv * 2));
  const int64_t slot = slot_ids[b];
  if (slot < 0 || slot >= n_slots) {
    raise_error(CIE_DEVERR_BAD_SLOT);
    return;
  }
  const int64_t pos = lens[slot];
  if (pos < 0 || pos / page_size >= bt_stride) {
    raise_error(CIE_DEVERR_BAD_LENGTH);
    return;
  }
  const int64_t page = block_table.at(slot * bt_stride + pos / page_size);
  if (page < 0 || page >= n_pages) {
    raise_error(CIE_DEVERR_BAD_PAGE);
    return;
  }
  const int64_t off = pos % page_size;
  __half* cache = which ? v_cache : k_cache;
  const __half* s = which ? src.v + b * src.v_tok + h * src.v_head
                          : src.k + b * src.k_tok + h * src.k_head;
  __half* d = cache + page * page_stride + h * head_stride + off * head_dim;
  copy_row_chunk<kVec>(d + c * kChunkHalves, s + c * kChunkHalves);
}

template <bool kVec>
__global__ void mixed_update_kernel(__half* __restrict__ k_cache, __half* __restrict__ v_cache,
                                    const int64_t* __restrict__ pages,
                                    const int64_t* __restrict__ offsets, Src src,
                                    int64_t num_tokens, int hkv, int head_dim, int page_size,
                                    int64_t n_pages, int64_t page_stride, int64_t head_stride) {
  const int chunks = head_dim / kChunkHalves;
  const int64_t total = num_tokens * 2 * hkv * chunks;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int c = static_cast<int>(idx % chunks);
  const int h = static_cast<int>((idx / chunks) % hkv);
  const int which = static_cast<int>((idx / (chunks * hkv)) % 2);
  const int64_t t = idx / (chunks * hkv * 2);
  const int64_t page = pages[t];
  const int64_t off = offsets[t];
  if (page < 0 || page >= n_pages) {
    raise_error(CIE_DEVERR_BAD_PAGE);
    return;
  }
  if (off < 0 || off >= page_size) {
    raise_error(CIE_DEVERR_BAD_OFFSET);
    return;
  }
  __half* cache = which ? v_cache : k_cache;
  const __half* s = which ? src.v + t * src.v_tok + h * src.v_head
                          : src.k + t * src.k_tok + h * src.k_head;
  __half* d = cache + page * page_stride + h * head_stride + off * head_dim;
  copy_row_chunk<kVec>(d + c * kChunkHalves, s + c * kChunkHalves);
}

int check_common(void* k_cache, void* v_cache, const void* k_new, const void* v_new,
                 int num_kv_heads, int head_dim, int page_size, int64_t n_pages,
                 int64_t page_stride, int64_t head_stride) {
  if (!k_cache || !v_cache || !k_new || !v_new)
    return fail(CIE_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (num_kv_heads < 1 || head_dim < 8 || head_dim % 8 || page_size < 1 || n_pages < 1)
    return fail(CIE_ERR_UNSUPPORTED, "num_kv_heads %d, head_dim %d, page_size %d", num_kv_heads,
                head_dim, page_size);
  if (head_stride < static_cast<int64_t>(page_size) * head_dim ||
      page_stride < head_stride * num_kv_heads)
    return fail(CIE_ERR_INVALID_ARGUMENT, "overlapping cache strides");
  return CIE_OK;
}

bool vec_ok(const void* k_cache, const void* v_cache, const Src& s, int64_t page_stride,
            int64_t head_stride) {
  return aligned16(k_cache) && aligned16(v_cache) && aligned16(s.k) && aligned16(s.v) &&
         (page_stride % 8 == 0) && (head_stride % 8 == 0) && (s.k_tok % 8 == 0) &&
         (s.k_head % 8 == 0) && (s.v_tok % 8 == 0) && (s.v_head % 8 == 0);
}

}  // namespace kvupd
}  // namespace cie

extern "C" {

static int kv_decode_update(void* k_cache, void* v_cache, const int64_t* lens,
                            const int64_t* slot_ids, cie::BlockTable block_table,
                            const void* k_new, const void* v_new, int batch, int num_kv_heads,
                            int head_dim, int page_size, int64_t n_pages, int64_t n_slots,
                            int64_t bt_stride, int64_t cache_page_stride,
                            int64_t cache_head_stride, int64_t k_tok_stride,
                            int64_t k_head_stride, int64_t v_tok_stride, int64_t v_head_stride,
                            cie_stream_t stream) {
  using namespace cie;
  using namespace cie::kvupd;
  if (batch < 0) return fail(CIE_ERR_INVALID_ARGUMENT, "batch < 0");
  if (batch == 0) return CIE_OK;
  int st = check_common(k_cache, v_cache, k_new, v_new, num_kv_heads, head_dim, page_size, n_pages,
                        cache_page_stride, cache_head_stride);
  if (st != CIE_OK) return st;
  if (!lens || !slot_ids || !block_table.ptr)
    return fail(CIE_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (n_slots < 1 || bt_stride < 1) return fail(CIE_ERR_INVALID_ARGUMENT, "n_slots / bt_stride");
  Src src{static_cast<const __half*>(k_new), static_cast<const __half*>(v_new), k_tok_stride,
          k_head_stride, v_tok_stride, v_head_stride};
  const int64_t total = static_cast<int64_t>(batch) * 2 * num_kv_heads * (head_dim / 8);
  const int threads = 256;
  const int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 0x7fffffff) return fail(CIE_ERR_OVERFLOW, "too many tokens");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto* kc = static_cast<__half*>(k_cache);
  auto* vc = static_cast<__half*>(v_cache);
  if (vec_ok(k_cache, v_cache, src, cache_page_stride, cache_head_stride))
    decode_update_kernel<true><<<static_cast<unsigned>(blocks), threads, 0, s>>>(
        kc, vc, lens, slot_ids, block_table, src, batch, num_kv_heads, head_dim, page_size,
        n_pages, n_slots, bt_stride, cache_page_stride, cache_head_stride);
  else
    decode_update_kernel<false><<<static_cast<unsigned>(blocks), threads, 0, s>>>(
        kc, vc, lens, slot_ids, block_table, src, batch, num_kv_heads, head_dim, page_size,
        n_pages, n_slots, bt_stride, cache_page_stride, cache_head_stride);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "decode_update launch: %s", cudaGetErrorString(e));
  return CIE_OK;
}

int cie_kv_decode_update(void* k_cache, void* v_cache, const int64_t* lens,
                         const int64_t* slot_ids, const int64_t* block_table, const void* k_new,
                         const void* v_new, int batch, int num_kv_heads, int head_dim,
                         int page_size, int64_t n_pages, int64_t n_slots, int64_t bt_stride,
                         int64_t cache_page_stride, int64_t cache_head_stride,
                         int64_t k_tok_stride, int64_t k_head_stride, int64_t v_tok_stride,
                         int64_t v_head_stride, cie_stream_t stream) {
  return kv_decode_update(k_cache, v_cache, lens, slot_ids, cie::BlockTable{block_table, 1},
                          k_new, v_new, batch, num_kv_heads, head_dim, page_size, n_pages,
                          n_slots, bt_stride, cache_page_stride, cache_head_stride, k_tok_stride,
                          k_head_stride, v_tok_stride, v_head_stride, stream);
}

int cie_kv_decode_update_bt32(void* k_cache, void* v_cache, const int64_t* lens,
                              const int64_t* slot_ids, const int32_t* block_table,
                              const void* k_new, const void* v_new, int batch, int num_kv_heads,
                              int head_dim, int page_size, int64_t n_pages, int64_t n_slots,
                              int64_t bt_stride, int64_t cache_page_stride,
                              int64_t cache_head_stride, int64_t k_tok_stride,
                              int64_t k_head_stride, int64_t v_tok_stride,
                              int64_t v_head_stride, cie_stream_t stream) {
  return kv_decode_update(k_cache, v_cache, lens, slot_ids, cie::BlockTable{block_table, 0},
                          k_new, v_new, batch, num_kv_heads, head_dim, page_size, n_pages,
                          n_slots, bt_stride, cache_page_stride, cache_head_stride, k_tok_stride,
                          k_head_stride, v_tok_stride, v_head_stride, stream);
}

int cie_kv_mixed_update(void* k_cache, void* v_cache, const int64_t* pages,
                        const int64_t* offsets, const void* k_new, const void* v_new,
                        int64_t num_tokens, int num_kv_heads, int head_dim, int page_size,
                        int64_t n_pages, int64_t cache_page_stride, int64_t cache_head_stride,
                        int64_t k_tok_stride, int64_t k_head_stride, int64_t v_tok_stride,
                        int64_t v_head_stride, cie_stream_t stream) {
  using namespace cie;
  using namespace cie::kvupd;
  if (num_tokens < 0) return fail(CIE_ERR_INVALID_ARGUMENT, "num_tokens < 0");
  if (num_tokens == 0) return CIE_OK;
  int st = check_common(k_cache, v_cache, k_new, v_new, num_kv_heads, head_dim, page_size, n_pages,
                        cache_page_stride, cache_head_stride);
  if (st != CIE_OK) return st;
  if (!pages || !offsets) return fail(CIE_ERR_INVALID_ARGUMENT, "null pointer argument");
  Src src{static_cast<const __half*>(k_new), static_cast<const __half*>(v_new), k_tok_stride,
          k_head_stride, v_tok_stride, v_head_stride};
  const int64_t total = num_tokens * 2 * num_kv_heads * (head_dim / 8);
  const int threads = 256;
  const int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 0x7fffffff) return fail(CIE_ERR_OVERFLOW, "too many tokens");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto* kc = static_cast<__half*>(k_cache);
  auto* vc = static_cast<__half*>(v_cache);
  if (vec_ok(k_cache, v_cache, src, cache_page_stride, cache_head_stride))
    mixed_update_kernel<true><<<static_cast<unsigned>(blocks), threads, 0, s>>>(
        kc, vc, pages, offsets, src, num_tokens, num_kv_heads, head_dim, page_size, n_pages,
        cache_page_stride, cache_head_stride);
  else
    mixed_update_kernel<false><<<static_cast<unsigned>(blocks), threads, 0, s>>>(
        kc, vc, pages, offsets, src, num_tokens, num_kv_heads, head_dim, page_size, n_pages,
        cache_page_stride, cache_head_stride);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "mixed_update launch: %s", cudaGetErrorString(e));
  return CIE_OK;
}

}  // extern "C"
