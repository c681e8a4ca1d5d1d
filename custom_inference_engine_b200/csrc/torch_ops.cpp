// Torch custom ops over the C ABI of libcie_attention.so.
//
// Schemas match the reference's triton_op registrations (attn/core.py:119-137)
// so callers, Dynamo graphs and the piecewise splitter (which matches
// torch.ops.inference.gqa_mixed_attention.default and reads its kv_lens
// kwarg) see the same ops. Checks mirror the reference host asserts
// (attn/core.py:18-34, 76-86) and raise RuntimeError. Outputs and the split
// workspace come from the caching allocator, so the ops are safe inside CUDA
// graph capture; nothing here synchronises with the host.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <algorithm>
#include <vector>

#include "cie_attention.h"
#include "cie_model_ops.h"

namespace {

void check_status(int st, const char* what) {
  TORCH_CHECK(st == CIE_OK, what, ": ", cie_status_string(st), ": ", cie_last_error_message());
}

void check_i64(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.scalar_type() == at::kLong, name, " must be int64");
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

// The block table holds int64 page ids (the reference's layout) or int32 ones
// (the *_bt32 entry points); the ops take either.
void check_table(const at::Tensor& t) {
  TORCH_CHECK(t.scalar_type() == at::kLong || t.scalar_type() == at::kInt,
              "block_table must be int64 or int32");
  TORCH_CHECK(t.is_cuda(), "block_table must be a CUDA tensor");
}

// Calls `call(fn64, int64 table)` or `call(fn32, int32 table)` by the table's dtype.
template <typename Call, typename F64, typename F32>
int with_table(const at::Tensor& t, Call&& call, F64 fn64, F32 fn32) {
  return t.scalar_type() == at::kInt ? call(fn32, t.data_ptr<int32_t>())
                                     : call(fn64, t.data_ptr<int64_t>());
}

void check_kv_pool(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "q, k, v must be CUDA tensors");
  TORCH_CHECK(q.scalar_type() == at::kHalf && k.scalar_type() == at::kHalf &&
                  v.scalar_type() == at::kHalf,
              "q, k, v must be float16");
  TORCH_CHECK(q.dim() == 4 && q.size(0) == 1, "q must be (1, T, H_q, D)");
  TORCH_CHECK(k.dim() == 4, "k must be (n_pages, H_kv, page_size, D)");
  TORCH_CHECK(k.sizes() == v.sizes(), "k and v shapes differ");
  TORCH_CHECK(q.size(2) % k.size(1) == 0, "H_q must be a multiple of H_kv");
  TORCH_CHECK(k.size(3) == q.size(3), "head_dim mismatch between q and k");
  TORCH_CHECK(q.is_contiguous(), "q must be contiguous");
  TORCH_CHECK(k.strides() == v.strides() && k.stride(3) == 1 && k.stride(2) == k.size(3),
              "k and v must share strides with unit inner stride and row stride head_dim");
}

at::Tensor decode_impl(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                       const at::Tensor& lens, const at::Tensor& slot_ids,
                       const at::Tensor& block_table, int64_t num_splits) {
  check_kv_pool(q, k, v);
  check_i64(lens, "lens");
  check_i64(slot_ids, "slot_ids");
  check_table(block_table);
  const int64_t B = slot_ids.size(0);
  TORCH_CHECK(lens.dim() == 1 && lens.size(0) == B, "lens must be (B,)");
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(1) == k.size(0),
              "block_table must be (n_slots, n_pages)");
  TORCH_CHECK(block_table.stride(1) == 1, "block_table rows must be contiguous");
  TORCH_CHECK(q.size(1) == B, "q must hold one token per sequence");
  TORCH_CHECK(lens.is_contiguous() && slot_ids.is_contiguous(), "lens / slot_ids must be contiguous");
  c10::cuda::CUDAGuard guard(q.device());
  at::Tensor o = at::empty_like(q);
  if (B == 0) return o;
  int S = static_cast<int>(num_splits);
  if (S <= 0) S = cie_decode_default_splits(static_cast<int>(B), q.get_device());
  const size_t ws_bytes =
      cie_decode_workspace_bytes(static_cast<int>(B), static_cast<int>(q.size(2)),
                                 static_cast<int>(q.size(3)), S);
  at::Tensor ws;
  if (ws_bytes > 0)
    ws = at::empty({static_cast<int64_t>(ws_bytes / sizeof(float))},
                   q.options().dtype(at::kFloat));
  const int st = with_table(
      block_table,
      [&](auto fn, auto* table) {
        return fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr<int64_t>(),
          slot_ids.data_ptr<int64_t>(), table, o.data_ptr(),
          ws_bytes > 0 ? ws.data_ptr() : nullptr, ws_bytes, static_cast<int>(B),
          static_cast<int>(q.size(2)), static_cast<int>(k.size(1)), static_cast<int>(q.size(3)),
          static_cast<int>(k.size(2)), k.size(0), block_table.size(0), block_table.stride(0),
          k.stride(0), k.stride(1), S,
          reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
      },
      cie_decode_attention, cie_decode_attention_bt32);
  check_status(st, "gqa_decode_attention");
  return o;
}

at::Tensor gqa_decode_attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                const at::Tensor& lens, const at::Tensor& slot_ids,
                                const at::Tensor& block_table) {
  return decode_impl(q, k, v, lens, slot_ids, block_table, 0);
}

at::Tensor gqa_decode_attention_splits(const at::Tensor& q, const at::Tensor& k,
                                       const at::Tensor& v, const at::Tensor& lens,
                                       const at::Tensor& slot_ids, const at::Tensor& block_table,
                                       int64_t num_splits) {
  return decode_impl(q, k, v, lens, slot_ids, block_table, num_splits);
}

at::Tensor gqa_mixed_attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                               c10::SymInt max_seqlen_sym, const at::Tensor& cu_seqlens,
                               const at::Tensor& kv_lens, const at::Tensor& slot_ids,
                               const at::Tensor& block_table) {
  const int64_t max_seqlen = max_seqlen_sym.expect_int();
  check_kv_pool(q, k, v);
  TORCH_CHECK(k.is_contiguous() && v.is_contiguous(), "k and v must be contiguous");
  check_i64(cu_seqlens, "cu_seqlens");
  check_i64(kv_lens, "kv_lens");
  check_i64(slot_ids, "slot_ids");
  check_table(block_table);
  const int64_t B = slot_ids.size(0);
  TORCH_CHECK(kv_lens.dim() == 1 && kv_lens.size(0) == B, "kv_lens must be (B,)");
  TORCH_CHECK(cu_seqlens.dim() == 1 && cu_seqlens.size(0) == B + 1, "cu_seqlens must be (B+1,)");
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(1) == k.size(0),
              "block_table must be (n_slots, n_pages)");
  TORCH_CHECK(block_table.stride(1) == 1, "block_table rows must be contiguous");
  TORCH_CHECK(cu_seqlens.is_contiguous() && kv_lens.is_contiguous() && slot_ids.is_contiguous(),
              "cu_seqlens / kv_lens / slot_ids must be contiguous");
  c10::cuda::CUDAGuard guard(q.device());
  at::Tensor o = at::empty_like(q);
  // the work plan and the partials of split tile pairs (automatic plan)
  const size_t ws_bytes = cie_mixed_workspace_bytes(static_cast<int>(B), q.size(1),
                                                    static_cast<int>(k.size(1)), 0,
                                                    q.get_device());
  at::Tensor ws = at::empty({static_cast<int64_t>((ws_bytes + 3) / sizeof(float))},
                            q.options().dtype(at::kFloat));
  const int st = with_table(
      block_table,
      [&](auto fn, auto* table) {
        return fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), max_seqlen, cu_seqlens.data_ptr<int64_t>(),
          kv_lens.data_ptr<int64_t>(), slot_ids.data_ptr<int64_t>(), table,
          o.data_ptr(), ws.data_ptr(), ws_bytes, static_cast<int>(B),
          q.size(1), static_cast<int>(q.size(2)), static_cast<int>(k.size(1)),
          static_cast<int>(q.size(3)), static_cast<int>(k.size(2)), k.size(0), block_table.size(0),
          block_table.stride(0), k.stride(0), k.stride(1), 0,
          reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
      },
      cie_mixed_attention, cie_mixed_attention_bt32);
  check_status(st, "gqa_mixed_attention");
  return o;
}

void check_update_src(const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& kn,
                      const at::Tensor& vn) {
  TORCH_CHECK(kc.is_cuda() && vc.is_cuda() && kn.is_cuda() && vn.is_cuda(),
              "caches and new rows must be CUDA tensors");
  TORCH_CHECK(kc.scalar_type() == at::kHalf && vc.scalar_type() == at::kHalf &&
                  kn.scalar_type() == at::kHalf && vn.scalar_type() == at::kHalf,
              "caches and new rows must be float16");
  TORCH_CHECK(kc.dim() == 4 && kc.sizes() == vc.sizes() && kc.strides() == vc.strides(),
              "k_cache / v_cache must be (n_pages, H_kv, page_size, D) with equal strides");
  TORCH_CHECK(kc.stride(3) == 1 && kc.stride(2) == kc.size(3), "cache rows must be dense");
  TORCH_CHECK(kn.dim() == 4 && kn.size(0) == 1 && kn.size(2) == kc.size(1) &&
                  kn.size(3) == kc.size(3) && kn.sizes() == vn.sizes(),
              "new rows must be (1, T, H_kv, D)");
  TORCH_CHECK(kn.stride(3) == 1 && vn.stride(3) == 1, "new rows need unit inner stride");
}

void kv_decode_update(at::Tensor& k_cache, at::Tensor& v_cache, const at::Tensor& lens,
                      const at::Tensor& slot_ids, const at::Tensor& block_table,
                      const at::Tensor& k_new, const at::Tensor& v_new) {
  check_update_src(k_cache, v_cache, k_new, v_new);
  check_i64(lens, "lens");
  check_i64(slot_ids, "slot_ids");
  check_table(block_table);
  TORCH_CHECK(block_table.dim() == 2 && block_table.stride(1) == 1, "block_table must be 2-D");
  TORCH_CHECK(k_new.size(1) == slot_ids.size(0), "one new row per slot id");
  TORCH_CHECK(lens.is_contiguous() && slot_ids.is_contiguous(), "lens / slot_ids contiguous");
  c10::cuda::CUDAGuard guard(k_cache.device());
  const int st = with_table(
      block_table,
      [&](auto fn, auto* table) {
        return fn(k_cache.data_ptr(), v_cache.data_ptr(), lens.data_ptr<int64_t>(),
          slot_ids.data_ptr<int64_t>(), table, k_new.data_ptr(),
          v_new.data_ptr(), static_cast<int>(slot_ids.size(0)), static_cast<int>(k_cache.size(1)),
          static_cast<int>(k_cache.size(3)), static_cast<int>(k_cache.size(2)), k_cache.size(0),
          lens.size(0) < block_table.size(0) ? lens.size(0) : block_table.size(0),
          block_table.stride(0), k_cache.stride(0), k_cache.stride(1), k_new.stride(1),
          k_new.stride(2), v_new.stride(1), v_new.stride(2),
          reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
      },
      cie_kv_decode_update, cie_kv_decode_update_bt32);
  check_status(st, "kv_decode_update");
}

void kv_mixed_update(at::Tensor& k_cache, at::Tensor& v_cache, const at::Tensor& pages,
                     const at::Tensor& offsets, const at::Tensor& k_new, const at::Tensor& v_new) {
  check_update_src(k_cache, v_cache, k_new, v_new);
  check_i64(pages, "pages");
  check_i64(offsets, "offsets");
  TORCH_CHECK(pages.dim() == 1 && offsets.dim() == 1 && pages.size(0) == offsets.size(0) &&
                  pages.size(0) == k_new.size(1),
              "pages / offsets must be (T,) matching the new rows");
  TORCH_CHECK(pages.is_contiguous() && offsets.is_contiguous(), "pages / offsets contiguous");
  c10::cuda::CUDAGuard guard(k_cache.device());
  const int st = cie_kv_mixed_update(
      k_cache.data_ptr(), v_cache.data_ptr(), pages.data_ptr<int64_t>(),
      offsets.data_ptr<int64_t>(), k_new.data_ptr(), v_new.data_ptr(), pages.size(0),
      static_cast<int>(k_cache.size(1)), static_cast<int>(k_cache.size(3)),
      static_cast<int>(k_cache.size(2)), k_cache.size(0), k_cache.stride(0), k_cache.stride(1),
      k_new.stride(1), k_new.stride(2), v_new.stride(1), v_new.stride(2),
      reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
  check_status(st, "kv_mixed_update");
}

void check_rope_src(const at::Tensor& qkv, const at::Tensor& cos, const at::Tensor& sin,
                    const at::Tensor& kc, const at::Tensor& vc) {
  TORCH_CHECK(qkv.is_cuda() && cos.is_cuda() && sin.is_cuda(), "qkv / cos / sin must be CUDA");
  TORCH_CHECK(qkv.scalar_type() == at::kHalf && cos.scalar_type() == at::kHalf &&
                  sin.scalar_type() == at::kHalf,
              "qkv / cos / sin must be float16");
  TORCH_CHECK(kc.is_cuda() && vc.is_cuda() && kc.scalar_type() == at::kHalf &&
                  vc.scalar_type() == at::kHalf,
              "caches must be float16 CUDA tensors");
  TORCH_CHECK(kc.dim() == 4 && kc.sizes() == vc.sizes() && kc.strides() == vc.strides() &&
                  kc.stride(3) == 1 && kc.stride(2) == kc.size(3),
              "k_cache / v_cache must be (n_pages, H_kv, page_size, D) with dense rows");
  TORCH_CHECK(qkv.dim() == 3 && qkv.size(0) == 1 && qkv.stride(2) == 1,
              "qkv must be (1, T, (H_q + 2 H_kv) * D) with unit inner stride");
  TORCH_CHECK(qkv.size(2) % kc.size(3) == 0 && qkv.size(2) / kc.size(3) > 2 * kc.size(1),
              "qkv width must be (H_q + 2 H_kv) * D");
  TORCH_CHECK(cos.dim() == 3 && cos.sizes() == sin.sizes() && cos.strides() == sin.strides() &&
                  cos.size(0) == 1 && cos.size(1) == qkv.size(1) && cos.size(2) == kc.size(3) &&
                  cos.stride(2) == 1,
              "cos / sin must be (1, T, D) with unit inner stride");
}

at::Tensor rope_out(const at::Tensor& qkv, const at::Tensor& kc) {
  const int64_t d = kc.size(3);
  const int64_t hq = qkv.size(2) / d - 2 * kc.size(1);
  return at::empty({1, qkv.size(1), hq, d}, qkv.options());
}

at::Tensor rope_kv_decode_update(const at::Tensor& qkv, const at::Tensor& cos,
                                 const at::Tensor& sin, at::Tensor& k_cache, at::Tensor& v_cache,
                                 const at::Tensor& lens, const at::Tensor& slot_ids,
                                 const at::Tensor& block_table) {
  check_rope_src(qkv, cos, sin, k_cache, v_cache);
  check_i64(lens, "lens");
  check_i64(slot_ids, "slot_ids");
  check_table(block_table);
  TORCH_CHECK(block_table.dim() == 2 && block_table.stride(1) == 1, "block_table must be 2-D");
  TORCH_CHECK(slot_ids.dim() == 1 && slot_ids.size(0) == qkv.size(1), "one token per slot id");
  TORCH_CHECK(lens.is_contiguous() && slot_ids.is_contiguous(), "lens / slot_ids contiguous");
  c10::cuda::CUDAGuard guard(qkv.device());
  at::Tensor q = rope_out(qkv, k_cache);
  const int st = with_table(
      block_table,
      [&](auto fn, auto* table) {
        return fn(qkv.data_ptr(), qkv.stride(1), cos.data_ptr(), sin.data_ptr(), cos.stride(1),
          q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), lens.data_ptr<int64_t>(),
          slot_ids.data_ptr<int64_t>(), table,
          static_cast<int>(slot_ids.size(0)), static_cast<int>(q.size(2)),
          static_cast<int>(k_cache.size(1)), static_cast<int>(k_cache.size(3)),
          static_cast<int>(k_cache.size(2)), k_cache.size(0),
          lens.size(0) < block_table.size(0) ? lens.size(0) : block_table.size(0),
          block_table.stride(0), k_cache.stride(0), k_cache.stride(1),
          reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
      },
      cie_rope_kv_decode_update, cie_rope_kv_decode_update_bt32);
  check_status(st, "rope_kv_decode_update");
  return q;
}

at::Tensor rope_kv_mixed_update(const at::Tensor& qkv, const at::Tensor& cos,
                                const at::Tensor& sin, at::Tensor& k_cache, at::Tensor& v_cache,
                                const at::Tensor& pages, const at::Tensor& offsets) {
  check_rope_src(qkv, cos, sin, k_cache, v_cache);
  check_i64(pages, "pages");
  check_i64(offsets, "offsets");
  TORCH_CHECK(pages.dim() == 1 && offsets.dim() == 1 && pages.size(0) == offsets.size(0) &&
                  pages.size(0) == qkv.size(1),
              "pages / offsets must be (T,) matching qkv");
  TORCH_CHECK(pages.is_contiguous() && offsets.is_contiguous(), "pages / offsets contiguous");
  c10::cuda::CUDAGuard guard(qkv.device());
  at::Tensor q = rope_out(qkv, k_cache);
  const int st = cie_rope_kv_mixed_update(
      qkv.data_ptr(), qkv.stride(1), cos.data_ptr(), sin.data_ptr(), cos.stride(1),
      q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), pages.data_ptr<int64_t>(),
      offsets.data_ptr<int64_t>(), pages.size(0), static_cast<int>(q.size(2)),
      static_cast<int>(k_cache.size(1)), static_cast<int>(k_cache.size(3)),
      static_cast<int>(k_cache.size(2)), k_cache.size(0), k_cache.stride(0), k_cache.stride(1),
      reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
  check_status(st, "rope_kv_mixed_update");
  return q;
}

// rope_kv_mixed_update + gqa_mixed_attention as one call (cie_rope_kv_mixed_attention):
// the pass's k / v rows are written to their pages and o is returned.
at::Tensor rope_kv_mixed_attention(const at::Tensor& qkv, const at::Tensor& cos,
                                   const at::Tensor& sin, at::Tensor& k_cache,
                                   at::Tensor& v_cache, const at::Tensor& pages,
                                   const at::Tensor& offsets, c10::SymInt max_seqlen_sym,
                                   const at::Tensor& cu_seqlens, const at::Tensor& kv_lens,
                                   const at::Tensor& slot_ids, const at::Tensor& block_table) {
  const int64_t max_seqlen = max_seqlen_sym.expect_int();
  check_rope_src(qkv, cos, sin, k_cache, v_cache);
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(), "k and v must be contiguous");
  check_i64(pages, "pages");
  check_i64(offsets, "offsets");
  TORCH_CHECK(pages.dim() == 1 && offsets.dim() == 1 && pages.size(0) == offsets.size(0) &&
                  pages.size(0) == qkv.size(1),
              "pages / offsets must be (T,) matching qkv");
  TORCH_CHECK(pages.is_contiguous() && offsets.is_contiguous(), "pages / offsets contiguous");
  check_i64(cu_seqlens, "cu_seqlens");
  check_i64(kv_lens, "kv_lens");
  check_i64(slot_ids, "slot_ids");
  check_table(block_table);
  const int64_t B = slot_ids.size(0);
  TORCH_CHECK(kv_lens.dim() == 1 && kv_lens.size(0) == B, "kv_lens must be (B,)");
  TORCH_CHECK(cu_seqlens.dim() == 1 && cu_seqlens.size(0) == B + 1, "cu_seqlens must be (B+1,)");
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(1) == k_cache.size(0) &&
                  block_table.stride(1) == 1,
              "block_table must be (n_slots, n_pages) with contiguous rows");
  TORCH_CHECK(cu_seqlens.is_contiguous() && kv_lens.is_contiguous() && slot_ids.is_contiguous(),
              "cu_seqlens / kv_lens / slot_ids must be contiguous");
  c10::cuda::CUDAGuard guard(qkv.device());
  at::Tensor o = rope_out(qkv, k_cache);
  const int64_t T = qkv.size(1);
  const int hq = static_cast<int>(o.size(2));
  const int hkv = static_cast<int>(k_cache.size(1));
  const size_t ws_bytes = cie_rope_kv_mixed_workspace_bytes(static_cast<int>(B), T, hq, hkv, 0,
                                                            qkv.get_device());
  at::Tensor ws = at::empty({static_cast<int64_t>((ws_bytes + 3) / sizeof(float))},
                            qkv.options().dtype(at::kFloat));
  const int st = with_table(
      block_table,
      [&](auto fn, auto* table) {
        return fn(qkv.data_ptr(), qkv.stride(1), cos.data_ptr(), sin.data_ptr(), cos.stride(1),
                  k_cache.data_ptr(), v_cache.data_ptr(), pages.data_ptr<int64_t>(),
                  offsets.data_ptr<int64_t>(), max_seqlen, cu_seqlens.data_ptr<int64_t>(),
                  kv_lens.data_ptr<int64_t>(), slot_ids.data_ptr<int64_t>(), table, o.data_ptr(),
                  ws.data_ptr(), ws_bytes, static_cast<int>(B), T, hq, hkv,
                  static_cast<int>(k_cache.size(3)), static_cast<int>(k_cache.size(2)),
                  k_cache.size(0), block_table.size(0), block_table.stride(0),
                  k_cache.stride(0), k_cache.stride(1), 0,
                  reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
      },
      cie_rope_kv_mixed_attention, cie_rope_kv_mixed_attention_bt32);
  check_status(st, "rope_kv_mixed_attention");
  return o;
}

at::Tensor rope_kv_decode_attention(const at::Tensor& qkv, const at::Tensor& cos,
                                    const at::Tensor& sin, at::Tensor& k_cache,
                                    at::Tensor& v_cache, const at::Tensor& lens,
                                    const at::Tensor& slot_ids, const at::Tensor& block_table) {
  check_rope_src(qkv, cos, sin, k_cache, v_cache);
  check_i64(lens, "lens");
  check_i64(slot_ids, "slot_ids");
  check_table(block_table);
  TORCH_CHECK(block_table.dim() == 2 && block_table.stride(1) == 1 &&
                  block_table.size(1) == k_cache.size(0),
              "block_table must be (n_slots, n_pages)");
  TORCH_CHECK(slot_ids.dim() == 1 && slot_ids.size(0) == qkv.size(1), "one token per slot id");
  TORCH_CHECK(lens.dim() == 1 && lens.is_contiguous() && slot_ids.is_contiguous(),
              "lens (per slot) / slot_ids must be contiguous 1-D");
  c10::cuda::CUDAGuard guard(qkv.device());
  at::Tensor o = rope_out(qkv, k_cache);
  const int64_t B = slot_ids.size(0);
  if (B == 0) return o;
  const int hq = static_cast<int>(o.size(2));
  const int S = cie_decode_default_splits(static_cast<int>(B), qkv.get_device());
  const size_t ws_bytes = cie_decode_workspace_bytes(static_cast<int>(B), hq,
                                                     static_cast<int>(k_cache.size(3)), S);
  at::Tensor ws;
  if (ws_bytes > 0)
    ws = at::empty({static_cast<int64_t>(ws_bytes / sizeof(float))}, qkv.options().dtype(at::kFloat));
  const int st = with_table(
      block_table,
      [&](auto fn, auto* table) {
        return fn(qkv.data_ptr(), qkv.stride(1), cos.data_ptr(), sin.data_ptr(), cos.stride(1),
          k_cache.data_ptr(), v_cache.data_ptr(), lens.data_ptr<int64_t>(),
          slot_ids.data_ptr<int64_t>(), table, o.data_ptr(),
          ws_bytes > 0 ? ws.data_ptr() : nullptr, ws_bytes, static_cast<int>(B), hq,
          static_cast<int>(k_cache.size(1)), static_cast<int>(k_cache.size(3)),
          static_cast<int>(k_cache.size(2)), k_cache.size(0),
          lens.size(0) < block_table.size(0) ? lens.size(0) : block_table.size(0),
          block_table.stride(0), k_cache.stride(0), k_cache.stride(1), S,
          reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
      },
      cie_rope_kv_decode_attention, cie_rope_kv_decode_attention_bt32);
  check_status(st, "rope_kv_decode_attention");
  return o;
}

// ---- Qwen2 body helpers (cie_model_ops.h) ----------------------------------

void check_rows(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kHalf, name, " must be a float16 CUDA tensor");
  TORCH_CHECK(t.dim() >= 1 && t.stride(-1) == 1, name, " must have a unit inner stride");
  for (int64_t d = 0; d + 2 < t.dim(); ++d)
    TORCH_CHECK(t.size(d) == 1 || t.stride(d) == t.stride(d + 1) * t.size(d + 1), name,
                " must be contiguous apart from its row stride");
}

int64_t row_stride(const at::Tensor& t) { return t.dim() >= 2 ? t.stride(-2) : t.size(-1); }

at::Tensor rms_norm(const at::Tensor& x, const at::Tensor& weight, double eps) {
  check_rows(x, "x");
  TORCH_CHECK(weight.is_cuda() && weight.scalar_type() == at::kHalf && weight.dim() == 1 &&
                  weight.is_contiguous() && weight.size(0) == x.size(-1),
              "weight must be a contiguous float16 (hidden,) CUDA tensor");
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor out = at::empty(x.sizes(), x.options());
  const int64_t rows = x.numel() / std::max<int64_t>(x.size(-1), 1);
  const int st = cie_rms_norm(const_cast<void*>(x.data_ptr()), nullptr, weight.data_ptr(),
                              out.data_ptr(), rows, static_cast<int>(x.size(-1)), row_stride(x), 0,
                              x.size(-1), static_cast<float>(eps),
                              reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
  check_status(st, "rms_norm");
  return out;
}

at::Tensor add_rms_norm(at::Tensor& residual, const at::Tensor& delta, const at::Tensor& weight,
                        double eps) {
  check_rows(residual, "residual");
  check_rows(delta, "delta");
  TORCH_CHECK(residual.sizes() == delta.sizes(), "residual and delta shapes differ");
  TORCH_CHECK(weight.is_cuda() && weight.scalar_type() == at::kHalf && weight.dim() == 1 &&
                  weight.is_contiguous() && weight.size(0) == residual.size(-1),
              "weight must be a contiguous float16 (hidden,) CUDA tensor");
  c10::cuda::CUDAGuard guard(residual.device());
  at::Tensor out = at::empty(residual.sizes(), residual.options());
  const int64_t rows = residual.numel() / std::max<int64_t>(residual.size(-1), 1);
  const int st = cie_rms_norm(residual.data_ptr(), delta.data_ptr(), weight.data_ptr(),
                              out.data_ptr(), rows, static_cast<int>(residual.size(-1)),
                              row_stride(residual), row_stride(delta), residual.size(-1),
                              static_cast<float>(eps),
                              reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
  check_status(st, "add_rms_norm");
  return out;
}

at::Tensor silu_and_mul(const at::Tensor& gate_up) {
  check_rows(gate_up, "gate_up");
  TORCH_CHECK(gate_up.size(-1) % 2 == 0, "gate_up must hold [gate | up]");
  c10::cuda::CUDAGuard guard(gate_up.device());
  const int64_t n = gate_up.size(-1) / 2;
  std::vector<int64_t> shape(gate_up.sizes().begin(), gate_up.sizes().end());
  shape.back() = n;
  at::Tensor out = at::empty(shape, gate_up.options());
  const int64_t rows = gate_up.numel() / std::max<int64_t>(gate_up.size(-1), 1);
  const auto* g = static_cast<const at::Half*>(gate_up.data_ptr());
  const int st = cie_silu_mul(g, g + n, out.data_ptr(), rows, static_cast<int>(n),
                              row_stride(gate_up), row_stride(gate_up), n,
                              reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
  check_status(st, "silu_and_mul");
  return out;
}

at::Tensor argmax_rows(const at::Tensor& x) {
  check_rows(x, "x");
  c10::cuda::CUDAGuard guard(x.device());
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end() - 1);
  at::Tensor out = at::empty(shape, x.options().dtype(at::kLong));
  const int64_t rows = x.numel() / std::max<int64_t>(x.size(-1), 1);
  const size_t ws_bytes = cie_argmax_workspace_bytes(rows);
  at::Tensor ws = at::empty({static_cast<int64_t>(std::max<size_t>(ws_bytes, 8) / 8)},
                            x.options().dtype(at::kLong));
  const int st = cie_argmax_rows(x.data_ptr(), rows, static_cast<int>(x.size(-1)), row_stride(x),
                                 out.data_ptr<int64_t>(), ws.data_ptr(), ws_bytes,
                                 reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
  check_status(st, "argmax_rows");
  return out;
}

// tokens = argmax(hidden . weight^T) over the vocabulary, in one pass over the
// weight (cie_lm_head_argmax); hidden (..., H) with a contiguous last dim.
at::Tensor lm_head_argmax(const at::Tensor& hidden, const at::Tensor& weight) {
  check_rows(hidden, "hidden");
  check_rows(weight, "weight");
  TORCH_CHECK(weight.dim() == 2 && weight.size(1) == hidden.size(-1),
              "weight must be (vocab, hidden_size)");
  c10::cuda::CUDAGuard guard(hidden.device());
  std::vector<int64_t> shape(hidden.sizes().begin(), hidden.sizes().end() - 1);
  at::Tensor out = at::empty(shape, hidden.options().dtype(at::kLong));
  const int64_t rows = hidden.numel() / std::max<int64_t>(hidden.size(-1), 1);
  if (rows == 0) return out;
  const size_t ws_bytes =
      cie_lm_head_argmax_workspace_bytes(static_cast<int>(rows), weight.size(0), hidden.get_device());
  at::Tensor ws = at::empty({static_cast<int64_t>(std::max<size_t>(ws_bytes, 8) / 8)},
                            hidden.options().dtype(at::kLong));
  const int st = cie_lm_head_argmax(
      hidden.data_ptr(), row_stride(hidden), weight.data_ptr(), weight.stride(0),
      static_cast<int>(rows), static_cast<int>(hidden.size(-1)), weight.size(0), nullptr, 0,
      out.data_ptr<int64_t>(), ws.data_ptr(), ws_bytes,
      reinterpret_cast<cie_stream_t>(at::cuda::getCurrentCUDAStream().stream()));
  check_status(st, "lm_head_argmax");
  return out;
}

}  // namespace

TORCH_LIBRARY(inference, m) {
  m.def(
      "gqa_decode_attention(Tensor q, Tensor k, Tensor v, Tensor lens, Tensor slot_ids, "
      "Tensor block_table) -> Tensor");
  m.def(
      "gqa_mixed_attention(Tensor q, Tensor k, Tensor v, SymInt max_seqlen, Tensor cu_seqlens, "
      "Tensor kv_lens, Tensor slot_ids, Tensor block_table) -> Tensor");
  m.def(
      "gqa_decode_attention_splits(Tensor q, Tensor k, Tensor v, Tensor lens, Tensor slot_ids, "
      "Tensor block_table, int num_splits) -> Tensor");
  m.def(
      "kv_decode_update(Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor lens, Tensor slot_ids, "
      "Tensor block_table, Tensor k_new, Tensor v_new) -> ()");
  m.def(
      "kv_mixed_update(Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor pages, Tensor offsets, "
      "Tensor k_new, Tensor v_new) -> ()");
  m.def(
      "rope_kv_decode_update(Tensor qkv, Tensor cos, Tensor sin, Tensor(a!) k_cache, "
      "Tensor(b!) v_cache, Tensor lens, Tensor slot_ids, Tensor block_table) -> Tensor");
  m.def(
      "rope_kv_mixed_update(Tensor qkv, Tensor cos, Tensor sin, Tensor(a!) k_cache, "
      "Tensor(b!) v_cache, Tensor pages, Tensor offsets) -> Tensor");
  m.def(
      "rope_kv_mixed_attention(Tensor qkv, Tensor cos, Tensor sin, Tensor(a!) k_cache, "
      "Tensor(b!) v_cache, Tensor pages, Tensor offsets, SymInt max_seqlen, Tensor cu_seqlens, "
      "Tensor kv_lens, Tensor slot_ids, Tensor block_table) -> Tensor");
  m.def(
      "rope_kv_decode_attention(Tensor qkv, Tensor cos, Tensor sin, Tensor(a!) k_cache, "
      "Tensor(b!) v_cache, Tensor lens, Tensor slot_ids, Tensor block_table) -> Tensor");
  m.def("rms_norm(Tensor x, Tensor weight, float eps) -> Tensor");
  m.def("add_rms_norm(Tensor(a!) residual, Tensor delta, Tensor weight, float eps) -> Tensor");
  m.def("silu_and_mul(Tensor gate_up) -> Tensor");
  m.def("argmax_rows(Tensor x) -> Tensor");
  m.def("lm_head_argmax(Tensor hidden, Tensor weight) -> Tensor");
}

TORCH_LIBRARY_IMPL(inference, CUDA, m) {
  m.impl("gqa_decode_attention", &gqa_decode_attention);
  m.impl("gqa_mixed_attention", &gqa_mixed_attention);
  m.impl("gqa_decode_attention_splits", &gqa_decode_attention_splits);
  m.impl("kv_decode_update", &kv_decode_update);
  m.impl("kv_mixed_update", &kv_mixed_update);
  m.impl("rope_kv_decode_update", &rope_kv_decode_update);
  m.impl("rope_kv_mixed_update", &rope_kv_mixed_update);
  m.impl("rope_kv_decode_attention", &rope_kv_decode_attention);
  m.impl("rope_kv_mixed_attention", &rope_kv_mixed_attention);
  m.impl("rms_norm", &rms_norm);
  m.impl("add_rms_norm", &add_rms_norm);
  m.impl("silu_and_mul", &silu_and_mul);
  m.impl("argmax_rows", &argmax_rows);
  m.impl("lm_head_argmax", &lm_head_argmax);
}
