/*
 * cie_attention.h -- C ABI of the B200 (sm_100a) paged GQA attention library
 * (libcie_attention.so).
 *
 * Every entry point takes plain device pointers, sizes and strides (in
 * elements), launches asynchronously on `stream`, performs no host<->device
 * synchronisation and allocates nothing. cie_decode_attention,
 * cie_mixed_attention, cie_kv_decode_update, cie_kv_mixed_update, the two
 * cie_rope_kv_*_update entry points and cie_rope_kv_decode_attention can be
 * captured in a CUDA graph. Return value: CIE_OK or a negative cie_status; on
 * error nothing was launched and cie_last_error_message() (thread-local) says
 * why.
 *
 * Layouts are the reference engine's (eteboun/custom_inference_engine):
 *   q / o        (1, T, num_q_heads, head_dim)  fp16, contiguous
 *   k / v pool   (n_pages, num_kv_heads, page_size, head_dim) fp16,
 *                row stride head_dim, unit inner stride (kv_cache/storage.py:32-48)
 *   block_table  (n_slots, bt_stride) int64, slot s's logical page j at
 *                block_table[s * bt_stride + j]   (kv_cache/storage.py:54-56)
 *   lens, kv_lens, slot_ids, pages, offsets: int64; cu_seqlens: int64 (B+1)
 * Supported shapes: head_dim 64, page_size 16, num_q_heads / num_kv_heads = 7
 * (Qwen2.5-0.5B: 14 / 2); decode takes num_kv_heads 1, 2 or 4.
 */
#ifndef CIE_ATTENTION_H_
#define CIE_ATTENTION_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; declared here so the header needs no CUDA headers. */
typedef struct CUstream_st* cie_stream_t;

enum cie_status {
  CIE_OK = 0,
  CIE_ERR_INVALID_ARGUMENT = -1, /* null pointer, negative size, bad stride   */
  CIE_ERR_UNSUPPORTED = -2,      /* head_dim / page_size / group not supported */
  CIE_ERR_OVERFLOW = -3,         /* an index would not fit the kernel's int32  */
  CIE_ERR_ALIGNMENT = -4,        /* pointer or stride breaks a 16-byte rule    */
  CIE_ERR_WORKSPACE = -5,        /* workspace missing or too small             */
  CIE_ERR_CUDA = -6              /* a CUDA runtime/driver call failed          */
};

/* Bits reported by cie_read_device_errors(): kernels never trap; a failed
 * device-side check or a wait that exceeded its time limit sets a bit and
 * the kernel returns early. */
enum cie_device_error_bits {
  CIE_DEVERR_BAD_SLOT = 1u << 0,      /* slot id outside [0, n_slots)             */
  CIE_DEVERR_BAD_LENGTH = 1u << 1,    /* length exceeds the block-table row       */
  CIE_DEVERR_BAD_PAGE = 1u << 2,      /* page id outside [0, n_pages)             */
  CIE_DEVERR_BAD_OFFSET = 1u << 3,    /* in-page offset outside [0, page_size)    */
  CIE_DEVERR_WAIT_TIMEOUT = 1u << 4,  /* an mbarrier wait ran past its limit      */
  CIE_DEVERR_BAD_SEQLENS = 1u << 5    /* cu_seqlens not monotone / beyond T       */
};

/* ---- library-wide ---------------------------------------------------------- */

int cie_version(void);
const char* cie_status_string(int status);
const char* cie_last_error_message(void);

/* Copies the device error bits of `device` into *bits and, when `clear` is
 * non-zero, resets them. Synchronous (it waits for `device`'s prior work). */
int cie_read_device_errors(int device, unsigned int* bits, int clear);

/* ---- split-KV paged GQA decode ------------------------------------------- */

/* Split count used when cie_decode_attention() is given num_splits <= 0:
 * enough (sequence, split) CTAs to keep every SM of `device` streaming
 * (two per SM), at most 64, rounded down to a power of two when it is less
 * than 5/4 of one (148 SMs: batch 8 -> 32, 16 -> 16, 32 -> 8). */
int cie_decode_default_splits(int batch, int device);

/* Bytes of fp32 workspace the split path needs (0 when num_splits == 1). */
size_t cie_decode_workspace_bytes(int batch, int num_q_heads, int head_dim, int num_splits);

/*
 * One query token per sequence over the paged KV pool.
 * Replaces attn/core.py:13-66 (decode_gqa_attention) and its kernels
 * kernels/decode_attention.py:12-179 (load) and :182-272 (merge); this is the
 * body of the torch op inference::gqa_decode_attention (attn/core.py:119-126).
 *   sequence b: query q[0, b], slot slot_ids[b], visible rows [0, lens[b])
 *   (lens includes the token just written by decode_update); lens[b] == 0
 *   gives a zero output row, as the reference merge does.
 * num_splits: KV splits per sequence (<= 0: cie_decode_default_splits).
 * workspace: >= cie_decode_workspace_bytes(...) bytes, 16-byte aligned
 * (may be NULL when the split count resolves to 1).
 * Launches the split kernel as a programmatic dependent of the preceding
 * kernel in `stream` (no input is read before its griddepcontrol.wait, so a
 * producer kernel that triggers early is safe) and, with more than one split,
 * the merge kernel as a programmatic dependent of the split kernel.
 */
int cie_decode_attention(const void* q, const void* k, const void* v, const int64_t* lens,
                         const int64_t* slot_ids, const int64_t* block_table, void* o,
                         void* workspace, size_t workspace_bytes, int batch, int num_q_heads,
                         int num_kv_heads, int head_dim, int page_size, int64_t n_pages,
                         int64_t n_slots, int64_t bt_stride, int64_t kv_page_stride,
                         int64_t kv_head_stride, int num_splits, cie_stream_t stream);

/*
 * Same computation and arguments as cie_decode_attention, minus the workspace:
 * the split partials go to a scratch array inside this library, so the call
 * allocates nothing and the caller passes only inputs and outputs.
 * No counterpart in the reference: it exists for callers that cannot allocate
 * device memory -- a host that only holds device pointers handed over an FFI
 * and has no device allocator, or a process that reserved all of HBM for
 * weights and the KV pool, where another cudaMalloc would fail or, because
 * cudaMalloc / cudaFree synchronise the device, stall the decode loop.
 * Limit: cie_decode_workspace_bytes(batch, num_q_heads, head_dim, splits) must
 * not exceed CIE_DECODE_NOALLOC_SCRATCH_BYTES (4 MiB, i.e. batch x splits <= 1134
 * for 14 heads of 64); larger requests return CIE_ERR_WORKSPACE.
 * Every GPU that loads the library holds the 4 MiB until the process exits.
 * A call outside a stream capture looks up the array's device address (with
 * the call's device current) and caches it per device; a call whose stream is
 * capturing uses the cached address, so make the first call on a device before
 * any stream capture (a first call inside a capture returns
 * CIE_ERR_INVALID_ARGUMENT). Arguments are checked as cie_decode_attention
 * checks them, before the scratch limit, with the same status codes. All calls
 * on a device share the array and it keeps the last call's contents (nothing
 * in it needs to start at zero); calls that overlap on the GPU race on it.
 */
#define CIE_DECODE_NOALLOC_SCRATCH_BYTES (4u << 20)

int cie_decode_attention_noalloc(const void* q, const void* k, const void* v,
                                 const int64_t* lens, const int64_t* slot_ids,
                                 const int64_t* block_table, void* o, int batch,
                                 int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                                 int64_t n_pages, int64_t n_slots, int64_t bt_stride,
                                 int64_t kv_page_stride, int64_t kv_head_stride, int num_splits,
                                 cie_stream_t stream);

/* ---- varlen mixed (chunked prefill + decode) attention --------------------- */

/* Bytes of device workspace cie_mixed_attention() needs for `batch`
 * sequences of `total_tokens` rows in all, with the same num_splits, on
 * `device` (its SM count sizes the automatic plan; -1: 148 SMs). The
 * workspace holds the work plan (made on the device by the call itself), a
 * counter per split tile pair and the fp32 partials of split pairs; about
 * 30 MB on 148 SMs with num_splits <= 0, nothing needs to start at zero. */
size_t cie_mixed_workspace_bytes(int batch, int64_t total_tokens, int num_kv_heads,
                                 int num_splits, int device);

/*
 * Causal attention for a batch of chunks in one call.
 * Replaces attn/core.py:69-111 (mixed_gqa_attention) and its kernel
 * kernels/prefill_attention.py:10-198; body of inference::gqa_mixed_attention
 * (attn/core.py:128-137).
 *   sequence b owns rows [cu_seqlens[b], cu_seqlens[b+1]) of q / o; its row i
 *   sits at position kv_lens[b] + i and attends to keys [0, kv_lens[b] + i]
 *   of slot slot_ids[b] (the chunk's own K/V are already in the pool).
 *   max_seqlen bounds every chunk length (the bucket's token count).
 *   Rows outside every [cu_seqlens[b], cu_seqlens[b+1]) are not written.
 * Work partition: a planning kernel (one CTA) lists the (sequence, kv head,
 * 36-token tile pair) units that exist, cuts long ones into key ranges and
 * orders the pieces largest first; the attention kernel (launched with
 * programmatic stream serialization) runs one CTA per piece, and the last
 * piece of a cut pair to finish merges the fp32 partials of the others.
 * num_splits <= 0: automatic cut (pieces of at most max(2, ceil(total key
 * blocks / SMs)) 128-key blocks, <= 16 per pair); num_splits = S in
 * [1, 16]: every pair is cut into ceil(nb / max(ceil(nb / S), 2)) ranges.
 * workspace: >= cie_mixed_workspace_bytes(batch, total_tokens, num_kv_heads,
 * num_splits, device) bytes, 16-byte aligned. batch <= 2048.
 */
int cie_mixed_attention(const void* q, const void* k, const void* v, int64_t max_seqlen,
                        const int64_t* cu_seqlens, const int64_t* kv_lens,
                        const int64_t* slot_ids, const int64_t* block_table, void* o,
                        void* workspace, size_t workspace_bytes, int batch,
                        int64_t total_tokens, int num_q_heads, int num_kv_heads, int head_dim,
                        int page_size, int64_t n_pages, int64_t n_slots, int64_t bt_stride,
                        int64_t kv_page_stride, int64_t kv_head_stride, int num_splits,
                        cie_stream_t stream);

/* ---- KV-page scatter ------------------------------------------------------- */

/*
 * Writes each decode token's K and V row into its page.
 * Replaces KVStorage.decode_update (kv_cache/storage.py:87-122): for
 * s = slot_ids[i], pos = lens[s] (the slot's length BEFORE this token), the row
 * lands at page block_table[s * bt_stride + pos / page_size], offset
 * pos % page_size. k_new / v_new are (1, batch, num_kv_heads, head_dim) views
 * with token stride *_tok_stride and head stride *_head_stride (elements;
 * inner stride 1). Bit-exact copy.
 */
int cie_kv_decode_update(void* k_cache, void* v_cache, const int64_t* lens,
                         const int64_t* slot_ids, const int64_t* block_table, const void* k_new,
                         const void* v_new, int batch, int num_kv_heads, int head_dim,
                         int page_size, int64_t n_pages, int64_t n_slots, int64_t bt_stride,
                         int64_t cache_page_stride, int64_t cache_head_stride,
                         int64_t k_tok_stride, int64_t k_head_stride, int64_t v_tok_stride,
                         int64_t v_head_stride, cie_stream_t stream);

/*
 * Writes token t's K and V row to page pages[t], offset offsets[t].
 * Replaces KVStorage.mixed_update (kv_cache/storage.py:62-85). Bit-exact copy.
 */
int cie_kv_mixed_update(void* k_cache, void* v_cache, const int64_t* pages,
                        const int64_t* offsets, const void* k_new, const void* v_new,
                        int64_t num_tokens, int num_kv_heads, int head_dim, int page_size,
                        int64_t n_pages, int64_t cache_page_stride, int64_t cache_head_stride,
                        int64_t k_tok_stride, int64_t k_head_stride, int64_t v_tok_stride,
                        int64_t v_head_stride, cie_stream_t stream);

/* ---- rotary embedding fused with the KV-page scatter ----------------------- */

/*
 * One launch per layer for what the reference does between the fused QKV
 * projection and the attention op (attn/core.py:193-206): rotary embedding of
 * q and k (transformers Qwen2 apply_rotary_pos_emb: x * cos + rotate_half(x) *
 * sin, each operation rounded to fp16 as there, so results are bit-identical)
 * and KVStorage.decode_update (kv_cache/storage.py:87-122).
 *   qkv     (1, batch, (num_q_heads + 2 num_kv_heads) * head_dim) fp16, rows
 *           qkv_tok_stride elements apart: q heads, then k heads, then v heads.
 *   cos/sin (1, batch, head_dim) fp16, rows cs_tok_stride apart.
 *   q_out   (1, batch, num_q_heads, head_dim) fp16 contiguous: rotated q.
 * Rotated k and plain v of token i land where cie_kv_decode_update puts them
 * (slot slot_ids[i] at position lens[slot]). Every row 16-byte aligned;
 * head_dim 64.
 */
int cie_rope_kv_decode_update(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                              const void* sin, int64_t cs_tok_stride, void* q_out,
                              void* k_cache, void* v_cache, const int64_t* lens,
                              const int64_t* slot_ids, const int64_t* block_table, int batch,
                              int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                              int64_t n_pages, int64_t n_slots, int64_t bt_stride,
                              int64_t cache_page_stride, int64_t cache_head_stride,
                              cie_stream_t stream);

/*
 * The same for a mixed pass (KVStorage.mixed_update, kv_cache/storage.py:62-85):
 * token t's rotated k and v go to page pages[t], offset offsets[t].
 */
int cie_rope_kv_mixed_update(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                             const void* sin, int64_t cs_tok_stride, void* q_out, void* k_cache,
                             void* v_cache, const int64_t* pages, const int64_t* offsets,
                             int64_t num_tokens, int num_q_heads, int num_kv_heads, int head_dim,
                             int page_size, int64_t n_pages, int64_t cache_page_stride,
                             int64_t cache_head_stride, cie_stream_t stream);

/* ---- rotary embedding + KV write + decode attention in one launch ---------- */

/*
 * The whole attention step of a decode pass after the fused QKV projection
 * (attn/core.py:193-215 of the reference: apply_rotary_pos_emb, then
 * KVStorage.decode_update, kv_cache/storage.py:87-122, then the decode
 * attention op): token i (slot s = slot_ids[i], position lens[s], the slot's
 * length BEFORE it) has its q rotated in registers, its rotated k and plain v
 * written to page block_table[s * bt_stride + lens[s] / page_size], row
 * lens[s] % page_size, and attends to the lens[s] + 1 keys of its slot,
 * itself included. qkv / cos / sin as for cie_rope_kv_decode_update; o as
 * for cie_decode_attention; `lens` is per SLOT (n_slots entries, as
 * KVStorage.lens) and is not advanced. Same results, bit for bit, as
 * cie_rope_kv_decode_update followed by cie_decode_attention with
 * lens[slot_ids] + 1; workspace as for cie_decode_attention. num_kv_heads
 * 1, 2 or 4.
 */
int cie_rope_kv_decode_attention(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                                 const void* sin, int64_t cs_tok_stride, void* k_cache,
                                 void* v_cache, const int64_t* lens, const int64_t* slot_ids,
                                 const int64_t* block_table, void* o, void* workspace,
                                 size_t workspace_bytes, int batch, int num_q_heads,
                                 int num_kv_heads, int head_dim, int page_size, int64_t n_pages,
                                 int64_t n_slots, int64_t bt_stride, int64_t cache_page_stride,
                                 int64_t cache_head_stride, int num_splits, cie_stream_t stream);

/* ---- rotary embedding + KV write + mixed attention in one call -------------- */

/*
 * The whole attention step of a mixed pass (chunked prefill + decode rows):
 * the rotary embedding of q and k from the fused QKV projection, the write of
 * every token's k and v row to (pages[t], offsets[t]) -- what
 * cie_rope_kv_mixed_update does -- and cie_mixed_attention over the pass, with
 * no second call. Replaces attn/core.py:193-206 + :217-233 of the reference
 * (apply_rotary_pos_emb, KVStorage.mixed_update, the mixed attention op). The
 * planning kernel of the attention runs in the same grid as the rotation and
 * the K/V write (extra CTAs), and the attention kernel starts after that grid,
 * so it reads the pages as written. pages / offsets must address the rows that
 * block_table gives the same positions (the reference's AttentionMetadata does).
 * Output and pages are bit-identical to cie_rope_kv_mixed_update followed by
 * cie_mixed_attention. Arguments: those of the two calls; the rotated q lives in
 * the workspace (cie_rope_kv_mixed_workspace_bytes bytes, 16-byte aligned, no
 * initialisation).
 */
size_t cie_rope_kv_mixed_workspace_bytes(int batch, int64_t total_tokens, int num_q_heads,
                                         int num_kv_heads, int num_splits, int device);

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
                                int num_splits, cie_stream_t stream);

/* ---- int32 block table ------------------------------------------------------
 * The reference keeps the block table as int64 (kv_cache/storage.py:52-56) and
 * every entry point above takes it so. These variants take the same table as
 * int32 page ids (half the bytes per entry; page ids must be < 2^31, which the
 * n_pages check already requires) and are otherwise identical -- same
 * arguments, statuses and results, bit for bit. The torch ops dispatch to them
 * when block_table has dtype int32.
 */
int cie_decode_attention_bt32(const void* q, const void* k, const void* v, const int64_t* lens,
                              const int64_t* slot_ids, const int32_t* block_table, void* o,
                              void* workspace, size_t workspace_bytes, int batch, int num_q_heads,
                              int num_kv_heads, int head_dim, int page_size, int64_t n_pages,
                              int64_t n_slots, int64_t bt_stride, int64_t kv_page_stride,
                              int64_t kv_head_stride, int num_splits, cie_stream_t stream);

int cie_mixed_attention_bt32(const void* q, const void* k, const void* v, int64_t max_seqlen,
                             const int64_t* cu_seqlens, const int64_t* kv_lens,
                             const int64_t* slot_ids, const int32_t* block_table, void* o,
                             void* workspace, size_t workspace_bytes, int batch,
                             int64_t total_tokens, int num_q_heads, int num_kv_heads,
                             int head_dim, int page_size, int64_t n_pages, int64_t n_slots,
                             int64_t bt_stride, int64_t kv_page_stride, int64_t kv_head_stride,
                             int num_splits, cie_stream_t stream);

int cie_kv_decode_update_bt32(void* k_cache, void* v_cache, const int64_t* lens,
                              const int64_t* slot_ids, const int32_t* block_table,
                              const void* k_new, const void* v_new, int batch, int num_kv_heads,
                              int head_dim, int page_size, int64_t n_pages, int64_t n_slots,
                              int64_t bt_stride, int64_t cache_page_stride,
                              int64_t cache_head_stride, int64_t k_tok_stride,
                              int64_t k_head_stride, int64_t v_tok_stride,
                              int64_t v_head_stride, cie_stream_t stream);

int cie_rope_kv_decode_update_bt32(const void* qkv, int64_t qkv_tok_stride, const void* cos,
                                   const void* sin, int64_t cs_tok_stride, void* q_out,
                                   void* k_cache, void* v_cache, const int64_t* lens,
                                   const int64_t* slot_ids, const int32_t* block_table, int batch,
                                   int num_q_heads, int num_kv_heads, int head_dim,
                                   int page_size, int64_t n_pages, int64_t n_slots,
                                   int64_t bt_stride, int64_t cache_page_stride,
                                   int64_t cache_head_stride, cie_stream_t stream);

int cie_rope_kv_decode_attention_bt32(
    const void* qkv, int64_t qkv_tok_stride, const void* cos, const void* sin,
    int64_t cs_tok_stride, void* k_cache, void* v_cache, const int64_t* lens,
    const int64_t* slot_ids, const int32_t* block_table, void* o, void* workspace,
    size_t workspace_bytes, int batch, int num_q_heads, int num_kv_heads, int head_dim,
    int page_size, int64_t n_pages, int64_t n_slots, int64_t bt_stride, int64_t cache_page_stride,
    int64_t cache_head_stride, int num_splits, cie_stream_t stream);

int cie_rope_kv_mixed_attention_bt32(
    const void* qkv, int64_t qkv_tok_stride, const void* cos, const void* sin,
    int64_t cs_tok_stride, void* k_cache, void* v_cache, const int64_t* pages,
    const int64_t* offsets, int64_t max_seqlen, const int64_t* cu_seqlens, const int64_t* kv_lens,
    const int64_t* slot_ids, const int32_t* block_table, void* o, void* workspace,
    size_t workspace_bytes, int batch, int64_t total_tokens, int num_q_heads, int num_kv_heads,
    int head_dim, int page_size, int64_t n_pages, int64_t n_slots, int64_t bt_stride,
    int64_t cache_page_stride, int64_t cache_head_stride, int num_splits, cie_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CIE_ATTENTION_H_ */
