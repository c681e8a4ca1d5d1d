/*
 * cie_model_ops.h -- element-wise kernels of the Qwen2 decoder body around
 * the attention path, in libcie_attention.so (same conventions and status
 * codes as cie_attention.h: device pointers, element strides, asynchronous on
 * `stream`, no allocation, no host synchronisation, graph-capturable).
 *
 * These have no counterpart in the reference's attention FFI: the reference
 * runs Hugging Face's Qwen2 modules (Qwen2RMSNorm, the decoder layer's
 * residual adds, Qwen2MLP) and leaves their fusion to torch.compile. The
 * model runner of this package calls them instead of those modules. They
 * follow torch's fp16 arithmetic step for step (fp32 inside, the same
 * roundings to fp16); only the order of RMSNorm's sum of squares differs.
 */
#ifndef CIE_MODEL_OPS_H_
#define CIE_MODEL_OPS_H_

#include <stdint.h>

#include "cie_attention.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * RMSNorm of `rows` rows of `hidden` fp16 values, Qwen2RMSNorm's arithmetic:
 *   out = weight * fp16(x * rsqrt(mean(x^2) + eps))      (fp32 inside)
 * With delta == NULL, x = h (read only). With delta != NULL the residual add
 * comes first and is written back: h = fp16(h + delta), x = the new h (the
 * decoder layer's `residual + hidden_states` followed by the next norm).
 * Row strides in elements; every row 16-byte aligned; hidden % 8 == 0.
 */
int cie_rms_norm(void* h, const void* delta, const void* weight, void* out, int64_t rows,
                 int hidden, int64_t h_stride, int64_t delta_stride, int64_t out_stride,
                 float eps, cie_stream_t stream);

/*
 * Qwen2MLP's act_fn(gate) * up with act_fn = SiLU:
 *   out = fp16(fp16(g / (1 + exp(-g))) * up)             (fp32 inside)
 * gate / up / out: `rows` rows of `size` fp16 values at the given row
 * strides (gate and up may be the two halves of one fused projection).
 * Every row 16-byte aligned; size % 8 == 0.
 */
int cie_silu_mul(const void* gate, const void* up, void* out, int64_t rows, int size,
                 int64_t gate_stride, int64_t up_stride, int64_t out_stride,
                 cie_stream_t stream);

/*
 * out[r] = index of the largest of the n fp16 values of row r (rows `stride`
 * elements apart; 16-byte aligned rows are read 8 values at a time): the first
 * index when several are equal, a NaN counting as the largest -- torch.argmax
 * (dim=-1). For greedy decoding over the 151936-way logits (the reference's
 * argmax after lm_head, scheduler/decode_module.py:103). out: int64. Two
 * launches: parts of every row, then the parts; `workspace` holds the parts
 * (>= cie_argmax_workspace_bytes(rows) bytes, 8-byte aligned, no
 * initialisation). rows <= 65535.
 */
size_t cie_argmax_workspace_bytes(int64_t rows);
int cie_argmax_rows(const void* x, int64_t rows, int n, int64_t stride, int64_t* out,
                    void* workspace, size_t workspace_bytes, cie_stream_t stream);

/*
 * The greedy token after the last-token lm_head, in one pass over the weight
 * (the lm_head GEMM + argmax of scheduler/decode_module.py:103-107 and
 * scheduler/mixed_module.py:58-65): tokens[b] = argmax over v of
 * fp16(hidden[b] . weight[v]), with cie_argmax_rows' semantics (first index of
 * the maximum, NaN largest). hidden (batch, hidden_size) and weight (vocab,
 * hidden_size) fp16 at the given row strides (elements; rows 16-byte aligned);
 * hidden_size a multiple of 64 up to 1024; vocab < 2^30. `logits` (optional,
 * may be NULL) receives the fp16 logits (batch, vocab) at logits_stride; they
 * are the tensor core's fp32 dot products rounded once to fp16, as a fp16 GEMM
 * with fp32 accumulation returns them (the summation order may differ from
 * another GEMM's in the last fp32 bit). Batches above 64 run in slices of 64
 * rows (one pass over the weight each). `workspace`:
 * cie_lm_head_argmax_workspace_bytes(batch, vocab, device) bytes, 16-byte
 * aligned, no initialisation.
 */
size_t cie_lm_head_argmax_workspace_bytes(int batch, int64_t vocab, int device);
int cie_lm_head_argmax(const void* hidden, int64_t hidden_stride, const void* weight,
                       int64_t weight_stride, int batch, int hidden_size, int64_t vocab,
                       void* logits, int64_t logits_stride, int64_t* tokens, void* workspace,
                       size_t workspace_bytes, cie_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CIE_MODEL_OPS_H_ */
