"""Paged GQA attention ops and the Qwen2 attention module that calls them.

Same public names and call contracts as the reference's attn/core.py, with
the Triton kernels replaced by the sm_100a CUDA kernels of
``libcie_attention.so``:

* ``decode_gqa_attention`` / ``mixed_gqa_attention`` -- host functions
  (attn/core.py:13-111): the reference's shape asserts, then the CUDA op;
* ``gqa_decode_attention_op`` / ``gqa_mixed_attention_op`` -- the torch ops
  ``inference::gqa_decode_attention`` and ``inference::gqa_mixed_attention``
  (attn/core.py:119-137), same schemas, so the piecewise splitter, which
  matches ``torch.ops.inference.gqa_mixed_attention.default`` and reads its
  ``kv_lens`` kwarg, keeps working;
* ``TritonQwen2Attention`` / ``use_triton_attention`` -- the drop-in
  replacement of HF ``Qwen2Attention`` (attn/core.py:139-250). The names are
  kept so existing callers need no edit; ``CudaQwen2Attention`` and
  ``use_cuda_attention`` are aliases.

Importing this module loads the CUDA extension and raises
``native.NativeLibraryMissing`` if it is not built: there is no fallback.
"""
from __future__ import annotations

import torch

from custom_inference_engine_b200 import native

native.load_ops()

# The op OVERLOADS, not the packets: a call through ``torch.ops.inference.X.default``
# is what Dynamo records as the node target, and the reference's piecewise
# splitter matches exactly ``torch.ops.inference.gqa_mixed_attention.default``
# (piecewise/utils.py:5-7), as a ``triton_op`` call in the reference produces.
gqa_decode_attention_op = torch.ops.inference.gqa_decode_attention.default
gqa_mixed_attention_op = torch.ops.inference.gqa_mixed_attention.default
rope_kv_decode_update_op = torch.ops.inference.rope_kv_decode_update.default
rope_kv_mixed_update_op = torch.ops.inference.rope_kv_mixed_update.default
rope_kv_decode_attention_op = torch.ops.inference.rope_kv_decode_attention.default
rope_kv_mixed_attention_op = torch.ops.inference.rope_kv_mixed_attention.default
_gqa_decode_attention_splits = torch.ops.inference.gqa_decode_attention_splits.default

# The reference tunes Triton tiles here (attn/core.py:114-116). The CUDA decode
# path has one knob, the number of KV splits per sequence; 0 lets the library
# size it from the batch and the SM count of the device.
GQA_DECODE_CONFIG = {"num_programs": 0}
GQA_PREFILL_CONFIG = {}


def decode_gqa_attention(q, k, v, lens, slot_ids, block_table, num_programs=0, BLOCK_N=None,
                         num_warps=None, wrap=None):
    """One query token per sequence over the paged pool (attn/core.py:13-66).

    q (1, B, H_q, D); k, v (n_pages, H_kv, page_size, D); lens (B,) rows
    visible to each query (the slot length including the token just written);
    slot_ids (B,); block_table (n_slots, n_pages). ``num_programs`` is the
    split-KV count (0: chosen by the library). ``BLOCK_N``, ``num_warps`` and
    ``wrap`` are the reference's Triton launch knobs; they are accepted and
    ignored.
    """
    total_T, H_q, D = q.shape[1:]
    N_PAGES, H_kv, PAGE_SIZE, _ = k.shape
    B = slot_ids.shape[0]
    assert H_q % H_kv == 0
    assert lens.shape == (B,)
    assert N_PAGES == block_table.shape[1]
    assert total_T == B
    assert q.is_contiguous()
    assert k.stride() == v.stride() and k.stride(3) == 1 and k.stride(2) == D
    return _gqa_decode_attention_splits(q, k, v, lens, slot_ids, block_table, int(num_programs))


def mixed_gqa_attention(q, k, v, max_seqlen: int, cu_seqlens, kv_lens, slot_ids, block_table,
                        BLOCK_M=None, BLOCK_N=None, num_warps=None, wrap=None):
    """Causal varlen attention for chunked prefill + decode rows (attn/core.py:69-111).

    Sequence b owns q rows [cu_seqlens[b], cu_seqlens[b+1]); its row i sits at
    position kv_lens[b] + i and sees keys 0 .. kv_lens[b] + i of slot
    slot_ids[b]. Rows outside every sequence are not written (the output is
    ``torch.empty_like(q)``, as in the reference). Tile knobs are ignored.
    """
    total_T, H_q, D = q.shape[1:]
    N_PAGES, H_kv, PAGE_SIZE, _ = k.shape
    B = slot_ids.shape[0]
    assert H_q % H_kv == 0
    assert kv_lens.shape == (B,)
    assert cu_seqlens.shape == (B + 1,)
    assert N_PAGES == block_table.shape[1]
    assert k.shape == v.shape and k.shape[3] == D
    assert q.is_contiguous() and k.is_contiguous() and v.is_contiguous()
    return gqa_mixed_attention_op(q, k, v, max_seqlen=max_seqlen, cu_seqlens=cu_seqlens,
                                  kv_lens=kv_lens, slot_ids=slot_ids, block_table=block_table)


class TritonQwen2Attention(torch.nn.Module):
    """HF ``Qwen2Attention`` replacement that runs the paged CUDA attention.

    With ``kv_manager`` (a ``KVStorage``) and ``metadata`` (an
    ``AttentionMetadata``) it computes the fused QKV projection, then:

    * decode pass: ONE launch (``inference::rope_kv_decode_attention``) rotates
      q and k, writes the new K/V row of every token into its page and runs the
      decode attention over the slot's keys, the new one included;
    * mixed pass: one launch rotates q and k and writes the new K/V rows
      (``inference::rope_kv_mixed_update``), then the mixed attention op;

    then ``o_proj``. The results are bit-identical to HF's
    ``apply_rotary_pos_emb`` followed by ``KVStorage.decode_update`` /
    ``mixed_update`` and the attention op. ``fuse_decode_attention = False``
    splits the decode pass into the RoPE + KV launch and the attention op;
    ``fuse_rope = False`` restores the reference's sequence (HF RoPE, then
    ``kv_manager``'s update methods). A mixed pass whose metadata has
    ``fuse_mixed_attention`` set is one call too
    (``inference::rope_kv_mixed_attention``); metadata written by the
    reference's modules never sets it, because the reference's piecewise
    backend splits the graph at ``inference::gqa_mixed_attention`` nodes
    (piecewise/utils.py:5-23), which the one-call form does not contain.
    Without ``kv_manager`` it defers to the wrapped HF module.
    """

    fuse_rope = True
    fuse_decode_attention = True

    def __init__(self, original_attn):
        super().__init__()
        if getattr(original_attn, "sliding_window", None) is not None:
            raise ValueError("sliding-window attention is not supported")
        self.original = original_attn
        self.layer_idx = original_attn.layer_idx
        self.num_heads = original_attn.config.num_attention_heads
        self.head_dim = original_attn.head_dim
        if abs(original_attn.scaling - self.head_dim ** -0.5) > 1e-12:
            raise ValueError("attention scaling must be head_dim ** -0.5")
        projs = (original_attn.q_proj, original_attn.k_proj, original_attn.v_proj)
        if any(p.bias is None for p in projs):
            raise ValueError("Qwen2 q/k/v projections carry biases")
        self.qkv_sizes = [p.out_features for p in projs]
        with torch.no_grad():
            self.register_buffer("qkv_weight", torch.cat([p.weight for p in projs]),
                                 persistent=False)
            self.register_buffer("qkv_bias", torch.cat([p.bias for p in projs]),
                                 persistent=False)

    def forward(self, hidden_states, position_embeddings, attention_mask=None,
                past_key_values=None, kv_manager=None, **kwargs):
        if kv_manager is None:
            return self.original(hidden_states, position_embeddings, attention_mask,
                                 past_key_values=past_key_values, **kwargs)
        metadata = kwargs.get("metadata")
        if metadata is None:
            raise ValueError("'metadata' is required with a custom kv_manager.")
        from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

        total_T = hidden_states.shape[1]
        shape = (1, total_T, -1, self.head_dim)
        qkv = torch.nn.functional.linear(hidden_states, self.qkv_weight, self.qkv_bias)
        cos, sin = position_embeddings
        layer = self.layer_idx
        if self.fuse_rope and self.fuse_decode_attention and metadata.full_decode:
            # RoPE, K/V write and decode attention: one launch
            o = rope_kv_decode_attention_op(qkv, cos, sin, kv_manager.keys[layer],
                                            kv_manager.values[layer], kv_manager.lens,
                                            metadata.slot_ids, kv_manager.block_table)
            return self.original.o_proj(o.reshape(1, total_T, self.num_heads * self.head_dim)), None
        if (self.fuse_rope and not metadata.full_decode
                and getattr(metadata, "fuse_mixed_attention", False)):
            # RoPE, K/V write and mixed attention: one call
            lens = getattr(metadata, "attn_lens", None)
            if lens is None:
                lens = kv_manager.lens[metadata.slot_ids]
            o = rope_kv_mixed_attention_op(qkv, cos, sin, kv_manager.keys[layer],
                                           kv_manager.values[layer], metadata.pages,
                                           metadata.offsets, max_seqlen=metadata.max_seqlen,
                                           cu_seqlens=metadata.cu_seqlens, kv_lens=lens,
                                           slot_ids=metadata.slot_ids,
                                           block_table=kv_manager.block_table)
            return self.original.o_proj(o.reshape(1, total_T, self.num_heads * self.head_dim)), None
        if self.fuse_rope:
            if metadata.full_decode:
                q = rope_kv_decode_update_op(qkv, cos, sin, kv_manager.keys[layer],
                                             kv_manager.values[layer], kv_manager.lens,
                                             metadata.slot_ids, kv_manager.block_table)
            else:
                q = rope_kv_mixed_update_op(qkv, cos, sin, kv_manager.keys[layer],
                                            kv_manager.values[layer], metadata.pages,
                                            metadata.offsets)
        else:
            q, k, v = qkv.split(self.qkv_sizes, dim=-1)
            q, k = apply_rotary_pos_emb(q.view(shape), k.view(shape), cos, sin, unsqueeze_dim=2)
            v = v.view(shape)
            if metadata.full_decode:
                kv_manager.decode_update(layer, metadata.slot_ids, k, v)
            else:
                kv_manager.mixed_update(layer, metadata.pages, metadata.offsets, k, v)
        lens = getattr(metadata, "attn_lens", None)
        if metadata.full_decode:
            if lens is None:
                lens = kv_manager.lens[metadata.slot_ids] + 1
            o = gqa_decode_attention_op(q, kv_manager.keys[layer], kv_manager.values[layer],
                                        lens, slot_ids=metadata.slot_ids,
                                        block_table=kv_manager.block_table)
        else:
            if lens is None:
                lens = kv_manager.lens[metadata.slot_ids]
            o = gqa_mixed_attention_op(q, kv_manager.keys[layer], kv_manager.values[layer],
                                       kv_lens=lens,
                                       max_seqlen=metadata.max_seqlen,
                                       cu_seqlens=metadata.cu_seqlens,
                                       slot_ids=metadata.slot_ids,
                                       block_table=kv_manager.block_table)
        out = self.original.o_proj(o.reshape(1, total_T, self.num_heads * self.head_dim))
        return out, None


def replace_attention(module):
    """Swap every HF ``Qwen2Attention`` under ``module`` for ``TritonQwen2Attention``."""
    from transformers.models.qwen2.modeling_qwen2 import Qwen2Attention

    for name, child in module.named_children():
        if isinstance(child, Qwen2Attention):
            setattr(module, name, TritonQwen2Attention(child))
        elif not isinstance(child, TritonQwen2Attention):
            replace_attention(child)


def use_triton_attention(model):
    """Route ``model``'s attention through the paged CUDA ops (idempotent)."""
    if not getattr(model, "_uses_triton_attention", False):
        replace_attention(model)
        model._uses_triton_attention = True


CudaQwen2Attention = TritonQwen2Attention
use_cuda_attention = use_triton_attention
