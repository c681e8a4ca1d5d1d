"""Thin Python callers of the C ABI (``include/cie_attention.h``) on torch tensors.

These are what a ctypes binding of the library looks like: every call passes
raw device pointers, sizes and element strides, and runs on the given stream
(default: torch's current stream). Used by the parity tests and by the
benchmark's end-to-end leg; the torch ops in ``attn.core`` reach the same
entry points through ``_cie_torch_ops.so``.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import native


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _entry(name: str, block_table: torch.Tensor):
    """Entry point ``name``, or its ``_bt32`` variant for an int32 block table."""
    if block_table.dtype == torch.int32:
        name += "_bt32"
    elif block_table.dtype != torch.int64:
        raise TypeError(f"block_table must be int64 or int32, not {block_table.dtype}")
    return getattr(native.lib(), name)


def decode_workspace_bytes(batch: int, num_q_heads: int, head_dim: int, num_splits: int) -> int:
    return int(native.lib().cie_decode_workspace_bytes(batch, num_q_heads, head_dim, num_splits))


def decode_default_splits(batch: int, device: int = 0) -> int:
    return int(native.lib().cie_decode_default_splits(batch, device))


def decode_attention(q, k, v, lens, slot_ids, block_table, out=None, num_splits: int = 0,
                     workspace: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """cie_decode_attention on (1, B, H_q, D) q and (n_pages, H_kv, 16, D) pools."""
    B = slot_ids.shape[0]
    hq, d = q.shape[2], q.shape[3]
    S = num_splits if num_splits > 0 else decode_default_splits(B, q.device.index or 0)
    if out is None:
        out = torch.empty_like(q)
    need = decode_workspace_bytes(B, hq, d, S)
    if need > 0 and workspace is None:
        workspace = torch.empty(need // 4, dtype=torch.float32, device=q.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    st = _entry("cie_decode_attention", block_table)(
        _p(q), _p(k), _p(v), _p(lens), _p(slot_ids), _p(block_table), _p(out), _p(workspace),
        ws_bytes, B, hq, k.shape[1], d, k.shape[2], k.shape[0], block_table.shape[0],
        block_table.stride(0), k.stride(0), k.stride(1), S, native.stream_ptr(stream))
    native.check(st, "cie_decode_attention")
    return out


def decode_attention_noalloc(q, k, v, lens, slot_ids, block_table, out=None,
                             num_splits: int = 0, stream=None) -> torch.Tensor:
    """cie_decode_attention_noalloc: same result, split scratch inside the library."""
    if out is None:
        out = torch.empty_like(q)
    st = native.lib().cie_decode_attention_noalloc(
        _p(q), _p(k), _p(v), _p(lens), _p(slot_ids), _p(block_table), _p(out),
        slot_ids.shape[0], q.shape[2], k.shape[1], q.shape[3], k.shape[2], k.shape[0],
        block_table.shape[0], block_table.stride(0), k.stride(0), k.stride(1), num_splits,
        native.stream_ptr(stream))
    native.check(st, "cie_decode_attention_noalloc")
    return out


def mixed_workspace_bytes(batch: int, total_tokens: int, num_kv_heads: int = 2,
                          num_splits: int = 0, device: int = 0) -> int:
    return int(native.lib().cie_mixed_workspace_bytes(batch, total_tokens, num_kv_heads,
                                                        num_splits, device))


def mixed_attention(q, k, v, max_seqlen: int, cu_seqlens, kv_lens, slot_ids, block_table,
                    out=None, num_splits: int = 0, workspace: Optional[torch.Tensor] = None,
                    stream=None) -> torch.Tensor:
    """cie_mixed_attention; rows outside every sequence are left as they were in ``out``."""
    B = slot_ids.shape[0]
    T = q.shape[1]
    if out is None:
        out = torch.empty_like(q)
    if workspace is None:
        need = mixed_workspace_bytes(B, T, k.shape[1], num_splits, q.device.index or 0)
        workspace = torch.empty(max(need // 4, 1), dtype=torch.float32, device=q.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    st = _entry("cie_mixed_attention", block_table)(
        _p(q), _p(k), _p(v), int(max_seqlen), _p(cu_seqlens), _p(kv_lens), _p(slot_ids),
        _p(block_table), _p(out), _p(workspace), ws_bytes, B, T, q.shape[2], k.shape[1],
        q.shape[3], k.shape[2], k.shape[0], block_table.shape[0], block_table.stride(0),
        k.stride(0), k.stride(1), num_splits, native.stream_ptr(stream))
    native.check(st, "cie_mixed_attention")
    return out


def kv_decode_update(k_cache, v_cache, lens, slot_ids, block_table, k_new, v_new,
                     stream=None) -> None:
    """cie_kv_decode_update; ``lens`` is the per-slot length tensor (n_slots,)."""
    st = _entry("cie_kv_decode_update", block_table)(
        _p(k_cache), _p(v_cache), _p(lens), _p(slot_ids), _p(block_table), _p(k_new), _p(v_new),
        slot_ids.shape[0], k_cache.shape[1], k_cache.shape[3], k_cache.shape[2],
        k_cache.shape[0], min(lens.shape[0], block_table.shape[0]), block_table.stride(0),
        k_cache.stride(0), k_cache.stride(1), k_new.stride(1), k_new.stride(2), v_new.stride(1),
        v_new.stride(2), native.stream_ptr(stream))
    native.check(st, "cie_kv_decode_update")


def kv_mixed_update(k_cache, v_cache, pages, offsets, k_new, v_new, stream=None) -> None:
    """cie_kv_mixed_update: token t -> (pages[t], offsets[t])."""
    st = native.lib().cie_kv_mixed_update(
        _p(k_cache), _p(v_cache), _p(pages), _p(offsets), _p(k_new), _p(v_new), pages.shape[0],
        k_cache.shape[1], k_cache.shape[3], k_cache.shape[2], k_cache.shape[0],
        k_cache.stride(0), k_cache.stride(1), k_new.stride(1), k_new.stride(2), v_new.stride(1),
        v_new.stride(2), native.stream_ptr(stream))
    native.check(st, "cie_kv_mixed_update")


def _rope_q_out(qkv, k_cache, out):
    d, hkv = k_cache.shape[3], k_cache.shape[1]
    hq = qkv.shape[-1] // d - 2 * hkv
    if out is None:
        out = torch.empty((1, qkv.shape[1], hq, d), dtype=qkv.dtype, device=qkv.device)
    return out, hq


def rope_kv_decode_update(qkv, cos, sin, k_cache, v_cache, lens, slot_ids, block_table,
                          out=None, stream=None):
    """cie_rope_kv_decode_update: rotated q (returned) and the token's rotated k / v
    written at its slot's current length."""
    out, hq = _rope_q_out(qkv, k_cache, out)
    st = _entry("cie_rope_kv_decode_update", block_table)(
        _p(qkv), qkv.stride(1), _p(cos), _p(sin), cos.stride(1), _p(out), _p(k_cache),
        _p(v_cache), _p(lens), _p(slot_ids), _p(block_table), slot_ids.shape[0], hq,
        k_cache.shape[1], k_cache.shape[3], k_cache.shape[2], k_cache.shape[0],
        min(lens.shape[0], block_table.shape[0]), block_table.stride(0), k_cache.stride(0),
        k_cache.stride(1), native.stream_ptr(stream))
    native.check(st, "cie_rope_kv_decode_update")
    return out


def rope_kv_mixed_update(qkv, cos, sin, k_cache, v_cache, pages, offsets, out=None,
                         stream=None):
    """cie_rope_kv_mixed_update: rotated q (returned); token t's rotated k / v to
    (pages[t], offsets[t])."""
    out, hq = _rope_q_out(qkv, k_cache, out)
    st = native.lib().cie_rope_kv_mixed_update(
        _p(qkv), qkv.stride(1), _p(cos), _p(sin), cos.stride(1), _p(out), _p(k_cache),
        _p(v_cache), _p(pages), _p(offsets), pages.shape[0], hq, k_cache.shape[1],
        k_cache.shape[3], k_cache.shape[2], k_cache.shape[0], k_cache.stride(0),
        k_cache.stride(1), native.stream_ptr(stream))
    native.check(st, "cie_rope_kv_mixed_update")
    return out


def rope_kv_decode_attention(qkv, cos, sin, k_cache, v_cache, lens, slot_ids, block_table,
                             out=None, num_splits: int = 0, workspace=None, stream=None):
    """cie_rope_kv_decode_attention: rotary embedding, K/V write of each token
    at its slot's current length (``lens`` per slot, not advanced) and decode
    attention over the slot's keys including the new one, in one launch."""
    out, hq = _rope_q_out(qkv, k_cache, out)
    B = slot_ids.shape[0]
    d = k_cache.shape[3]
    S = num_splits if num_splits > 0 else decode_default_splits(B, qkv.device.index or 0)
    need = decode_workspace_bytes(B, hq, d, S)
    if need > 0 and workspace is None:
        workspace = torch.empty(need // 4, dtype=torch.float32, device=qkv.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    st = _entry("cie_rope_kv_decode_attention", block_table)(
        _p(qkv), qkv.stride(1), _p(cos), _p(sin), cos.stride(1), _p(k_cache), _p(v_cache),
        _p(lens), _p(slot_ids), _p(block_table), _p(out), _p(workspace), ws_bytes, B, hq,
        k_cache.shape[1], d, k_cache.shape[2], k_cache.shape[0],
        min(lens.shape[0], block_table.shape[0]), block_table.stride(0), k_cache.stride(0),
        k_cache.stride(1), S, native.stream_ptr(stream))
    native.check(st, "cie_rope_kv_decode_attention")
    return out


def lm_head_argmax(hidden, weight, logits: bool = False, stream=None):
    """cie_lm_head_argmax: greedy tokens (int64, one per hidden row) of
    hidden (B, H) . weight (V, H)^T; with ``logits`` also the fp16 logits (B, V)."""
    B, H = hidden.shape
    V = weight.shape[0]
    dev = hidden.device
    tokens = torch.empty(B, dtype=torch.int64, device=dev)
    out = torch.empty(B, V, dtype=torch.float16, device=dev) if logits else None
    need = int(native.lib().cie_lm_head_argmax_workspace_bytes(B, V, dev.index or 0))
    ws = torch.empty(max(need // 8, 1), dtype=torch.int64, device=dev)
    st = native.lib().cie_lm_head_argmax(
        _p(hidden), hidden.stride(0), _p(weight), weight.stride(0), B, H, V, _p(out), V,
        _p(tokens), _p(ws), ws.numel() * 8, native.stream_ptr(stream))
    native.check(st, "cie_lm_head_argmax")
    return (tokens, out) if logits else tokens


def rope_kv_mixed_attention(qkv, cos, sin, k_cache, v_cache, pages, offsets, max_seqlen: int,
                            cu_seqlens, kv_lens, slot_ids, block_table, out=None,
                            num_splits: int = 0, stream=None):
    """cie_rope_kv_mixed_attention: token t's rotated k and its v written to
    (pages[t], offsets[t]), then the mixed attention of the pass over the pages
    (q rotated on the way); returns o (1, T, H_q, D)."""
    out, hq = _rope_q_out(qkv, k_cache, out)
    B, T = slot_ids.shape[0], qkv.shape[1]
    dev = qkv.device
    need = int(native.lib().cie_rope_kv_mixed_workspace_bytes(B, T, hq, k_cache.shape[1],
                                                                num_splits, dev.index or 0))
    ws = torch.empty(max(need // 4, 1) + 1, dtype=torch.float32, device=dev)
    st = _entry("cie_rope_kv_mixed_attention", block_table)(
        _p(qkv), qkv.stride(1), _p(cos), _p(sin), cos.stride(1), _p(k_cache), _p(v_cache),
        _p(pages), _p(offsets), int(max_seqlen), _p(cu_seqlens), _p(kv_lens), _p(slot_ids),
        _p(block_table), _p(out), _p(ws), ws.numel() * 4, B, T, hq, k_cache.shape[1],
        k_cache.shape[3], k_cache.shape[2], k_cache.shape[0], block_table.shape[0],
        block_table.stride(0), k_cache.stride(0), k_cache.stride(1), num_splits,
        native.stream_ptr(stream))
    native.check(st, "cie_rope_kv_mixed_attention")
    return out
