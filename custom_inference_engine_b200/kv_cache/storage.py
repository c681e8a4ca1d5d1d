"""Paged K/V pools with the reference KVStorage interface (kv_cache/storage.py:4-141).

Layout per layer: ``(n_pages, H_kv, page_size, head_dim)`` for K and for V,
``n_pages = ceil(max_cache_len / page_size)``; ``lens (n_slots,)`` int64,
``block_table (n_slots, n_pages)`` int64 (or int32, ``block_table_dtype``) and
``last_generated (n_slots,)``.
Slot 0 and page 0 are padding. ``decode_update`` / ``mixed_update`` are the
mutating ops ``inference::kv_decode_update`` / ``inference::kv_mixed_update``
(one CUDA launch each for K and V of every token and head); Dynamo sees them
as opaque in-place ops, so they can be captured in CUDA graphs.
"""
from __future__ import annotations

import math

import torch

from custom_inference_engine_b200 import native

native.load_ops()
_decode_update = torch.ops.inference.kv_decode_update.default
_mixed_update = torch.ops.inference.kv_mixed_update.default


class KVStorage:

    def __init__(self, config, max_cache_len, page_size, n_slots, device, dtype, *,
                 block_table_dtype=torch.int64):
        """``block_table_dtype`` (keyword only, not in the reference): int64, the
        reference's layout, or int32 (half the bytes per entry; every op of this
        package takes either)."""
        if block_table_dtype not in (torch.int64, torch.int32):
            raise ValueError(f"block_table_dtype must be int64 or int32, not {block_table_dtype}")
        self.config = config
        self.max_cache_len = max_cache_len
        self.page_size = page_size
        self.n_slots = n_slots
        self.device = device
        self.dtype = dtype

        self.n_pages = math.ceil(max_cache_len / page_size)
        self.unused_idx = 0

        self.num_layers = config.num_hidden_layers
        self.num_q_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.head_dim = getattr(config, "head_dim",
                                config.hidden_size // config.num_attention_heads)

        shape = (self.n_pages, self.num_kv_heads, self.page_size, self.head_dim)
        self.keys = [torch.zeros(shape, device=device, dtype=dtype)
                     for _ in range(self.num_layers)]
        self.values = [torch.zeros(shape, device=device, dtype=dtype)
                       for _ in range(self.num_layers)]
        self.lens = torch.zeros((n_slots,), dtype=torch.long, device=device)
        self.block_table = torch.zeros((n_slots, self.n_pages), dtype=block_table_dtype,
                                       device=device)
        self.last_generated = torch.zeros((n_slots,), dtype=torch.long, device=device)

    def mixed_update(self, layer_num: int, pages: torch.Tensor, offsets: torch.Tensor,
                     k_proj: torch.Tensor, v_proj: torch.Tensor) -> None:
        """Token t's K/V rows -> (pages[t], :, offsets[t]) of layer ``layer_num``."""
        _mixed_update(self.keys[layer_num], self.values[layer_num], pages, offsets,
                      k_proj, v_proj)

    def decode_update(self, layer_num: int, slot_ids: torch.Tensor, k_proj: torch.Tensor,
                      v_proj: torch.Tensor) -> None:
        """Each slot's new token -> page block_table[slot, lens//16], offset lens%16."""
        _decode_update(self.keys[layer_num], self.values[layer_num], self.lens, slot_ids,
                       self.block_table, k_proj, v_proj)

    # The padding slot's length is reset with an in-place fill of a one-element
    # slice rather than ``lens[0] = 0``: the latter copies a host scalar, which a
    # CUDA graph capture rejects.
    def decode_advance(self, slot_ids: torch.Tensor) -> None:
        self.lens[slot_ids] += 1
        self.lens[self.unused_idx:self.unused_idx + 1].zero_()

    def mixed_advance(self, slot_ids: torch.Tensor, lens: torch.Tensor) -> None:
        self.lens[slot_ids] += lens
        self.lens[self.unused_idx:self.unused_idx + 1].zero_()

    def reset(self, slot_ids) -> None:
        self.lens[slot_ids] = 0
        self.block_table[slot_ids] = 0
