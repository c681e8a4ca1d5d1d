"""Static device buffers that describe one forward pass to the attention ops.

Same interface and padding rules as the reference's AttentionMetadata
(attn/metadata.py:3-55), so its scheduler modules can fill it unchanged:

* ``write_slot_ids`` pads with slot 0 (the padding slot; decode rows on slot 0
  read page 0 only, because ``lens[0]`` is kept at 0);
* ``write_cu_seqlens`` pads with its last value, so padded sequences have no
  tokens and the mixed kernel skips them;
* ``write_pages`` / ``write_offsets`` pad with 0: padded tokens all write
  page 0, offset 0 (the page that is never handed to a real slot).
"""
from __future__ import annotations

import torch


class AttentionMetadata:

    def __init__(self, token_count: int, full_decode: bool, device: torch.device):
        self.device = device
        self.slot_ids = None
        self.cu_seqlens = None
        self.pages = torch.zeros((token_count,), dtype=torch.long, device=device)
        self.offsets = torch.zeros((token_count,), dtype=torch.long, device=device)
        self.max_seqlen = token_count
        self.full_decode = full_decode
        # Optional, not in the reference: the attention lengths of this pass
        # (decode: lens[slot_ids] + 1, mixed: lens[slot_ids]) computed once by
        # the caller; when None every layer computes them from the KV storage.
        self.attn_lens = None
        # Optional, not in the reference: a mixed pass with this set runs its
        # RoPE, K/V write and attention as one call (rope_kv_mixed_attention);
        # left False, the pass keeps the reference's gqa_mixed_attention op,
        # which the reference's piecewise splitter cuts the graph at.
        self.fuse_mixed_attention = False

    def prepare_full_graph(self, batch_size: int):
        """Fixed-size slot / cu_seqlens buffers for a captured CUDA graph."""
        self.slot_ids = torch.zeros((batch_size,), dtype=torch.long, device=self.device)
        self.cu_seqlens = torch.zeros((batch_size + 1,), dtype=torch.long, device=self.device)

    @staticmethod
    def _fill(dst: torch.Tensor, values, pad_value) -> None:
        values = torch.as_tensor(values, dtype=torch.long, device=dst.device)
        n = len(values)
        dst[:n] = values
        dst[n:] = pad_value

    def write_slot_ids(self, ids):
        self._fill(self.slot_ids, ids, 0)

    def write_cu_seqlens(self, cu_seqlens):
        cu = torch.as_tensor(cu_seqlens, dtype=torch.long, device=self.cu_seqlens.device)
        self._fill(self.cu_seqlens, cu, cu[-1])

    def write_pages(self, pages):
        self._fill(self.pages, pages, 0)

    def write_offsets(self, offsets):
        self._fill(self.offsets, offsets, 0)
