"""Seeded synthetic inputs with the shapes of the reference's benchmark configs.

Every tensor follows the reference layouts: q ``(1, T, 14, 64)`` fp16, K/V
pools ``(n_pages, 2, 16, 64)`` fp16 with page 0 reserved for padding
(kv_cache/storage.py:32-56, scheduler/scheduler.py slot 0 / page 0), a
``(n_slots, n_pages)`` int64 block table whose row ``s`` lists slot ``s``'s
pages, and int64 ``lens`` / ``slot_ids`` / ``cu_seqlens``. No public dataset
is involved: values are N(0, 1) fp16 draws from a seeded generator.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Optional, Sequence

import numpy as np
import torch

H_Q, H_KV, HEAD_DIM, PAGE_SIZE = 14, 2, 64, 16


@dataclasses.dataclass
class DecodeCase:
    q: torch.Tensor            # (1, B, H_Q, D) fp16
    k: torch.Tensor            # (n_pages, H_KV, PAGE, D) fp16
    v: torch.Tensor
    lens: torch.Tensor         # (B,) int64, rows visible to each query
    slot_ids: torch.Tensor     # (B,) int64
    block_table: torch.Tensor  # (n_slots, n_pages) int64

    @property
    def batch(self) -> int:
        return int(self.slot_ids.shape[0])

    def algorithmic_bytes(self) -> int:
        """K/V rows read + q read + o written + block-table entries read."""
        L = self.lens.tolist()
        kv = sum(int(x) for x in L) * H_KV * HEAD_DIM * 2 * 2
        qo = self.batch * H_Q * HEAD_DIM * 2 * 2
        bt = sum(math.ceil(int(x) / PAGE_SIZE) for x in L) * 8
        return kv + qo + bt


@dataclasses.dataclass
class MixedCase:
    q: torch.Tensor            # (1, T, H_Q, D)
    k: torch.Tensor
    v: torch.Tensor
    max_seqlen: int
    cu_seqlens: torch.Tensor   # (B+1,)
    kv_lens: torch.Tensor      # (B,) rows already in the cache before the chunk
    slot_ids: torch.Tensor
    block_table: torch.Tensor

    def chunk_lens(self):
        cu = self.cu_seqlens.tolist()
        return [cu[i + 1] - cu[i] for i in range(len(cu) - 1)]

    def causal_flops(self) -> int:
        """4*D*H_Q per unmasked (query, key) pair: QK^T and PV, 2 flops/MAC."""
        pairs = 0
        for L, kv in zip(self.chunk_lens(), self.kv_lens.tolist()):
            pairs += L * int(kv) + L * (L + 1) // 2
        return 4 * HEAD_DIM * H_Q * pairs

    def algorithmic_bytes(self) -> int:
        kv = sum(int(kv) + L for L, kv in zip(self.chunk_lens(), self.kv_lens.tolist()))
        T = sum(self.chunk_lens())
        return kv * H_KV * HEAD_DIM * 2 * 2 + T * H_Q * HEAD_DIM * 2 * 2


def _paged_pool(lens_total: Sequence[int], seed: int, device, extra_pages: int = 0):
    """Pool + block table for len(lens_total) slots (slot 0 = padding).

    Slot ``b+1`` owns ``ceil(lens_total[b]/16)`` pages taken from a random
    permutation of pages ``1..n_pages-1``; page 0 is never handed out.
    The numpy PCG64 stream is platform-independent, so the same seed gives
    the same bytes on every host.
    """
    g = np.random.default_rng(seed)
    need = [math.ceil(int(x) / PAGE_SIZE) for x in lens_total]
    n_pages = sum(need) + 1 + extra_pages
    perm = torch.from_numpy(g.permutation(n_pages - 1).astype(np.int64)) + 1
    n_slots = len(lens_total) + 1
    block_table = torch.zeros((n_slots, n_pages), dtype=torch.int64)
    off = 0
    for b, n in enumerate(need):
        block_table[b + 1, :n] = perm[off:off + n]
        off += n
    return n_pages, block_table.to(device), g


def _randn(shape, g: np.random.Generator, device, on_device_gen: Optional[torch.Generator]):
    if on_device_gen is not None:
        return torch.randn(shape, generator=on_device_gen, device=device,
                           dtype=torch.float32).to(torch.float16)
    x = g.standard_normal(size=shape, dtype=np.float32).astype(np.float16)
    return torch.from_numpy(x).to(device)


def make_decode_case(lens: Sequence[int], seed: int = 0, device="cpu",
                     extra_pages: int = 0, generate_on_device: bool = False) -> DecodeCase:
    """Decode inputs: one query per sequence, sequence b in slot b+1."""
    lens = [int(x) for x in lens]
    B = len(lens)
    n_pages, bt, g = _paged_pool(lens, seed, device, extra_pages)
    dg = None
    if generate_on_device:
        dg = torch.Generator(device=device).manual_seed(seed + 1)
    q = _randn((1, B, H_Q, HEAD_DIM), g, device, dg)
    k = _randn((n_pages, H_KV, PAGE_SIZE, HEAD_DIM), g, device, dg)
    v = _randn((n_pages, H_KV, PAGE_SIZE, HEAD_DIM), g, device, dg)
    return DecodeCase(q=q, k=k, v=v,
                      lens=torch.tensor(lens, dtype=torch.int64, device=device),
                      slot_ids=torch.arange(1, B + 1, dtype=torch.int64, device=device),
                      block_table=bt)


def config1_lens(seed: int = 0, batch: int = 8, max_len: int = 2048):
    """Config 1: kv_lens ~ U[1, 2048] from torch.Generator seed 0."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(1, max_len + 1, (batch,), generator=g).tolist()


def make_mixed_case(chunk_lens: Sequence[int], kv_lens: Sequence[int], seed: int = 0,
                    device="cpu", max_seqlen: Optional[int] = None, pad_batch: int = 0,
                    generate_on_device: bool = False) -> MixedCase:
    """Mixed inputs: sequence b (slot b+1) has kv_lens[b] cached rows and a
    chunk of chunk_lens[b] new rows that are already written into the pool
    (mixed_update runs before the attention op, attn/core.py:217-233).

    ``pad_batch`` appends that many L=0 sequences on slot 0, the way
    AttentionMetadata.write_cu_seqlens pads (attn/metadata.py:39-43).
    ``max_seqlen`` defaults to the total token count (the bucket size).
    """
    chunk_lens = [int(x) for x in chunk_lens]
    kv_lens = [int(x) for x in kv_lens]
    totals = [a + b for a, b in zip(chunk_lens, kv_lens)]
    n_pages, bt, g = _paged_pool(totals, seed, device)
    T_used = sum(chunk_lens)
    T = max_seqlen if max_seqlen is not None else T_used
    assert T >= T_used
    dg = None
    if generate_on_device:
        dg = torch.Generator(device=device).manual_seed(seed + 1)
    q = _randn((1, T, H_Q, HEAD_DIM), g, device, dg)
    k = _randn((n_pages, H_KV, PAGE_SIZE, HEAD_DIM), g, device, dg)
    v = _randn((n_pages, H_KV, PAGE_SIZE, HEAD_DIM), g, device, dg)
    cu = [0]
    for L in chunk_lens:
        cu.append(cu[-1] + L)
    cu += [cu[-1]] * pad_batch
    slots = list(range(1, len(chunk_lens) + 1)) + [0] * pad_batch
    kvl = kv_lens + [0] * pad_batch
    return MixedCase(q=q, k=k, v=v, max_seqlen=T,
                     cu_seqlens=torch.tensor(cu, dtype=torch.int64, device=device),
                     kv_lens=torch.tensor(kvl, dtype=torch.int64, device=device),
                     slot_ids=torch.tensor(slots, dtype=torch.int64, device=device),
                     block_table=bt)


def config3_shape(seed: int = 0, n_seqs: int = 32, budget: int = 2048,
                  max_kv: int = 8192):
    """Config 3: L = 1 w.p. 0.5 else U[16, 512], drawn in order and clipped
    so that every later sequence keeps at least one token of the budget;
    kv_len ~ U[0, 8192]."""
    g = torch.Generator().manual_seed(seed)
    chunk, kv = [], []
    left = budget
    for i in range(n_seqs):
        if torch.rand((), generator=g).item() < 0.5:
            L = 1
        else:
            L = int(torch.randint(16, 513, (), generator=g).item())
        L = max(1, min(L, left - (n_seqs - i - 1)))
        chunk.append(L)
        left -= L
        kv.append(int(torch.randint(0, max_kv + 1, (), generator=g).item()))
    return chunk, kv
