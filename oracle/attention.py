"""CPU restatement of the reference engine's paged GQA attention path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the
CUDA kernels, never the thing measured or shipped.

Two families of functions live here:

* ``*_fp32``: the plain "reference math" -- gather the sequence's pages
  through ``block_table``, then fp32 ``softmax(Q K^T * D**-0.5) V`` with a
  causal limit at ``kv_len + i`` for mixed rows. This is the tolerance
  oracle (max-abs 2e-3 on fp16 outputs) and the timed CPU baseline.
* ``*_blockwise``: a step-for-step restatement of the reference Triton
  kernels' block loop (online softmax, scale applied after the fp16 dot,
  probabilities rounded to fp16 before P.V, the split-KV merge). It is
  pinned against fixtures produced by the reference kernels themselves
  (``tests/golden/make_golden.py``) and documents exactly what rounding the
  reference performs.
* ``*_update_ref``: the KV-page scatter, bit-exact.
* ``rope_ref``: the rotary embedding the reference applies to q and k
  before the scatter, in fp16 as its torch ops round.

All citations are ``path:line`` inside the reference project
(eteboun/custom_inference_engine).

Tensor conventions (identical to the reference):
  q            (1, T, H_Q, D) fp16
  k, v pools   (n_pages, H_KV, PAGE_SIZE, D) fp16
  block_table  (n_slots, n_pages) int64
  lens / kv_lens / slot_ids (B,) int64, cu_seqlens (B+1,) int64
"""
from __future__ import annotations

import math

import torch

H_Q = 14
H_KV = 2
GROUP = H_Q // H_KV
HEAD_DIM = 64
PAGE_SIZE = 16
# attn/core.py:148 asserts scaling == head_dim ** -0.5; the kernels multiply
# the fp32 dot by D ** -0.5 (kernels/decode_attention.py:123).
SCALE = HEAD_DIM ** -0.5


def _gather_pages(pool: torch.Tensor, block_table: torch.Tensor, slot: int,
                  n_keys: int) -> torch.Tensor:
    """Rows ``0..n_keys-1`` of one slot's paged K or V as (H_kv, n_keys, D).

    Follows the row -> (block_table[slot, row // PAGE_SIZE], row % PAGE_SIZE)
    addressing of kernels/decode_attention.py:76-111 and
    kernels/prefill_attention.py:95-131.
    """
    page_size = pool.shape[2]
    n_pages = (n_keys + page_size - 1) // page_size
    pages = block_table[slot, :n_pages]
    g = pool[pages]                                   # (n, H_kv, P, D)
    g = g.permute(1, 0, 2, 3).reshape(pool.shape[1], n_pages * page_size,
                                      pool.shape[3])
    return g[:, :n_keys]


# --------------------------------------------------------------------------
# Plain fp32 reference math (the tolerance oracle / CPU baseline)
# --------------------------------------------------------------------------

def decode_attention_fp32(q, k, v, lens, slot_ids, block_table):
    """fp32 softmax attention of one query token per sequence.

    Semantics of attn/core.py:13-66 + kernels/decode_attention.py:12-272:
    sequence b attends to rows ``[0, lens[b])`` of slot ``slot_ids[b]``; a
    sequence with ``lens[b] == 0`` outputs zeros (the merge guard at
    kernels/decode_attention.py:260-264).
    """
    _, T, hq, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    B = slot_ids.shape[0]
    assert T == B
    out = torch.zeros((1, T, hq, d), dtype=torch.float32)
    lens_l = lens.tolist()
    slots_l = slot_ids.tolist()
    for b in range(B):
        L = int(lens_l[b])
        if L <= 0:
            continue
        kk = _gather_pages(k, block_table, slots_l[b], L).float()
        vv = _gather_pages(v, block_table, slots_l[b], L).float()
        qq = q[0, b].float().view(hkv, g, d)
        s = torch.matmul(qq, kk.transpose(1, 2)) * SCALE     # (hkv, g, L)
        p = torch.softmax(s, dim=-1)
        out[0, b] = torch.matmul(p, vv).reshape(hq, d)
    return out.to(torch.float16)


def mixed_attention_fp32(q, k, v, max_seqlen, cu_seqlens, kv_lens, slot_ids,
                         block_table):
    """fp32 causal varlen attention for chunked prefill + decode rows.

    Semantics of attn/core.py:69-111 + kernels/prefill_attention.py:10-198:
    token ``i`` of sequence ``b`` (global row ``cu_seqlens[b] + i``) sits at
    position ``kv_lens[b] + i`` and attends to keys ``0 .. kv_lens[b] + i``.
    Rows that belong to no sequence are never written by the reference
    (``o = torch.empty_like(q)``); here they are returned as zeros and
    ``valid_token_rows`` tells the caller which rows are defined.
    """
    _, T, hq, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    B = slot_ids.shape[0]
    out = torch.zeros((1, T, hq, d), dtype=torch.float32)
    cu = cu_seqlens.tolist()
    kvl = kv_lens.tolist()
    slots = slot_ids.tolist()
    for b in range(B):
        start, end = int(cu[b]), int(cu[b + 1])
        L = end - start
        if L <= 0:
            continue
        n_keys = int(kvl[b]) + L
        kk = _gather_pages(k, block_table, slots[b], n_keys).float()
        vv = _gather_pages(v, block_table, slots[b], n_keys).float()
        qq = q[0, start:end].float().view(L, hkv, g, d).permute(1, 0, 2, 3)
        qq = qq.reshape(hkv, L * g, d)
        s = torch.matmul(qq, kk.transpose(1, 2)) * SCALE     # (hkv, L*g, keys)
        pos = int(kvl[b]) + torch.arange(L).repeat_interleave(g)
        keys = torch.arange(n_keys)
        s = s.masked_fill(keys[None, None, :] > pos[None, :, None],
                          float("-inf"))
        p = torch.softmax(s, dim=-1)
        o = torch.matmul(p, vv).view(hkv, L, g, d).permute(1, 0, 2, 3)
        out[0, start:end] = o.reshape(L, hq, d)
    return out.to(torch.float16)


def valid_token_rows(cu_seqlens, T: int) -> torch.Tensor:
    """Bool mask (T,) of rows written by the mixed kernel (rows inside some
    ``[cu_seqlens[b], cu_seqlens[b+1])``)."""
    cu = cu_seqlens.tolist()
    m = torch.zeros(T, dtype=torch.bool)
    for b in range(len(cu) - 1):
        if cu[b + 1] > cu[b]:
            m[cu[b]:cu[b + 1]] = True
    return m


# --------------------------------------------------------------------------
# Step-for-step restatement of the reference Triton kernels
# --------------------------------------------------------------------------

def _dot_f16_f32(a16: torch.Tensor, b16: torch.Tensor) -> torch.Tensor:
    """``tl.dot`` of fp16 operands with fp32 accumulation: products of fp16
    values are exact in fp32; sums are fp32."""
    return torch.matmul(a16.float(), b16.float())


def decode_attention_blockwise(q, k, v, lens, slot_ids, block_table,
                               num_programs: int = 16, block_n: int = 16):
    """Restates decode_gqa_attention_kernel_load + _merge.

    Load (kernels/decode_attention.py:33-179): program (p, h_kv, b) visits
    row blocks ``start = p*BN, p*BN + P*BN, ...`` below L (:71-75), computes
    ``S = dot(q, k^T) * D**-0.5`` in fp32 (:114-125), updates the running
    max ``m``, ``l = l*alpha + sum(exp(S - m_new))`` and
    ``acc = acc*alpha + dot(fp16(P), V)`` (:127-141).
    Merge (:196-272): ``O = sum_p e^{m_p-M} acc_p / sum_p e^{m_p-M} l_p``,
    zero when every ``m_p`` is -inf.
    """
    _, T, hq, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    B = slot_ids.shape[0]
    P = num_programs
    out = torch.zeros((1, T, hq, d), dtype=torch.float16)
    for b in range(B):
        L = int(lens[b])
        slot = int(slot_ids[b])
        for h in range(hkv):
            qh = q[0, b, h * g:(h + 1) * g]                  # (g, d) fp16
            kk = _gather_pages(k, block_table, slot, max(L, 0))[h] if L > 0 else None
            vv = _gather_pages(v, block_table, slot, max(L, 0))[h] if L > 0 else None
            ms, ls, accs = [], [], []
            for p in range(P):
                m = torch.full((g,), float("-inf"))
                l = torch.zeros(g)
                acc = torch.zeros(g, d)
                for start in range(p * block_n, L, P * block_n):
                    stop = min(start + block_n, L)
                    s = _dot_f16_f32(qh, kk[start:stop].T) * SCALE
                    m_new = torch.maximum(m, s.max(dim=1).values)
                    pr = torch.exp(s - m_new[:, None])
                    alpha = torch.exp(m - m_new)
                    l = l * alpha + pr.sum(dim=1)
                    acc = acc * alpha[:, None] + _dot_f16_f32(
                        pr.to(torch.float16), vv[start:stop])
                    m = m_new
                ms.append(m)
                ls.append(l)
                accs.append(acc)
            M = torch.stack(ms)                                 # (P, g)
            Lp = torch.stack(ls)
            A = torch.stack(accs)                               # (P, g, d)
            mx = M.max(dim=0).values
            finite = torch.isfinite(mx)
            safe = torch.where(finite, mx, torch.zeros_like(mx))
            alpha = torch.exp(M - safe[None])
            num = (A * alpha[:, :, None]).sum(0)
            den = (Lp * alpha).sum(0)
            o = torch.where(finite[:, None], num / den[:, None],
                            torch.zeros_like(num))
            out[0, b, h * g:(h + 1) * g] = o.to(torch.float16)
    return out


def mixed_attention_blockwise(q, k, v, max_seqlen, cu_seqlens, kv_lens,
                              slot_ids, block_table, block_m: int = 16,
                              block_n: int = 64):
    """Restates mixed_gqa_attention_kernel (kernels/prefill_attention.py).

    Program (t, h_kv, b) exits when ``t*BM >= L`` (:49-50); otherwise it loops
    key blocks of BN from 0 to ``kv_len + min(L, (t+1)*BM)`` (:87-93), masks
    ``key > kv_len + row`` (:145-155), runs the online softmax with fp32 ``l``
    and fp16-rounded P for the P.V dot (:157-184) and stores ``acc / l``
    (:187-198). Rows outside any sequence stay zero here.
    """
    _, T, hq, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    B = slot_ids.shape[0]
    out = torch.zeros((1, T, hq, d), dtype=torch.float16)
    for b in range(B):
        s0, s1 = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
        L = s1 - s0
        kv_len = int(kv_lens[b])
        slot = int(slot_ids[b])
        if L <= 0:
            continue
        n_keys = kv_len + L
        for h in range(hkv):
            kk = _gather_pages(k, block_table, slot, n_keys)[h]
            vv = _gather_pages(v, block_table, slot, n_keys)[h]
            for t in range(math.ceil(max_seqlen / block_m)):
                if t * block_m >= L:
                    break
                r0, r1 = t * block_m, min((t + 1) * block_m, L)
                qt = q[0, s0 + r0:s0 + r1, h * g:(h + 1) * g]     # (R, g, d)
                R = r1 - r0
                qt = qt.reshape(R * g, d)
                pos = kv_len + torch.arange(r0, r1).repeat_interleave(g)
                end = kv_len + min(L, (t + 1) * block_m)
                m = torch.full((R * g,), float("-inf"))
                l = torch.zeros(R * g)
                acc = torch.zeros(R * g, d)
                for start in range(0, end, block_n):
                    stop = min(start + block_n, n_keys)
                    keys = torch.arange(start, stop)
                    s = _dot_f16_f32(qt, kk[start:stop].T) * SCALE
                    s = s.masked_fill(keys[None, :] > pos[:, None], float("-inf"))
                    m_new = torch.maximum(m, s.max(dim=1).values)
                    alpha = torch.exp(m - m_new)
                    pr = torch.exp(s - m_new[:, None])
                    l = l * alpha + pr.sum(dim=1)
                    acc = acc * alpha[:, None] + _dot_f16_f32(
                        pr.to(torch.float16), vv[start:stop])
                    m = m_new
                o = (acc / l[:, None]).view(R, g, d)
                out[0, s0 + r0:s0 + r1, h * g:(h + 1) * g] = o.to(torch.float16)
    return out


# --------------------------------------------------------------------------
# KV page scatter (bit-exact)
# --------------------------------------------------------------------------

def decode_update_ref(k_cache, v_cache, lens, slot_ids, block_table, k_proj,
                      v_proj):
    """KVStorage.decode_update (kv_cache/storage.py:87-122), in place.

    ``lens`` is the full per-slot length tensor (``KVStorage.lens``); the new
    token of ``slot_ids[i]`` lands at page ``block_table[slot, lens//16]``,
    offset ``lens % 16``. ``k_proj``/``v_proj`` are (1, B, H_kv, D) and may be
    strided views.
    """
    page_size = k_cache.shape[2]
    hkv, d = k_cache.shape[1], k_cache.shape[3]
    ln = lens[slot_ids]
    pages = block_table[slot_ids, ln // page_size]
    starts = ln % page_size
    k_cache[pages, :, starts] = k_proj.reshape(-1, hkv, d)
    v_cache[pages, :, starts] = v_proj.reshape(-1, hkv, d)


def mixed_update_ref(k_cache, v_cache, pages, offsets, k_proj, v_proj):
    """KVStorage.mixed_update (kv_cache/storage.py:62-85), in place."""
    hkv, d = k_cache.shape[1], k_cache.shape[3]
    k_cache[pages, :, offsets] = k_proj.reshape(-1, hkv, d)
    v_cache[pages, :, offsets] = v_proj.reshape(-1, hkv, d)


# --------------------------------------------------------------------------
# rotary embedding before the scatter
# --------------------------------------------------------------------------

def rope_ref(x, cos, sin):
    """The rotary embedding of ``x`` (1, T, H, D) fp16 with per-token tables
    ``cos`` / ``sin`` (1, T, D) fp16, as the reference applies it to the
    split QKV projection before the KV write (attn/core.py:193-198, through
    transformers' Qwen2 ``apply_rotary_pos_emb`` with ``unsqueeze_dim=2``):
    ``x * cos + rotate_half(x) * sin`` where ``rotate_half`` maps the halves
    (x1, x2) to (-x2, x1). Every op rounds to fp16 the way torch's half
    arithmetic does (product, product, sum)."""
    c = cos.unsqueeze(2)
    s = sin.unsqueeze(2)
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * c + rot * s
