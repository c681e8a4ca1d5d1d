"""RoPE + K/V write + mixed attention as one call (cie_rope_kv_mixed_attention,
inference::rope_kv_mixed_attention).

It must give the bits of the two-call sequence it replaces -- the fused RoPE +
K/V write (cie_rope_kv_mixed_update, bit-identical to HF's apply_rotary_pos_emb
+ KVStorage.mixed_update, attn/core.py:193-206 of the reference) followed by the
mixed attention op (attn/core.py:217-233) -- for the output and for every page
(page 0, where padding tokens collide, excluded), with int64 and int32 block
tables; and a model whose mixed passes use it must give the same greedy tokens.
"""
import pytest
import torch

from custom_inference_engine_b200 import cabi, native
from custom_inference_engine_b200 import model_runner as MR
from custom_inference_engine_b200 import workloads as W
from custom_inference_engine_b200.attn import core

pytestmark = pytest.mark.gpu
HQ, HKV, D, PAGE = 14, 2, 64, 16


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    native.device_errors(0, clear=True)
    yield
    assert native.device_errors(0, clear=True) == 0


def _pass(chunks, kv_lens, seed, dev, pad_tokens=0, pad_batch=0):
    """A mixed pass: pools holding each sequence's cached rows, the fused QKV
    rows and rotary tables of the pass's tokens, and the metadata the
    reference writes (pages / offsets of token positions through the block
    table; padding tokens on page 0, offset 0)."""
    T = sum(chunks) + pad_tokens
    m = W.make_mixed_case(chunks, kv_lens, seed=seed, device=dev, max_seqlen=T,
                          pad_batch=pad_batch, generate_on_device=True)
    g = torch.Generator(device=dev).manual_seed(seed + 7)
    qkv = torch.randn(1, T, (HQ + 2 * HKV) * D, generator=g, device=dev).half()
    pos = torch.zeros(T, dtype=torch.long, device=dev)
    pages = torch.zeros(T, dtype=torch.long, device=dev)
    o = 0
    for b, (L, kv) in enumerate(zip(chunks, kv_lens)):
        p = torch.arange(kv, kv + L, device=dev)
        pos[o:o + L] = p
        pages[o:o + L] = m.block_table[b + 1, p // PAGE]
        o += L
    offsets = pos % PAGE
    offsets[sum(chunks):] = 0
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=dev).float() / D))
    emb = torch.cat([pos[:, None].float() * inv] * 2, dim=-1)
    cos, sin = emb.cos()[None].half(), emb.sin()[None].half()
    return m, qkv, cos, sin, pages, offsets


CASES = {
    "small": ([1, 40, 130, 1], [9, 0, 200, 3000], 0, 0),
    "padded": ([17, 1, 64], [100, 37, 0], 15, 2),
    "chunks_512": ([512, 512], [1500, 7000], 0, 0),
    "config3": tuple(W.config3_shape(seed=0)) + (0, 0),
}


@pytest.mark.parametrize("name", list(CASES))
@pytest.mark.parametrize("table_dtype", [torch.int64, torch.int32])
def test_one_call_matches_the_two_call_sequence(name, table_dtype, cuda_device):
    chunks, kv_lens, pad_tokens, pad_batch = CASES[name]
    m, qkv, cos, sin, pages, offsets = _pass(chunks, kv_lens, 11, cuda_device, pad_tokens,
                                             pad_batch)
    bt = m.block_table.to(table_dtype)
    k1, v1 = m.k.clone(), m.v.clone()
    q = core.rope_kv_mixed_update_op(qkv, cos, sin, k1, v1, pages, offsets)
    want = core.gqa_mixed_attention_op(q, k1, v1, max_seqlen=m.max_seqlen,
                                       cu_seqlens=m.cu_seqlens, kv_lens=m.kv_lens,
                                       slot_ids=m.slot_ids, block_table=bt)
    k2, v2 = m.k.clone(), m.v.clone()
    got = core.rope_kv_mixed_attention_op(qkv, cos, sin, k2, v2, pages, offsets,
                                          max_seqlen=m.max_seqlen, cu_seqlens=m.cu_seqlens,
                                          kv_lens=m.kv_lens, slot_ids=m.slot_ids,
                                          block_table=bt)
    rows = sum(chunks)   # rows past the last sequence are left as they were
    assert torch.equal(got[0, :rows], want[0, :rows])
    assert torch.equal(k2[1:], k1[1:]) and torch.equal(v2[1:], v1[1:])
    # the C ABI, with the split count fixed
    k3, v3 = m.k.clone(), m.v.clone()
    q3 = cabi.rope_kv_mixed_update(qkv, cos, sin, k3, v3, pages, offsets)
    want3 = cabi.mixed_attention(q3, k3, v3, m.max_seqlen, m.cu_seqlens, m.kv_lens, m.slot_ids,
                                 bt, num_splits=2)
    k4, v4 = m.k.clone(), m.v.clone()
    got4 = cabi.rope_kv_mixed_attention(qkv, cos, sin, k4, v4, pages, offsets, m.max_seqlen,
                                        m.cu_seqlens, m.kv_lens, m.slot_ids, bt, num_splits=2)
    assert torch.equal(got4[0, :rows], want3[0, :rows])
    assert torch.equal(k4[1:], k3[1:]) and torch.equal(v4[1:], v3[1:])


def test_a_pass_without_sequences_still_writes_its_rows(cuda_device):
    m, qkv, cos, sin, pages, offsets = _pass([5, 9], [3, 40], 5, cuda_device)
    k1, v1 = m.k.clone(), m.v.clone()
    core.rope_kv_mixed_update_op(qkv, cos, sin, k1, v1, pages, offsets)
    k2, v2 = m.k.clone(), m.v.clone()
    empty = m.cu_seqlens.new_zeros(1)
    core.rope_kv_mixed_attention_op(qkv, cos, sin, k2, v2, pages, offsets,
                                    max_seqlen=m.max_seqlen, cu_seqlens=empty,
                                    kv_lens=m.kv_lens[:0], slot_ids=m.slot_ids[:0],
                                    block_table=m.block_table)
    assert torch.equal(k2[1:], k1[1:]) and torch.equal(v2[1:], v1[1:])


def test_runner_tokens_with_one_call_mixed_passes(cuda_device):
    cfg = MR.qwen2_config(num_hidden_layers=2, vocab_size=4096, intermediate_size=2048)
    model = MR.random_qwen2(cfg, seed=0, device=cuda_device)
    prompts = [list(range(5, 5 + n)) for n in (5, 40, 130, 1)]
    out = {}
    for fused in (True, False):
        runner = MR.PagedRunner(model, max_cache_len=2048, n_slots=5, token_budget=64,
                                fused_mixed_attention=fused)
        slots = [1, 2, 3, 4]
        for s, p in zip(slots, prompts):
            runner.admit(s, len(p) + 10)
        pre = runner.prefill(slots, prompts)
        # a mixed pass with decode rows
        nxt = runner.mixed_step(slots, [[t] for t in pre.first_tokens])
        out[fused] = (pre.first_tokens, pre.last_logits, nxt)
    assert out[True][0] == out[False][0] and out[True][2] == out[False][2]
    assert torch.equal(out[True][1], out[False][1])
