"""int32 block tables through every entry point that reads one.

The reference keeps the block table as int64 (kv_cache/storage.py:52-56). The
``*_bt32`` entry points (and the torch ops, which dispatch on the table's
dtype) take the same table as int32 page ids; outputs and pool writes must be
bit-identical to the int64 table's, and a model served from an int32 table
must give the same greedy tokens.
"""
import pytest
import torch

from custom_inference_engine_b200 import cabi, native
from custom_inference_engine_b200 import model_runner as MR
from custom_inference_engine_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    native.device_errors(0, clear=True)
    yield
    assert native.device_errors(0, clear=True) == 0


def _decode_case(dev):
    c = W.make_decode_case([1, 17, 300, 1024, 0, 4096, 33, 2000], seed=21)
    return [t.to(dev) for t in (c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)]


@pytest.mark.parametrize("splits", [1, 3, 0])
def test_decode_bt32_bit_identical(splits, cuda_device):
    q, k, v, lens, slots, bt = _decode_case(cuda_device)
    want = cabi.decode_attention(q, k, v, lens, slots, bt, num_splits=splits)
    got = cabi.decode_attention(q, k, v, lens, slots, bt.int(), num_splits=splits)
    assert torch.equal(got, want)
    from custom_inference_engine_b200.attn import core
    op = core.gqa_decode_attention_op(q, k, v, lens, slot_ids=slots, block_table=bt.int())
    assert torch.equal(op, core.gqa_decode_attention_op(q, k, v, lens, slot_ids=slots,
                                                        block_table=bt))


def test_mixed_bt32_bit_identical(cuda_device):
    from custom_inference_engine_b200.attn import core
    m = W.make_mixed_case([1, 40, 130, 512, 1], [9, 0, 200, 3000, 77], seed=22)
    q, k, v, cu, kvl, slots, bt = [t.to(cuda_device) for t in (m.q, m.k, m.v, m.cu_seqlens,
                                                               m.kv_lens, m.slot_ids,
                                                               m.block_table)]
    out = {}
    for table in (bt, bt.int()):
        out[table.dtype] = core.gqa_mixed_attention_op(q, k, v, max_seqlen=m.max_seqlen,
                                                       cu_seqlens=cu, kv_lens=kvl, slot_ids=slots,
                                                       block_table=table)
    assert torch.equal(out[torch.int32], out[torch.int64])
    got = cabi.mixed_attention(q, k, v, m.max_seqlen, cu, kvl, slots, bt.int(), num_splits=3)
    want = cabi.mixed_attention(q, k, v, m.max_seqlen, cu, kvl, slots, bt, num_splits=3)
    rows = torch.cat([torch.arange(a, b) for a, b in zip(m.cu_seqlens[:-1].tolist(),
                                                        m.cu_seqlens[1:].tolist())])
    assert torch.equal(got[0, rows.to(cuda_device)], want[0, rows.to(cuda_device)])


def test_kv_writes_bt32_bit_identical(cuda_device):
    q, k, v, lens, slots, bt = _decode_case(cuda_device)
    B = slots.shape[0]
    g = torch.Generator(device=cuda_device).manual_seed(5)
    slot_lens = torch.zeros(bt.shape[0], dtype=torch.int64, device=cuda_device)
    slot_lens[slots] = (lens - 1).clamp(min=0)
    kn = torch.randn(1, B, 2, 64, generator=g, device=cuda_device).half()
    vn = torch.randn(1, B, 2, 64, generator=g, device=cuda_device).half()
    qkv = torch.randn(1, B, 18 * 64, generator=g, device=cuda_device).half()
    cos = torch.randn(1, B, 64, generator=g, device=cuda_device).half()
    sin = torch.randn(1, B, 64, generator=g, device=cuda_device).half()
    res = {}
    for table in (bt, bt.int()):
        kk, vv = k.clone(), v.clone()
        cabi.kv_decode_update(kk, vv, slot_lens, slots, table, kn, vn)
        qr = cabi.rope_kv_decode_update(qkv, cos, sin, kk, vv, slot_lens, slots, table)
        o = cabi.rope_kv_decode_attention(qkv, cos, sin, kk, vv, slot_lens, slots, table)
        res[table.dtype] = (kk, vv, qr, o)
    for a, b in zip(res[torch.int32], res[torch.int64]):
        assert torch.equal(a, b)


def test_runner_greedy_tokens_with_an_int32_table(cuda_device):
    cfg = MR.qwen2_config(num_hidden_layers=2, vocab_size=4096, intermediate_size=2048)
    model = MR.random_qwen2(cfg, seed=0, device=cuda_device)
    prompts = [list(range(3, 3 + n)) for n in (5, 40, 130)]
    toks = {}
    for dt in (torch.int64, torch.int32):
        runner = MR.PagedRunner(model, max_cache_len=2048, n_slots=4, token_budget=64,
                                block_table_dtype=dt)
        assert runner.kv.block_table.dtype == dt
        slots = [1, 2, 3]
        for s, p in zip(slots, prompts):
            runner.admit(s, len(p) + 12)
        pre = runner.prefill(slots, prompts)
        graph = runner.decode_graph(slots, pre.first_tokens, capture=True)
        toks[dt] = [pre.first_tokens] + [graph.step().tolist() for _ in range(8)]
    assert toks[torch.int32] == toks[torch.int64]
