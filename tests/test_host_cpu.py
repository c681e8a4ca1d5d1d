"""Host-side pieces that need no GPU: op registration and schemas, fake
kernels for Dynamo, the no-CPU-fallback rule, metadata padding, workloads."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from custom_inference_engine_b200 import workloads as W
from custom_inference_engine_b200.attn import core
from custom_inference_engine_b200.attn.metadata import AttentionMetadata


def test_op_schemas_match_the_reference_triton_ops():
    dec = torch.ops.inference.gqa_decode_attention.default._schema
    mix = torch.ops.inference.gqa_mixed_attention.default._schema
    assert str(dec) == ("inference::gqa_decode_attention(Tensor q, Tensor k, Tensor v, "
                        "Tensor lens, Tensor slot_ids, Tensor block_table) -> Tensor")
    assert str(mix) == ("inference::gqa_mixed_attention(Tensor q, Tensor k, Tensor v, "
                        "SymInt max_seqlen, Tensor cu_seqlens, Tensor kv_lens, "
                        "Tensor slot_ids, Tensor block_table) -> Tensor")
    upd = torch.ops.inference.kv_decode_update.default._schema
    assert upd.arguments[0].alias_info.is_write and upd.arguments[1].alias_info.is_write
    # the module exposes the overloads, which is what a call records as the FX
    # node target (the reference's piecewise splitter matches this object)
    assert core.gqa_mixed_attention_op is torch.ops.inference.gqa_mixed_attention.default
    assert core.gqa_decode_attention_op is torch.ops.inference.gqa_decode_attention.default


def test_fake_kernels_propagate_shapes():
    with FakeTensorMode():
        q = torch.empty(1, 5, 14, 64, dtype=torch.float16, device="cuda")
        k = torch.empty(9, 2, 16, 64, dtype=torch.float16, device="cuda")
        i = torch.zeros(5, dtype=torch.long, device="cuda")
        bt = torch.zeros(6, 9, dtype=torch.long, device="cuda")
        o = core.gqa_decode_attention_op(q, k, k, i, slot_ids=i, block_table=bt)
        assert o.shape == q.shape and o.dtype == q.dtype
        cu = torch.zeros(6, dtype=torch.long, device="cuda")
        o = core.gqa_mixed_attention_op(q, k, k, max_seqlen=5, cu_seqlens=cu, kv_lens=i,
                                        slot_ids=i, block_table=bt)
        assert o.shape == q.shape


def test_no_cpu_fallback():
    q = torch.zeros(1, 2, 14, 64, dtype=torch.float16)
    k = torch.zeros(4, 2, 16, 64, dtype=torch.float16)
    i = torch.ones(2, dtype=torch.long)
    with pytest.raises(NotImplementedError):
        core.gqa_decode_attention_op(q, k, k, i, slot_ids=i, block_table=torch.zeros(3, 4).long())


def test_host_asserts_mirror_reference():
    q = torch.zeros(1, 2, 14, 64, dtype=torch.float16)
    k = torch.zeros(4, 2, 16, 64, dtype=torch.float16)
    with pytest.raises(AssertionError):   # N_PAGES == block_table.shape[1]
        core.decode_gqa_attention(q, k, k, torch.ones(2).long(), torch.ones(2).long(),
                                  torch.zeros(3, 5).long())
    with pytest.raises(AssertionError):   # cu_seqlens (B+1,)
        core.mixed_gqa_attention(q, k, k, 2, torch.zeros(2).long(), torch.zeros(2).long(),
                                 torch.zeros(2).long(), torch.zeros(3, 4).long())


def test_metadata_padding_rules():
    m = AttentionMetadata(token_count=6, full_decode=False, device="cpu")
    m.prepare_full_graph(4)
    m.write_slot_ids([3, 5])
    assert m.slot_ids.tolist() == [3, 5, 0, 0]
    m.write_cu_seqlens([0, 2, 5])
    assert m.cu_seqlens.tolist() == [0, 2, 5, 5, 5]
    m.write_pages([7, 7, 9])
    m.write_offsets([1, 2, 3])
    assert m.pages.tolist() == [7, 7, 9, 0, 0, 0]
    assert m.offsets.tolist() == [1, 2, 3, 0, 0, 0]
    assert m.max_seqlen == 6


def test_workload_shapes_and_bytes():
    c = W.make_decode_case([1, 16, 17], seed=0)
    assert c.k.shape == (1 + 1 + 1 + 2, 2, 16, 64)
    assert c.block_table.shape == (4, 5)
    used = c.block_table[1:].flatten().tolist()
    assert sorted(p for p in used if p) == [1, 2, 3, 4]
    assert c.algorithmic_bytes() == 34 * 512 + 3 * 3584 + 4 * 8
    m = W.make_mixed_case([3, 1], [5, 0], seed=0, pad_batch=2, max_seqlen=8)
    assert m.cu_seqlens.tolist() == [0, 3, 4, 4, 4]
    assert m.slot_ids.tolist() == [1, 2, 0, 0]
    assert m.causal_flops() == 4 * 64 * 14 * (3 * 5 + 6 + 1)
