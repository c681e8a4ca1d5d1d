"""The ops capture into CUDA graphs and replay with new device-side inputs.

The engine's DecodeModule / FullMixedModule capture the whole forward, the
update and attention ops included, and replay it with new slot ids, lengths
and block tables written into the same buffers. The ops therefore may not
synchronise with the host or depend on host-side copies of lengths.
"""
import pytest
import torch

from custom_inference_engine_b200 import native
from custom_inference_engine_b200 import workloads as W

pytestmark = pytest.mark.gpu


def test_decode_update_and_attention_replay(cuda_device):
    from custom_inference_engine_b200.attn import core
    upd = torch.ops.inference.kv_decode_update
    B = 16
    lens0 = [100 + 37 * i for i in range(B)]
    c = W.make_decode_case([x + 8 for x in lens0], seed=9, device=cuda_device)
    slot_lens = torch.zeros(c.block_table.shape[0], dtype=torch.long, device=cuda_device)
    slot_lens[1:] = torch.tensor(lens0, device=cuda_device)
    kn = torch.randn(1, B, 2, 64, device=cuda_device).half()
    vn = torch.randn(1, B, 2, 64, device=cuda_device).half()
    k, v = c.k.clone(), c.v.clone()

    def step():
        upd(k, v, slot_lens, c.slot_ids, c.block_table, kn, vn)
        return core.gqa_decode_attention_op(c.q, k, v, slot_lens[c.slot_ids] + 1,
                                            slot_ids=c.slot_ids, block_table=c.block_table)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    for it in range(3):
        slot_lens[1:] += 1
        kn.normal_()
        vn.normal_()
        graph.replay()
        k_ref, v_ref = k.clone(), v.clone()
        eager = step()  # writes the same rows again, same values
        torch.cuda.synchronize()
        assert torch.equal(k, k_ref) and torch.equal(v, v_ref)
        assert torch.equal(out, eager)
    assert native.device_errors(0) == 0


def test_mixed_update_and_attention_replay(cuda_device):
    from custom_inference_engine_b200.attn import core
    upd = torch.ops.inference.kv_mixed_update
    c = W.make_mixed_case([40, 1, 17], [30, 90, 0], seed=12, device=cuda_device,
                          max_seqlen=64, pad_batch=1)
    T = c.q.shape[1]
    pages = torch.zeros(T, dtype=torch.long, device=cuda_device)
    offsets = torch.zeros(T, dtype=torch.long, device=cuda_device)
    kn = torch.randn(1, T, 2, 64, device=cuda_device).half()
    vn = torch.randn(1, T, 2, 64, device=cuda_device).half()
    k, v = c.k.clone(), c.v.clone()

    def fill_positions():
        cu = c.cu_seqlens.tolist()
        kvl = c.kv_lens.tolist()
        sl = c.slot_ids.tolist()
        pg, of = [0] * T, [0] * T
        for b in range(len(sl)):
            for i in range(cu[b + 1] - cu[b]):
                pos = kvl[b] + i
                pg[cu[b] + i] = int(c.block_table[sl[b], pos // 16])
                of[cu[b] + i] = pos % 16
        pages.copy_(torch.tensor(pg))
        offsets.copy_(torch.tensor(of))

    def step():
        upd(k, v, pages, offsets, kn, vn)
        return core.gqa_mixed_attention_op(c.q, k, v, kv_lens=c.kv_lens, max_seqlen=c.max_seqlen,
                                           cu_seqlens=c.cu_seqlens, slot_ids=c.slot_ids,
                                           block_table=c.block_table)

    fill_positions()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    rows = slice(0, int(c.cu_seqlens[-1]))
    for it in range(2):
        kn.normal_()
        vn.normal_()
        c.q.normal_()
        graph.replay()
        eager = step()
        torch.cuda.synchronize()
        assert torch.equal(out[0, rows], eager[0, rows])
    assert native.device_errors(0) == 0
