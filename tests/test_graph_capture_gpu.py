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


def test_one_mixed_graph_serves_changing_batches(cuda_device):
    """Capturable dynamic-batch mixed attention: ONE graph captured at the
    largest shape (6 sequences, 96 tokens) replays correctly for batches of
    1 to 6 sequences with other chunk lengths, cached lengths and slots, all
    written into the captured device buffers; unused sequences are padded the
    reference's way (slot 0, cu_seqlens repeating its last value, so L = 0)."""
    import oracle
    from custom_inference_engine_b200.attn import core

    dev = cuda_device
    B_max, T, n_slots, pages_per_slot = 6, 96, 7, 32
    g = torch.Generator().manual_seed(99)
    n_pages = 1 + (n_slots - 1) * pages_per_slot
    k = torch.randn(n_pages, 2, 16, 64, generator=g).half()
    v = torch.randn(n_pages, 2, 16, 64, generator=g).half()
    bt = torch.zeros(n_slots, n_pages, dtype=torch.long)
    perm = torch.randperm(n_pages - 1, generator=g) + 1
    for s in range(1, n_slots):
        bt[s, :pages_per_slot] = perm[(s - 1) * pages_per_slot:s * pages_per_slot]
    kd, vd, btd = k.to(dev), v.to(dev), bt.to(dev)
    q = torch.zeros(1, T, 14, 64, dtype=torch.half, device=dev)
    cu = torch.zeros(B_max + 1, dtype=torch.long, device=dev)
    kvl = torch.zeros(B_max, dtype=torch.long, device=dev)
    slots = torch.zeros(B_max, dtype=torch.long, device=dev)

    def step():
        return core.gqa_mixed_attention_op(q, kd, vd, kv_lens=kvl, max_seqlen=T, cu_seqlens=cu,
                                           slot_ids=slots, block_table=btd)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    compositions = [([1], [300], [4]),
                    ([40, 1, 1, 30], [0, 77, 250, 12], [2, 5, 1, 6]),
                    ([16, 16, 16, 16, 16, 16], [3, 100, 0, 401, 64, 17], [6, 5, 4, 3, 2, 1]),
                    ([1, 95], [20, 200], [3, 1])]
    for chunks, kv_lens, sl in compositions:
        n = len(chunks)
        cum = [0]
        for c in chunks:
            cum.append(cum[-1] + c)
        cu.copy_(torch.tensor(cum + [cum[-1]] * (B_max - n)))
        kvl.copy_(torch.tensor(kv_lens + [0] * (B_max - n)))
        slots.copy_(torch.tensor(sl + [0] * (B_max - n)))
        q.copy_(torch.randn(1, T, 14, 64, generator=g).half())
        graph.replay()
        torch.cuda.synchronize()
        ref = oracle.mixed_attention_fp32(q.cpu(), k, v, T, cu.cpu(), kvl.cpu(), slots.cpu(), bt)
        rows = slice(0, cum[-1])
        err = (out[0, rows].float().cpu() - ref[0, rows].float()).abs().max().item()
        assert err <= 2e-3, (chunks, err)
    assert native.device_errors(0) == 0
