"""Host logic of the paged model runner: page hand-out and the metadata of a
mixed pass (which page and offset every new token's K/V goes to)."""
import torch

from custom_inference_engine_b200 import model_runner as MR


def _runner():
    cfg = MR.qwen2_config(num_hidden_layers=1, vocab_size=64, intermediate_size=128)
    model = MR.random_qwen2(cfg, seed=0, device="cpu", dtype=torch.float32)
    return MR.PagedRunner(model, max_cache_len=64 * 16, n_slots=4, token_budget=32)


def test_pages_are_scattered_and_disjoint():
    r = _runner()
    r.admit(1, 40)
    r.admit(2, 17)
    p1 = r.kv.block_table[1, :3].tolist()
    p2 = r.kv.block_table[2, :2].tolist()
    assert 0 not in p1 + p2 and len(set(p1 + p2)) == 5
    assert r.kv.block_table[1, 3:].eq(0).all() and r.kv.block_table[2, 2:].eq(0).all()


def test_mixed_metadata_places_every_token():
    r = _runner()
    r.admit(1, 40)
    r.admit(3, 40)
    r.host_lens[3] = 20  # slot 3 already holds 20 tokens
    md, positions, cu = r.mixed_metadata([1, 3], [5, 14])
    assert cu == [0, 5, 19]
    assert positions.tolist() == list(range(5)) + list(range(20, 34))
    bt = r.kv.block_table
    for t, (s, pos) in enumerate([(1, p) for p in range(5)] + [(3, p) for p in range(20, 34)]):
        assert int(md.pages[t]) == int(bt[s, pos // 16])
        assert int(md.offsets[t]) == pos % 16
    assert md.slot_ids.tolist() == [1, 3] and md.cu_seqlens.tolist() == [0, 5, 19]
    assert not md.full_decode and md.max_seqlen == 19


def test_release_returns_pages_and_clears_the_slot():
    r = _runner()
    free = len(r.free_pages)
    r.admit(2, 50)
    assert len(r.free_pages) == free - 4
    r.host_lens[2] = 9
    r.release(2)
    assert len(r.free_pages) == free and r.host_lens[2] == 0
    assert r.kv.block_table[2].eq(0).all() and int(r.kv.lens[2]) == 0
