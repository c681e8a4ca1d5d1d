"""The fused rotary-embedding + KV-scatter kernel is bit-exact against the
reference sequence: HF ``apply_rotary_pos_emb`` on the split QKV projection
(fp16 torch ops on the device), then the K/V row writes of
KVStorage.decode_update / mixed_update (kv_cache/storage.py:62-122), here as
torch index_put. q comes back rotated; page 0 (padding rows) is excluded.
"""
import pytest
import torch

from custom_inference_engine_b200 import cabi, native
from custom_inference_engine_b200.attn import core

pytestmark = pytest.mark.gpu
HQ, HKV, D, PAGE = 14, 2, 64, 16


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    native.device_errors(0, clear=True)
    yield
    assert native.device_errors(0, clear=True) == 0


def _rope_tables(positions, dev):
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding
    from custom_inference_engine_b200.model_runner import qwen2_config

    rot = Qwen2RotaryEmbedding(qwen2_config(), device=dev)
    x = torch.zeros(1, len(positions), 8, dtype=torch.float16, device=dev)
    return rot(x, torch.tensor([positions], device=dev))


def _reference(qkv, cos, sin, k_cache, v_cache, pages, offsets):
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    T = qkv.shape[1]
    q, k, v = qkv.split([HQ * D, HKV * D, HKV * D], dim=-1)
    q, k = apply_rotary_pos_emb(q.view(1, T, HQ, D), k.view(1, T, HKV, D), cos, sin,
                                unsqueeze_dim=2)
    kc, vc = k_cache.clone(), v_cache.clone()
    kc[pages, :, offsets] = k.reshape(T, HKV, D)
    vc[pages, :, offsets] = v.reshape(T, HKV, D)
    return q, kc, vc


def _pool(dev, n_pages=64, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    k = torch.randn(n_pages, HKV, PAGE, D, generator=g, device=dev).half()
    v = torch.randn(n_pages, HKV, PAGE, D, generator=g, device=dev).half()
    return k, v


@pytest.mark.parametrize("T", [1, 5, 300])
def test_mixed_addressing_bit_exact(T, cuda_device):
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(T)
    # a strided qkv (a slice of a wider projection) with realistic magnitudes
    wide = (torch.randn(1, T, (HQ + 2 * HKV) * D + 64, generator=g, device=dev) * 3).half()
    qkv = wide[..., 32:32 + (HQ + 2 * HKV) * D]
    assert qkv.stride(1) == wide.stride(1)  # rows of the wider tensor
    positions = torch.randint(0, 30000, (T,), generator=g, device=dev).tolist()
    cos, sin = _rope_tables(positions, dev)
    k_cache, v_cache = _pool(dev)
    pages = torch.randperm(63, generator=g, device=dev)[:T % 63 + 1].repeat(T)[:T] + 1
    offsets = torch.randint(0, PAGE, (T,), generator=g, device=dev)
    # distinct destinations so that the reference's index_put has no duplicate rows
    key = pages * PAGE + offsets
    keep = torch.unique(key, return_inverse=False).numel() == T
    if not keep:
        offsets = torch.arange(T, device=dev) % PAGE
        pages = torch.arange(T, device=dev) // PAGE + 1
    q_ref, k_ref, v_ref = _reference(qkv, cos, sin, k_cache, v_cache, pages, offsets)
    kc, vc = k_cache.clone(), v_cache.clone()
    q = cabi.rope_kv_mixed_update(qkv, cos, sin, kc, vc, pages, offsets)
    assert torch.equal(q, q_ref)
    assert torch.equal(kc[1:], k_ref[1:]) and torch.equal(vc[1:], v_ref[1:])
    # the torch op gives the same bits
    kc2, vc2 = k_cache.clone(), v_cache.clone()
    q2 = core.rope_kv_mixed_update_op(qkv, cos, sin, kc2, vc2, pages, offsets)
    assert torch.equal(q2, q) and torch.equal(kc2, kc) and torch.equal(vc2, vc)


def test_decode_addressing_bit_exact(cuda_device):
    dev = cuda_device
    B, n_slots, bt_stride = 6, 9, 40
    g = torch.Generator(device=dev).manual_seed(3)
    k_cache, v_cache = _pool(dev, n_pages=256)
    block_table = torch.zeros(n_slots, bt_stride, dtype=torch.long, device=dev)
    block_table[1:] = (torch.randperm(255, generator=g, device=dev)[:(n_slots - 1) * 30]
                       .view(n_slots - 1, 30) + 1).repeat(1, 2)[:, :bt_stride]
    lens = torch.zeros(n_slots, dtype=torch.long, device=dev)
    lens[1:] = torch.randint(0, 30 * PAGE, (n_slots - 1,), generator=g, device=dev)
    slot_ids = torch.tensor([3, 1, 8, 5, 2, 7], device=dev)
    qkv = (torch.randn(1, B, (HQ + 2 * HKV) * D, generator=g, device=dev) * 3).half()
    cos, sin = _rope_tables(lens[slot_ids].tolist(), dev)
    pos = lens[slot_ids]
    pages = block_table[slot_ids, pos // PAGE]
    offsets = pos % PAGE
    q_ref, k_ref, v_ref = _reference(qkv, cos, sin, k_cache, v_cache, pages, offsets)
    kc, vc = k_cache.clone(), v_cache.clone()
    q = cabi.rope_kv_decode_update(qkv, cos, sin, kc, vc, lens, slot_ids, block_table)
    assert torch.equal(q, q_ref)
    assert torch.equal(kc[1:], k_ref[1:]) and torch.equal(vc[1:], v_ref[1:])
    kc2, vc2 = k_cache.clone(), v_cache.clone()
    q2 = core.rope_kv_decode_update_op(qkv, cos, sin, kc2, vc2, lens, slot_ids, block_table)
    assert torch.equal(q2, q) and torch.equal(kc2, kc) and torch.equal(vc2, vc)


def test_bad_page_is_reported_not_written(cuda_device):
    dev = cuda_device
    k_cache, v_cache = _pool(dev)
    qkv = torch.randn(1, 2, (HQ + 2 * HKV) * D, device=dev).half()
    cos, sin = _rope_tables([0, 1], dev)
    pages = torch.tensor([3, 64], device=dev)  # 64 is past the pool
    offsets = torch.tensor([0, 1], device=dev)
    kc, vc = k_cache.clone(), v_cache.clone()
    cabi.rope_kv_mixed_update(qkv, cos, sin, kc, vc, pages, offsets)
    assert native.device_errors(0, clear=True) & 4  # CIE_DEVERR_BAD_PAGE
    assert not torch.equal(kc[3, :, 0], k_cache[3, :, 0])  # the good row was written


@pytest.mark.parametrize("splits", [0, 1, 3, 16])
def test_rope_kv_decode_attention_one_launch(splits, cuda_device):
    """RoPE + K/V write + decode attention in one launch gives the bits of the
    two-launch sequence (cie_rope_kv_decode_update, then cie_decode_attention
    over lens[slot] + 1 keys): the same output and the same pages. Positions
    cover the first row of a page, the last row, a page boundary, a
    one-token history and a padding row on slot 0."""
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(100 + splits)
    n_slots = 9
    per_slot = 40                                     # pages per slot: up to 640 tokens
    n_pages = 1 + (n_slots - 1) * per_slot
    k0 = torch.randn(n_pages, HKV, PAGE, D, generator=g, device=dev).half()
    v0 = torch.randn(n_pages, HKV, PAGE, D, generator=g, device=dev).half()
    perm = torch.randperm(n_pages - 1, generator=torch.Generator().manual_seed(splits)) + 1
    bt = torch.zeros(n_slots, n_pages, dtype=torch.long)
    for s in range(1, n_slots):
        bt[s, :per_slot] = perm[(s - 1) * per_slot:s * per_slot]
    bt = bt.to(dev)
    lens = torch.tensor([0, 0, 15, 16, 31, 100, 1, 639, 47], dtype=torch.long, device=dev)
    slots = torch.tensor([2, 3, 4, 5, 6, 7, 8, 1, 0], dtype=torch.long, device=dev)
    B = slots.shape[0]
    wide = (torch.randn(1, B, (HQ + 2 * HKV) * D + 64, generator=g, device=dev) * 3).half()
    qkv = wide[..., 64:]
    cos, sin = _rope_tables(lens[slots].tolist(), dev)
    # two launches
    k1, v1 = k0.clone(), v0.clone()
    q = cabi.rope_kv_decode_update(qkv, cos, sin, k1, v1, lens, slots, bt)
    o_two = cabi.decode_attention(q, k1, v1, lens[slots] + 1, slots, bt, num_splits=splits)
    # one launch
    k2, v2 = k0.clone(), v0.clone()
    o_one = cabi.rope_kv_decode_attention(qkv, cos, sin, k2, v2, lens, slots, bt,
                                          num_splits=splits)
    torch.cuda.synchronize()
    assert torch.equal(o_one, o_two)
    assert torch.equal(k2[1:], k1[1:]) and torch.equal(v2[1:], v1[1:])
    # the torch op (default splits) agrees
    if splits == 0:
        k3, v3 = k0.clone(), v0.clone()
        o_op = torch.ops.inference.rope_kv_decode_attention(qkv, cos, sin, k3, v3, lens, slots, bt)
        assert torch.equal(o_op, o_two) and torch.equal(k3[1:], k1[1:])
