"""A combined K/V page layout through the C ABI: one pool of shape
(n_pages, 2, H_kv, page_size, D) whose page holds both heads' K rows and then
both heads' V rows (8 KiB per page; K = pool[:, 0], V = pool[:, 1], page stride
4096 elements). The reference keeps two separate pools (kv_cache/storage.py:
32-48); every entry point takes page and head strides, so the combined layout
needs no other kernels. Each op on the combined views must give the bits it
gives on separate contiguous pools holding the same values."""
import pytest
import torch

from custom_inference_engine_b200 import cabi, native
from custom_inference_engine_b200.attn import core  # noqa: F401  (registers inference::*)

pytestmark = pytest.mark.gpu
HQ, HKV, D, PAGE = 14, 2, 64, 16


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    native.device_errors(0, clear=True)
    yield
    assert native.device_errors(0, clear=True) == 0


def _pools(n_pages, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    pool = torch.randn(n_pages, 2, HKV, PAGE, D, generator=g, device=dev).half()
    k, v = pool[:, 0], pool[:, 1]
    assert k.stride(0) == 2 * HKV * PAGE * D and not k.is_contiguous()
    return pool, k, v, k.contiguous(), v.contiguous()


def _table(n_slots, per_slot, n_pages, seed, dev):
    perm = torch.randperm(n_pages - 1, generator=torch.Generator().manual_seed(seed)) + 1
    bt = torch.zeros(n_slots, n_pages, dtype=torch.long)
    for s in range(1, n_slots):
        bt[s, :per_slot] = perm[(s - 1) * per_slot:s * per_slot]
    return bt.to(dev)


@pytest.mark.parametrize("splits", [0, 1, 7])
def test_decode_attention_combined_pool(splits, cuda_device):
    dev = cuda_device
    n_slots, per_slot = 7, 70
    n_pages = 1 + (n_slots - 1) * per_slot
    _, k, v, kc, vc = _pools(n_pages, dev, seed=1 + splits)
    bt = _table(n_slots, per_slot, n_pages, splits, dev)
    lens = torch.tensor([1, 16, 17, 500, 1111, 70 * 16], dtype=torch.long, device=dev)
    slots = torch.tensor([3, 1, 6, 2, 5, 4], dtype=torch.long, device=dev)
    q = torch.randn(1, 6, HQ, D, device=dev).half()
    o_sep = cabi.decode_attention(q, kc, vc, lens, slots, bt, num_splits=splits)
    o_comb = cabi.decode_attention(q, k, v, lens, slots, bt, num_splits=splits)
    torch.cuda.synchronize()
    assert torch.equal(o_comb, o_sep)
    if splits == 0:  # the torch op accepts the strided pools as well
        o_op = torch.ops.inference.gqa_decode_attention(q, k, v, lens, slot_ids=slots,
                                                        block_table=bt)
        assert torch.equal(o_op, o_sep)


def test_mixed_attention_combined_pool(cuda_device):
    dev = cuda_device
    n_slots, per_slot = 6, 80
    n_pages = 1 + (n_slots - 1) * per_slot
    _, k, v, kc, vc = _pools(n_pages, dev, seed=11)
    bt = _table(n_slots, per_slot, n_pages, 5, dev)
    chunks = [1, 200, 33, 512, 1]
    kvs = [700, 0, 64, 600, 1200]
    T = sum(chunks)
    cu = torch.tensor([0] + torch.tensor(chunks).cumsum(0).tolist(), dtype=torch.long,
                      device=dev)
    kvl = torch.tensor(kvs, dtype=torch.long, device=dev)
    slots = torch.tensor([1, 2, 3, 4, 5], dtype=torch.long, device=dev)
    q = torch.randn(1, T, HQ, D, device=dev).half()
    o_sep = cabi.mixed_attention(q, kc, vc, max(chunks), cu, kvl, slots, bt)
    o_comb = cabi.mixed_attention(q, k, v, max(chunks), cu, kvl, slots, bt)
    torch.cuda.synchronize()
    assert torch.equal(o_comb, o_sep)


def test_kv_updates_combined_pool(cuda_device):
    dev = cuda_device
    n_slots, per_slot = 5, 8
    n_pages = 1 + (n_slots - 1) * per_slot
    pool, k, v, kc, vc = _pools(n_pages, dev, seed=21)
    bt = _table(n_slots, per_slot, n_pages, 9, dev)
    lens = torch.tensor([0, 0, 15, 16, 100], dtype=torch.long, device=dev)
    slots = torch.tensor([2, 4, 1, 3], dtype=torch.long, device=dev)
    fused = torch.randn(1, 4, (HQ + 2 * HKV) * D, device=dev).half()
    kn = fused[..., HQ * D:(HQ + HKV) * D].view(1, 4, HKV, D)
    vn = fused[..., (HQ + HKV) * D:].view(1, 4, HKV, D)
    cabi.kv_decode_update(kc, vc, lens, slots, bt, kn, vn)
    cabi.kv_decode_update(k, v, lens, slots, bt, kn, vn)
    pages = torch.tensor([3, 7, 7, 12, 30], dtype=torch.long, device=dev)
    offsets = torch.tensor([0, 15, 14, 9, 1], dtype=torch.long, device=dev)
    rows = torch.randn(1, 5, (HQ + 2 * HKV) * D, device=dev).half()
    km = rows[..., HQ * D:(HQ + HKV) * D].view(1, 5, HKV, D)
    vm = rows[..., (HQ + HKV) * D:].view(1, 5, HKV, D)
    cabi.kv_mixed_update(kc, vc, pages, offsets, km, vm)
    cabi.kv_mixed_update(k, v, pages, offsets, km, vm)
    torch.cuda.synchronize()
    assert torch.equal(k, kc) and torch.equal(v, vc)
    assert torch.equal(pool[:, 0], kc) and torch.equal(pool[:, 1], vc)


def test_rope_kv_decode_attention_combined_pool(cuda_device):
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding
    from custom_inference_engine_b200.model_runner import qwen2_config

    dev = cuda_device
    n_slots, per_slot = 6, 40
    n_pages = 1 + (n_slots - 1) * per_slot
    _, k, v, kc, vc = _pools(n_pages, dev, seed=31)
    bt = _table(n_slots, per_slot, n_pages, 13, dev)
    lens = torch.tensor([0, 0, 15, 16, 300, 639], dtype=torch.long, device=dev)
    slots = torch.tensor([2, 3, 4, 5, 1, 0], dtype=torch.long, device=dev)
    qkv = torch.randn(1, 6, (HQ + 2 * HKV) * D, device=dev).half()
    rot = Qwen2RotaryEmbedding(qwen2_config(), device=dev)
    cos, sin = rot(torch.zeros(1, 6, 8, dtype=torch.float16, device=dev),
                   lens[slots].view(1, -1))
    o_sep = cabi.rope_kv_decode_attention(qkv, cos, sin, kc, vc, lens, slots, bt)
    o_comb = cabi.rope_kv_decode_attention(qkv, cos, sin, k, v, lens, slots, bt)
    torch.cuda.synchronize()
    assert torch.equal(o_comb, o_sep)
    assert torch.equal(k[1:], kc[1:]) and torch.equal(v[1:], vc[1:])
