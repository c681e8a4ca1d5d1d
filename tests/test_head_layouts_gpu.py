"""Head layouts other than Qwen2.5-0.5B's 14 / 2: the C ABI takes any number
of kv heads for mixed attention and 1, 2 or 4 for decode, always 7 query
heads per kv head (GQA group 7), head_dim 64, 16-token pages. Parity against
the fp32 oracle (max-abs 2e-3 on fp16 outputs) and bit-exact KV pages."""
import pytest
import torch

import oracle
from custom_inference_engine_b200 import cabi, native

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _pool(lens, hkv, seed, slack_pages=2):
    """Pages of len(lens) slots (slot b + 1) scattered over a pool; page 0 unused."""
    g = torch.Generator().manual_seed(seed)
    per_slot = [(L + 15) // 16 + slack_pages for L in lens]
    n_pages = 1 + sum(per_slot)
    perm = (torch.randperm(n_pages - 1, generator=g) + 1).tolist()
    bt = torch.zeros(len(lens) + 1, n_pages, dtype=torch.long)
    o = 0
    for i, n in enumerate(per_slot):
        bt[i + 1, :n] = torch.tensor(perm[o:o + n])
        o += n
    k = torch.randn(n_pages, hkv, 16, 64, generator=g).half()
    v = torch.randn(n_pages, hkv, 16, 64, generator=g).half()
    return k, v, bt, g


@pytest.mark.parametrize("hkv", [1, 4])
@pytest.mark.parametrize("splits", [1, 5, 0])
def test_decode_kv_heads(hkv, splits, cuda_device):
    lens = [1, 16, 17, 300, 777, 2049]
    k, v, bt, g = _pool(lens, hkv, seed=10 + hkv)
    B = len(lens)
    q = torch.randn(1, B, 7 * hkv, 64, generator=g).half()
    L = torch.tensor(lens, dtype=torch.long)
    slots = torch.arange(1, B + 1, dtype=torch.long)
    ref = oracle.decode_attention_fp32(q, k, v, L, slots, bt)
    dev = cuda_device
    out = cabi.decode_attention(q.to(dev), k.to(dev), v.to(dev), L.to(dev), slots.to(dev),
                                bt.to(dev), num_splits=splits)
    err = (out.float().cpu() - ref.float()).abs().max().item()
    assert err <= TOL, err
    assert native.device_errors(0) == 0


@pytest.mark.parametrize("hkv", [1, 3])
def test_mixed_kv_heads(hkv, cuda_device):
    chunks = [1, 40, 17, 100, 1]
    kvs = [250, 0, 33, 700, 5]
    k, v, bt, g = _pool([c + kv for c, kv in zip(chunks, kvs)], hkv, seed=20 + hkv)
    T = sum(chunks)
    q = torch.randn(1, T, 7 * hkv, 64, generator=g).half()
    cu = torch.tensor([0] + torch.tensor(chunks).cumsum(0).tolist(), dtype=torch.long)
    kvl = torch.tensor(kvs, dtype=torch.long)
    slots = torch.arange(1, len(chunks) + 1, dtype=torch.long)
    ref = oracle.mixed_attention_fp32(q, k, v, max(chunks), cu, kvl, slots, bt)
    dev = cuda_device
    out = cabi.mixed_attention(q.to(dev), k.to(dev), v.to(dev), max(chunks), cu.to(dev),
                               kvl.to(dev), slots.to(dev), bt.to(dev))
    err = (out.float().cpu() - ref.float()).abs().max().item()
    assert err <= TOL, err
    assert native.device_errors(0) == 0


def test_decode_update_four_kv_heads(cuda_device):
    hkv = 4
    lens_slots = [0, 15, 16, 40]
    k, v, bt, g = _pool([L + 1 for L in lens_slots], hkv, seed=31)
    lens = torch.tensor([0] + lens_slots, dtype=torch.long)      # per slot, slot 0 padding
    slots = torch.tensor([2, 4, 1, 3], dtype=torch.long)
    fused = torch.randn(1, 4, (7 * hkv + 2 * hkv) * 64, generator=g).half()
    kn = fused[..., 7 * hkv * 64:8 * hkv * 64].view(1, 4, hkv, 64)   # strided views
    vn = fused[..., 8 * hkv * 64:9 * hkv * 64].view(1, 4, hkv, 64)
    k_ref, v_ref = k.clone(), v.clone()
    oracle.decode_update_ref(k_ref, v_ref, lens, slots, bt, kn, vn)
    dev = cuda_device
    kd, vd = k.to(dev), v.to(dev)
    cabi.kv_decode_update(kd, vd, lens.to(dev), slots.to(dev), bt.to(dev), kn.to(dev),
                          vn.to(dev))
    assert torch.equal(kd[1:].cpu(), k_ref[1:]) and torch.equal(vd[1:].cpu(), v_ref[1:])
    assert native.device_errors(0) == 0
