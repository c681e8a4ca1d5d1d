"""The CUDA KV-page scatter is bit-exact against the reference KVStorage.

Fixtures hold the pools before and after the reference's decode_update /
mixed_update (kv_cache/storage.py:62-122). Page 0 absorbs padded rows, which
may write it several times with no defined winner, so it is excluded.
"""
import types

import pytest
import torch

from conftest import load_golden
from custom_inference_engine_b200 import cabi, native

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    native.device_errors(0, clear=True)
    yield
    assert native.device_errors(0, clear=True) == 0


def _views(fused):
    T = fused.shape[1]
    return (fused[..., 14 * 64:16 * 64].view(1, T, 2, 64),
            fused[..., 16 * 64:18 * 64].view(1, T, 2, 64))


def test_decode_update_cabi_bit_exact(cuda_device):
    g = load_golden("kv_decode_update")
    d = {k: v.to(cuda_device) for k, v in g.items() if torch.is_tensor(v)}
    k, v = d["k_before"].clone(), d["v_before"].clone()
    kn, vn = _views(d["fused"])
    assert not vn.is_contiguous()
    cabi.kv_decode_update(k, v, d["lens"], d["slot_ids"], d["block_table"], kn, vn)
    assert torch.equal(k[1:].cpu(), g["k_after"][1:])
    assert torch.equal(v[1:].cpu(), g["v_after"][1:])


def test_mixed_update_cabi_bit_exact(cuda_device):
    g = load_golden("kv_mixed_update")
    d = {k: v.to(cuda_device) for k, v in g.items() if torch.is_tensor(v)}
    k, v = d["k_before"].clone(), d["v_before"].clone()
    kn, vn = _views(d["fused"])
    cabi.kv_mixed_update(k, v, d["pages"], d["offsets"], kn, vn)
    assert torch.equal(k[1:].cpu(), g["k_after"][1:])
    assert torch.equal(v[1:].cpu(), g["v_after"][1:])


def test_kvstorage_methods_bit_exact(cuda_device):
    from custom_inference_engine_b200.kv_cache.storage import KVStorage
    g = load_golden("kv_decode_update")
    cfg = types.SimpleNamespace(num_hidden_layers=2, num_attention_heads=14,
                                num_key_value_heads=2, hidden_size=896, head_dim=64)
    kv = KVStorage(cfg, max_cache_len=g["k_before"].shape[0] * 16, page_size=16,
                   n_slots=g["lens"].shape[0], device=cuda_device, dtype=torch.float16)
    kv.keys[1].copy_(g["k_before"])
    kv.values[1].copy_(g["v_before"])
    kv.lens.copy_(g["lens"])
    kv.block_table.copy_(g["block_table"])
    kn, vn = _views(g["fused"].to(cuda_device))
    kv.decode_update(1, g["slot_ids"].to(cuda_device), kn, vn)
    assert torch.equal(kv.keys[1][1:].cpu(), g["k_after"][1:])
    assert torch.equal(kv.values[1][1:].cpu(), g["v_after"][1:])
    assert torch.equal(kv.keys[0].cpu(), torch.zeros_like(g["k_after"]))

    m = load_golden("kv_mixed_update")
    kv.keys[1].copy_(m["k_before"])
    kv.values[1].copy_(m["v_before"])
    kn, vn = _views(m["fused"].to(cuda_device))
    kv.mixed_update(1, m["pages"].to(cuda_device), m["offsets"].to(cuda_device), kn, vn)
    assert torch.equal(kv.keys[1][1:].cpu(), m["k_after"][1:])
    assert torch.equal(kv.values[1][1:].cpu(), m["v_after"][1:])


def test_unaligned_source_rows_take_scalar_path(cuda_device):
    # token stride of 18*64+4 elements is not a multiple of 16 bytes
    g = load_golden("kv_mixed_update")
    T = g["fused"].shape[1]
    wide = torch.zeros(1, T, 18 * 64 + 4, dtype=torch.float16)
    wide[..., :18 * 64] = g["fused"]
    wide = wide.to(cuda_device)
    kn = wide[..., 14 * 64:16 * 64].view(1, T, 2, 64)
    vn = wide[..., 16 * 64:18 * 64].view(1, T, 2, 64)
    k = g["k_before"].to(cuda_device)
    v = g["v_before"].to(cuda_device)
    cabi.kv_mixed_update(k, v, g["pages"].to(cuda_device), g["offsets"].to(cuda_device), kn, vn)
    assert torch.equal(k[1:].cpu(), g["k_after"][1:])
    assert torch.equal(v[1:].cpu(), g["v_after"][1:])


def test_out_of_range_page_is_flagged_not_written(cuda_device):
    g = load_golden("kv_mixed_update")
    k = g["k_before"].to(cuda_device)
    v = g["v_before"].to(cuda_device)
    kn, vn = _views(g["fused"].to(cuda_device))
    pages = g["pages"].clone()
    pages[0] = k.shape[0] + 3
    cabi.kv_mixed_update(k, v, pages.to(cuda_device), g["offsets"].to(cuda_device), kn, vn)
    assert native.device_errors(0) & 4  # CIE_DEVERR_BAD_PAGE
