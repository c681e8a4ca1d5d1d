"""Parity of the sm_100a split-KV decode kernel (C ABI and torch op).

Bar: max-abs <= 2e-3 on fp16 outputs against (a) the reference Triton
kernels' own outputs (golden fixtures) and (b) fp32 softmax attention (the
CPU oracle at small sizes, the same math in torch fp32 on the GPU at full
sizes). Zero-length rows must be exactly zero.
"""
import pytest
import torch

from conftest import load_golden
from custom_inference_engine_b200 import cabi, native
from custom_inference_engine_b200 import workloads as W
import oracle

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _dev(g, dev, keys=("q", "k", "v", "lens", "slot_ids", "block_table")):
    return [g[k].to(dev) for k in keys]


def _maxabs(a, b):
    return (a.float().cpu() - b.float().cpu()).abs().max().item()


def torch_decode_fp32(q, k, v, lens, slot_ids, block_table):
    """fp32 reference math on the device for fixed-length batches (all lens equal)."""
    B = slot_ids.shape[0]
    L = int(lens[0])
    assert bool((lens == L).all())
    n = (L + 15) // 16
    pages = block_table[slot_ids, :n]                       # (B, n)
    kk = k[pages].permute(0, 2, 1, 3, 4).reshape(B, k.shape[1], n * 16, 64)[:, :, :L].float()
    vv = v[pages].permute(0, 2, 1, 3, 4).reshape(B, k.shape[1], n * 16, 64)[:, :, :L].float()
    qq = q[0].float().view(B, k.shape[1], -1, 64)
    s = torch.einsum("bhgd,bhld->bhgl", qq, kk) * 0.125
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("bhgl,bhld->bhgd", p, vv)
    return o.reshape(1, B, -1, 64).to(torch.float16)


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    native.device_errors(0, clear=True)
    yield
    assert native.device_errors(0, clear=True) == 0


@pytest.mark.parametrize("name", ["decode_edges", "decode_random"])
@pytest.mark.parametrize("splits", [1, 2, 3, 16, 0])
def test_golden_cases_cabi(name, splits, cuda_device):
    g = load_golden(name)
    q, k, v, lens, slot_ids, bt = _dev(g, cuda_device)
    o = cabi.decode_attention(q, k, v, lens, slot_ids, bt, num_splits=splits)
    torch.cuda.synchronize()
    assert _maxabs(o, g["out"]) <= TOL
    ref = oracle.decode_attention_fp32(g["q"], g["k"], g["v"], g["lens"], g["slot_ids"],
                                       g["block_table"])
    assert _maxabs(o, ref) <= TOL
    zero = (g["lens"] == 0).nonzero().flatten()
    assert bool((o[0, zero.to(cuda_device)] == 0).all())


def test_config1_full(cuda_device):
    g = load_golden("decode_config1")
    c = W.make_decode_case(W.config1_lens(), seed=int(g["seed"]))
    ref = oracle.decode_attention_fp32(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)
    args = [t.to(cuda_device) for t in (c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)]
    for splits in (0, 1, 16):
        o = cabi.decode_attention(*args, num_splits=splits)
        assert _maxabs(o, ref) <= TOL
        assert _maxabs(o, g["out"]) <= TOL


@pytest.mark.parametrize("L", [512, 4096, 16384])
@pytest.mark.parametrize("B", [1, 2, 4, 8, 16, 32, 64, 128, 256])
def test_config2_points_against_fp32(B, L, cuda_device):
    # every point of the config-2 grid at the default split count; (256, 16384)
    # is the largest pool: 262 145 pages, 2 GiB per K or V, K/V offsets up to
    # 5.4e8 elements and 4.2 M block-table entries, the size where the
    # reference's int32 offset guards (attn/core.py:24-34) start to matter;
    # this build addresses the pools with 64-bit offsets
    c = W.make_decode_case([L] * B, seed=7, device=cuda_device, generate_on_device=True)
    ref = torch_decode_fp32(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)
    o = cabi.decode_attention(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)
    assert torch.isfinite(o.float()).all()
    assert _maxabs(o, ref) <= TOL


def test_very_long_and_tiny_sequences_together(cuda_device):
    # one 262 144-key context (16 384 pages: 256 per split at the default 64
    # splits for B = 3) beside a 1-key and a 17-key sequence: most of the short
    # rows' splits have no page
    c = W.make_decode_case([262144, 1, 17], seed=9, device=cuda_device, generate_on_device=True)
    ref = torch.cat([torch_decode_fp32(c.q[:, b:b + 1], c.k, c.v, c.lens[b:b + 1],
                                       c.slot_ids[b:b + 1], c.block_table)
                     for b in range(3)], dim=1)
    for splits in (0, 1, 64):
        o = cabi.decode_attention(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table,
                                  num_splits=splits)
        assert torch.isfinite(o.float()).all()
        assert _maxabs(o, ref) <= TOL


@pytest.mark.parametrize("B,seed", [(3, 1), (37, 2), (200, 3)])
def test_ragged_batches(B, seed, cuda_device):
    # lengths drawn from 0 .. 9000 (zeros included) in one batch, default and
    # explicit split counts; zero-length rows must come out exactly zero
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(0, 9001, (B,), generator=g)
    lens[::7] = 0
    lens = lens.tolist()
    c = W.make_decode_case(lens, seed=seed, device=cuda_device, generate_on_device=True)
    parts = []
    for b, L in enumerate(lens):
        if L == 0:
            parts.append(torch.zeros(1, 1, 14, 64, dtype=torch.float16, device=cuda_device))
        else:
            parts.append(torch_decode_fp32(c.q[:, b:b + 1], c.k, c.v, c.lens[b:b + 1],
                                           c.slot_ids[b:b + 1], c.block_table))
    ref = torch.cat(parts, dim=1)
    zero = torch.tensor([L == 0 for L in lens], device=cuda_device)
    for splits in (0, 1, 5):
        o = cabi.decode_attention(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table,
                                  num_splits=splits)
        assert _maxabs(o, ref) <= TOL
        assert bool((o[0, zero] == 0).all())


@pytest.mark.parametrize("splits", [4, 8, 16, 32, 64])
def test_long_context_split_sweep(splits, cuda_device):
    # config 5 shape per GPU: 8 sequences x 32768 keys, pages scattered
    c = W.make_decode_case([32768] * 8, seed=5, device=cuda_device, generate_on_device=True)
    ref = torch_decode_fp32(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)
    o = cabi.decode_attention(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table,
                              num_splits=splits)
    assert _maxabs(o, ref) <= TOL


def test_torch_op_matches_cabi_bitwise(cuda_device):
    from custom_inference_engine_b200.attn import core
    g = load_golden("decode_random")
    q, k, v, lens, slot_ids, bt = _dev(g, cuda_device)
    S = cabi.decode_default_splits(slot_ids.shape[0], 0)
    a = core.gqa_decode_attention_op(q, k, v, lens, slot_ids=slot_ids, block_table=bt)
    b = cabi.decode_attention(q, k, v, lens, slot_ids, bt, num_splits=S)
    c = core.decode_gqa_attention(q, k, v, lens, slot_ids, bt, num_programs=S)
    assert torch.equal(a, b) and torch.equal(a, c)


def test_strided_pool_view(cuda_device):
    # K/V pools that are views into a larger buffer (page stride > H_kv*16*64)
    g = load_golden("decode_random")
    q, k, v, lens, slot_ids, bt = _dev(g, cuda_device)
    big_k = torch.zeros(k.shape[0], 3, 16, 64, dtype=k.dtype, device=cuda_device)
    big_v = torch.zeros_like(big_k)
    big_k[:, :2] = k
    big_v[:, :2] = v
    o = cabi.decode_attention(q, big_k[:, :2], big_v[:, :2], lens, slot_ids, bt, num_splits=2)
    assert _maxabs(o, g["out"]) <= TOL


def test_nonfinite_stale_rows_do_not_leak(cuda_device):
    # rows past a sequence's end inside its last page hold NaN: the output
    # must not see them (the reference masks them at load time)
    c = W.make_decode_case([20, 33], seed=3)
    ref = oracle.decode_attention_fp32(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)
    k, v = c.k.clone(), c.v.clone()
    for b, L in enumerate([20, 33]):
        last = int(c.block_table[b + 1, (L - 1) // 16])
        k[last, :, L % 16:] = float("nan")
        v[last, :, L % 16:] = float("nan")
    args = [t.to(cuda_device) for t in (c.q, k, v, c.lens, c.slot_ids, c.block_table)]
    o = cabi.decode_attention(*args, num_splits=1)
    assert _maxabs(o, ref) <= TOL


def test_invalid_arguments_rejected(cuda_device):
    g = load_golden("decode_random")
    q, k, v, lens, slot_ids, bt = _dev(g, cuda_device)
    with pytest.raises(RuntimeError, match="UNSUPPORTED"):
        cabi.decode_attention(q[..., :32].contiguous(), k[..., :32].contiguous(),
                              v[..., :32].contiguous(), lens, slot_ids, bt)
    with pytest.raises(RuntimeError, match="WORKSPACE"):
        cabi.decode_attention(q, k, v, lens, slot_ids, bt, num_splits=4,
                              workspace=torch.empty(4, dtype=torch.float32, device=cuda_device))
    from custom_inference_engine_b200.attn import core
    with pytest.raises(RuntimeError):
        core.gqa_decode_attention_op(q, k, v, lens[:-1], slot_ids=slot_ids, block_table=bt)


def test_out_of_range_slot_and_page_flag_device_errors(cuda_device):
    g = load_golden("decode_random")
    q, k, v, lens, slot_ids, bt = _dev(g, cuda_device)
    bad_slots = slot_ids.clone()
    bad_slots[0] = bt.shape[0] + 5
    cabi.decode_attention(q, k, v, lens, bad_slots, bt, num_splits=1)
    assert native.device_errors(0) & 1  # CIE_DEVERR_BAD_SLOT
    bad_bt = bt.clone()
    bad_bt[1, 0] = k.shape[0] + 100
    cabi.decode_attention(q, k, v, lens, slot_ids, bad_bt, num_splits=1)
    assert native.device_errors(0) & 4  # CIE_DEVERR_BAD_PAGE
