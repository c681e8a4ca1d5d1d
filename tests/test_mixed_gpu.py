"""Parity of the tcgen05 varlen mixed-attention kernel (C ABI and torch op).

Bar: max-abs <= 2e-3 on fp16 outputs of every row that belongs to a
sequence, against the reference Triton kernel's outputs (golden fixtures)
and fp32 causal softmax attention (CPU oracle at small sizes, the same math
in torch fp32 on the GPU at config-3 sizes). Rows outside every sequence are
never written.
"""
import pytest
import torch

from conftest import load_golden
from custom_inference_engine_b200 import cabi, native
from custom_inference_engine_b200 import workloads as W
import oracle

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _maxabs(a, b):
    return (a.float().cpu() - b.float().cpu()).abs().max().item()


def torch_mixed_fp32(c):
    """fp32 causal reference on the device, one sequence at a time."""
    out = torch.zeros(c.q.shape, dtype=torch.float32, device=c.q.device)
    cu = c.cu_seqlens.tolist()
    kvl = c.kv_lens.tolist()
    slots = c.slot_ids.tolist()
    for b in range(len(slots)):
        s0, s1 = cu[b], cu[b + 1]
        L = s1 - s0
        if L <= 0:
            continue
        n_keys = kvl[b] + L
        n = (n_keys + 15) // 16
        pages = c.block_table[slots[b], :n]
        kk = c.k[pages].permute(1, 0, 2, 3).reshape(2, n * 16, 64)[:, :n_keys].float()
        vv = c.v[pages].permute(1, 0, 2, 3).reshape(2, n * 16, 64)[:, :n_keys].float()
        qq = c.q[0, s0:s1].float().view(L, 2, 7, 64).permute(1, 0, 2, 3).reshape(2, L * 7, 64)
        s = torch.matmul(qq, kk.transpose(1, 2)) * 0.125
        pos = kvl[b] + torch.arange(L, device=c.q.device).repeat_interleave(7)
        keys = torch.arange(n_keys, device=c.q.device)
        s = s.masked_fill(keys[None, None, :] > pos[None, :, None], float("-inf"))
        o = torch.matmul(torch.softmax(s, dim=-1), vv).view(2, L, 7, 64).permute(1, 0, 2, 3)
        out[0, s0:s1] = o.reshape(L, 14, 64)
    return out.to(torch.float16)


def _run(c, sentinel=None, splits=0):
    out = None
    if sentinel is not None:
        out = torch.full_like(c.q, sentinel)
    return cabi.mixed_attention(c.q, c.k, c.v, c.max_seqlen, c.cu_seqlens, c.kv_lens,
                                c.slot_ids, c.block_table, out=out, num_splits=splits)


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    native.device_errors(0, clear=True)
    yield
    assert native.device_errors(0, clear=True) == 0


def _case_from_golden(g, dev):
    return W.MixedCase(q=g["q"].to(dev), k=g["k"].to(dev), v=g["v"].to(dev),
                       max_seqlen=int(g["max_seqlen"]), cu_seqlens=g["cu_seqlens"].to(dev),
                       kv_lens=g["kv_lens"].to(dev), slot_ids=g["slot_ids"].to(dev),
                       block_table=g["block_table"].to(dev))


@pytest.mark.parametrize("splits", [1, 3, 16, 0])
@pytest.mark.parametrize("name", ["mixed_small", "mixed_edges", "mixed_config3_small"])
def test_golden_cases_cabi(name, splits, cuda_device):
    g = load_golden(name)
    c = _case_from_golden(g, cuda_device)
    o = _run(c, sentinel=7.0, splits=splits)
    rows = oracle.valid_token_rows(g["cu_seqlens"], g["q"].shape[1])
    assert _maxabs(o[0, rows.to(cuda_device)], g["out"][0, rows]) <= TOL
    ref = oracle.mixed_attention_fp32(g["q"], g["k"], g["v"], int(g["max_seqlen"]),
                                      g["cu_seqlens"], g["kv_lens"], g["slot_ids"],
                                      g["block_table"])
    assert _maxabs(o[0, rows.to(cuda_device)], ref[0, rows]) <= TOL
    # rows outside every sequence keep the caller's contents
    assert bool((o[0, (~rows).to(cuda_device)] == 7.0).all())


@pytest.mark.parametrize("chunks,kvs", [
    ([1], [0]),                              # single key
    ([1] * 6, [0, 1, 15, 16, 127, 128]),     # decode rows at page / block edges
    ([18, 19, 36, 37], [0, 5, 128, 129]),    # query-tile edges
    ([128, 129, 255], [127, 0, 1]),          # key-block edges
    ([300], [4000]),
    ([36, 5], [60000, 30000]),               # pairs cut into the most pieces (merge of 16)
    ([2048], [0]),                           # one long prompt: every tile pair of a sequence
])
def test_edge_shapes(chunks, kvs, cuda_device):
    c = W.make_mixed_case(chunks, kvs, seed=sum(chunks) + sum(kvs))
    ref = oracle.mixed_attention_fp32(c.q, c.k, c.v, c.max_seqlen, c.cu_seqlens, c.kv_lens,
                                      c.slot_ids, c.block_table)
    cd = W.MixedCase(**{f: (getattr(c, f).to(cuda_device) if torch.is_tensor(getattr(c, f))
                            else getattr(c, f)) for f in c.__dataclass_fields__})
    for splits in (1, 4, 0):
        o = _run(cd, splits=splits)
        assert _maxabs(o, ref) <= TOL


def test_config3_full(cuda_device):
    chunk, kv = W.config3_shape(seed=0)
    c = W.make_mixed_case(chunk, kv, seed=0, device=cuda_device, max_seqlen=2048,
                          generate_on_device=True)
    ref = torch_mixed_fp32(c)
    for splits in (0, 1, 5):
        o = _run(c, splits=splits)
        assert torch.isfinite(o.float()).all()
        assert _maxabs(o, ref) <= TOL


@pytest.mark.parametrize("seed", [1, 2, 3, 4])
def test_config3_other_draws(seed, cuda_device):
    # further draws of the config-3 distribution (32 sequences, half of them
    # decode rows, chunks up to 512 tokens within a 2048-token budget, cached
    # lengths up to 8192), at the default plan
    chunk, kv = W.config3_shape(seed=seed)
    c = W.make_mixed_case(chunk, kv, seed=seed, device=cuda_device, max_seqlen=2048,
                          generate_on_device=True)
    o = _run(c)
    assert _maxabs(o, torch_mixed_fp32(c)) <= TOL


def test_512_token_chunks(cuda_device):
    g = torch.Generator().manual_seed(1)
    kv = torch.randint(0, 8193, (4,), generator=g).tolist()
    c = W.make_mixed_case([512] * 4, kv, seed=1, device=cuda_device, generate_on_device=True)
    ref = torch_mixed_fp32(c)
    for splits in (0, 1, 8):
        o = _run(c, splits=splits)
        assert _maxabs(o, ref) <= TOL


def test_nonfinite_stale_rows_do_not_leak(cuda_device):
    c = W.make_mixed_case([5, 20], [11, 40], seed=4)
    ref = oracle.mixed_attention_fp32(c.q, c.k, c.v, c.max_seqlen, c.cu_seqlens, c.kv_lens,
                                      c.slot_ids, c.block_table)
    k, v = c.k.clone(), c.v.clone()
    for b, n_keys in enumerate([16, 60]):
        last = int(c.block_table[b + 1, (n_keys - 1) // 16])
        if n_keys % 16:
            k[last, :, n_keys % 16:] = float("nan")
            v[last, :, n_keys % 16:] = float("nan")
    # the unused page 0 and every page no slot owns are NaN too
    used = set(c.block_table[1:].flatten().tolist())
    for p in range(k.shape[0]):
        if p not in used or p == 0:
            k[p] = float("nan")
            v[p] = float("nan")
    dev = cuda_device
    cd = W.MixedCase(q=c.q.to(dev), k=k.to(dev), v=v.to(dev), max_seqlen=c.max_seqlen,
                     cu_seqlens=c.cu_seqlens.to(dev), kv_lens=c.kv_lens.to(dev),
                     slot_ids=c.slot_ids.to(dev), block_table=c.block_table.to(dev))
    for splits in (1, 2):
        o = _run(cd, splits=splits)
        assert _maxabs(o, ref) <= TOL


def test_torch_op_matches_cabi_bitwise(cuda_device):
    from custom_inference_engine_b200.attn import core
    g = load_golden("mixed_edges")
    c = _case_from_golden(g, cuda_device)
    rows = oracle.valid_token_rows(g["cu_seqlens"], g["q"].shape[1]).to(cuda_device)
    a = core.gqa_mixed_attention_op(c.q, c.k, c.v, kv_lens=c.kv_lens, max_seqlen=c.max_seqlen,
                                    cu_seqlens=c.cu_seqlens, slot_ids=c.slot_ids,
                                    block_table=c.block_table)
    b = _run(c)
    d = core.mixed_gqa_attention(c.q, c.k, c.v, c.max_seqlen, c.cu_seqlens, c.kv_lens,
                                 c.slot_ids, c.block_table)
    assert torch.equal(a[0, rows], b[0, rows]) and torch.equal(a[0, rows], d[0, rows])
