"""Pins the CPU oracle against fixtures produced by the reference kernels.

The fixtures come from the reference's own Triton kernels run under the
Triton CPU interpreter (tests/golden/make_golden.py). Two oracles are
checked:

* ``*_blockwise`` restates the reference kernels step for step, so it must
  agree with them to within fp32 summation-order noise;
* ``*_fp32`` is plain fp32 softmax attention, the tolerance oracle for the
  CUDA kernels; it must agree with the reference within max-abs 2e-3.
"""
import hashlib

import numpy as np
import pytest
import torch

from conftest import load_golden
from custom_inference_engine_b200 import workloads as W
import oracle

TOL_FP32 = 2e-3          # north-star tolerance on fp16 outputs
TOL_BLOCKWISE = 1e-3     # fp16 rounding of P at different summation order

DECODE = ["decode_edges", "decode_random"]
MIXED = ["mixed_small", "mixed_edges", "mixed_config3_small"]


def _maxabs(a, b):
    return (a.float() - b.float()).abs().max().item()


@pytest.mark.parametrize("name", DECODE)
def test_decode_oracles_match_reference(name):
    g = load_golden(name)
    args = (g["q"], g["k"], g["v"], g["lens"], g["slot_ids"], g["block_table"])
    ref = g["out"]
    assert torch.isfinite(ref.float()).all()
    assert _maxabs(oracle.decode_attention_fp32(*args), ref) <= TOL_FP32
    bw = oracle.decode_attention_blockwise(*args, num_programs=int(g["num_programs"]),
                                           block_n=int(g["block_n"]))
    assert _maxabs(bw, ref) <= TOL_BLOCKWISE


def test_decode_zero_length_row_is_zero():
    g = load_golden("decode_edges")
    zero_rows = (g["lens"] == 0).nonzero().flatten()
    assert len(zero_rows) == 1
    assert (g["out"][0, zero_rows] == 0).all()
    o = oracle.decode_attention_fp32(g["q"], g["k"], g["v"], g["lens"], g["slot_ids"],
                                     g["block_table"])
    assert (o[0, zero_rows] == 0).all()


def test_decode_config1_regenerates_and_matches():
    g = load_golden("decode_config1")
    lens = W.config1_lens()
    assert lens == g["lens"].tolist()
    c = W.make_decode_case(lens, seed=int(g["seed"]))
    h = hashlib.sha256()
    for t in (c.q, c.k, c.v, c.block_table):
        h.update(t.contiguous().numpy().tobytes())
    assert h.hexdigest() == g["sha256"], "seeded inputs differ from the fixture's"
    o = oracle.decode_attention_fp32(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)
    assert _maxabs(o, g["out"]) <= TOL_FP32


@pytest.mark.parametrize("name", MIXED)
def test_mixed_oracles_match_reference(name):
    g = load_golden(name)
    args = (g["q"], g["k"], g["v"], int(g["max_seqlen"]), g["cu_seqlens"], g["kv_lens"],
            g["slot_ids"], g["block_table"])
    T = g["q"].shape[1]
    rows = oracle.valid_token_rows(g["cu_seqlens"], T)
    ref = g["out"][0, rows]
    assert torch.isfinite(ref.float()).all()
    assert _maxabs(oracle.mixed_attention_fp32(*args)[0, rows], ref) <= TOL_FP32
    bw = oracle.mixed_attention_blockwise(*args, block_m=int(g["block_m"]),
                                          block_n=int(g["block_n"]))
    assert _maxabs(bw[0, rows], ref) <= TOL_BLOCKWISE


def test_decode_update_oracle_bit_exact():
    g = load_golden("kv_decode_update")
    k, v = g["k_before"].clone(), g["v_before"].clone()
    fused = g["fused"]
    B = fused.shape[1]
    k_proj = fused[..., 14 * 64:16 * 64].view(1, B, 2, 64)
    v_proj = fused[..., 16 * 64:18 * 64].view(1, B, 2, 64)
    oracle.decode_update_ref(k, v, g["lens"], g["slot_ids"], g["block_table"], k_proj, v_proj)
    # page 0 absorbs padded rows; duplicate writes there have no defined winner
    assert torch.equal(k[1:], g["k_after"][1:])
    assert torch.equal(v[1:], g["v_after"][1:])
    assert not torch.equal(g["k_after"][1:], g["k_before"][1:])


def test_mixed_update_oracle_bit_exact():
    g = load_golden("kv_mixed_update")
    k, v = g["k_before"].clone(), g["v_before"].clone()
    fused = g["fused"]
    T = fused.shape[1]
    k_proj = fused[..., 14 * 64:16 * 64].view(1, T, 2, 64)
    v_proj = fused[..., 16 * 64:18 * 64].view(1, T, 2, 64)
    oracle.mixed_update_ref(k, v, g["pages"], g["offsets"], k_proj, v_proj)
    assert torch.equal(k[1:], g["k_after"][1:])
    assert torch.equal(v[1:], g["v_after"][1:])


def test_rope_oracle_matches_transformers_bit_exact():
    """oracle.rope_ref is transformers' Qwen2 apply_rotary_pos_emb (the
    function the reference calls, attn/core.py:193-198) bit for bit on fp16
    CPU tensors, for q and k head counts, at positions up to 32767."""
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    g = torch.Generator().manual_seed(0)
    T = 33
    q = (torch.randn(1, T, 14, 64, generator=g) * 3).half()
    k = (torch.randn(1, T, 2, 64, generator=g) * 3).half()
    pos = torch.randint(0, 32768, (T,), generator=g).float()
    inv = 1.0 / (1e6 ** (torch.arange(0, 64, 2).float() / 64))
    emb = torch.cat((pos[:, None] * inv, pos[:, None] * inv), dim=-1)
    cos, sin = emb.cos()[None].half(), emb.sin()[None].half()
    q_hf, k_hf = apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=2)
    assert torch.equal(oracle.rope_ref(q, cos, sin), q_hf)
    assert torch.equal(oracle.rope_ref(k, cos, sin), k_hf)
