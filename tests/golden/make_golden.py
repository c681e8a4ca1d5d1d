"""Generate golden fixtures from the reference engine's own kernels.

Run once on a CPU host where the reference project is checked out:

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

The reference's Triton kernels (kernels/decode_attention.py,
kernels/prefill_attention.py) run through their host functions
``attn.core.decode_gqa_attention`` / ``attn.core.mixed_gqa_attention``
(attn/core.py:13-111) under ``TRITON_INTERPRET=1``, with the tile configs the
reference registers its ops with (attn/core.py:114-116). The KV-page
scatter goldens come from the reference ``KVStorage.decode_update`` /
``mixed_update`` (kv_cache/storage.py:62-122) run on CPU tensors.

Inputs are built by ``custom_inference_engine_b200.workloads`` from seeds
(numpy PCG64, platform independent). Small cases store their inputs in the
``.npz``; the config-1 case stores the seed and a SHA-256 of the regenerated
inputs so the test can prove it rebuilt exactly the same tensors.

The reference registers op names that collide with this package's
(``inference::gqa_*``), so this script must not import
``custom_inference_engine_b200.attn``; it only imports ``workloads``.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def sha256_tensors(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().numpy().tobytes())
    return h.hexdigest()


def _np(t):
    return t.detach().cpu().numpy()


def decode_cases(W):
    cases = {}
    # edge lengths around page boundaries, a zero-length row and the
    # padding convention (slot 0, lens 1 -> page 0, attn/metadata.py:33-37)
    lens = [1, 15, 16, 17, 33, 100, 255, 256, 257, 0, 1]
    c = W.make_decode_case(lens, seed=11)
    c.slot_ids[-1] = 0
    cases["decode_edges"] = c
    c = W.make_decode_case([int(x) for x in np.random.default_rng(5).integers(1, 301, 6)],
                           seed=5)
    cases["decode_random"] = c
    return cases


def mixed_cases(W):
    cases = {}
    cases["mixed_small"] = W.make_mixed_case([1, 20, 1, 37], [50, 0, 7, 100], seed=21)
    cases["mixed_edges"] = W.make_mixed_case(
        [16, 17, 1, 64, 65, 3, 18, 36], [0, 15, 16, 31, 1, 200, 33, 0],
        seed=22, pad_batch=2, max_seqlen=220 + 13)
    chunk, kv = W.config3_shape(seed=3, n_seqs=8, budget=256, max_kv=256)
    cases["mixed_config3_small"] = W.make_mixed_case(chunk, kv, seed=23)
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of eteboun/custom_inference_engine")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()

    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    from custom_inference_engine_b200 import workloads as W
    import attn.core as ref_core                      # reference host functions
    from kv_cache.storage import KVStorage            # reference KV storage

    out = Path(args.out)
    dcfg = dict(ref_core.GQA_DECODE_CONFIG)
    mcfg = dict(ref_core.GQA_PREFILL_CONFIG)

    def run_decode(c):
        return ref_core.decode_gqa_attention(c.q, c.k, c.v, c.lens, c.slot_ids,
                                             c.block_table, **dcfg)

    def run_mixed(c):
        return ref_core.mixed_gqa_attention(c.q, c.k, c.v, max_seqlen=c.max_seqlen,
                                            cu_seqlens=c.cu_seqlens, kv_lens=c.kv_lens,
                                            slot_ids=c.slot_ids, block_table=c.block_table,
                                            **mcfg)

    for name, c in decode_cases(W).items():
        o = run_decode(c)
        np.savez_compressed(out / f"{name}.npz", q=_np(c.q), k=_np(c.k), v=_np(c.v),
                            lens=_np(c.lens), slot_ids=_np(c.slot_ids),
                            block_table=_np(c.block_table), out=_np(o),
                            num_programs=dcfg["num_programs"], block_n=dcfg["BLOCK_N"])
        print(name, tuple(o.shape))

    # config 1 in full: inputs regenerated from the seed, pinned by hash
    lens = W.config1_lens()
    c = W.make_decode_case(lens, seed=0)
    o = run_decode(c)
    np.savez_compressed(out / "decode_config1.npz", out=_np(o), lens=np.array(lens),
                        seed=0, sha256=sha256_tensors(c.q, c.k, c.v, c.block_table),
                        num_programs=dcfg["num_programs"], block_n=dcfg["BLOCK_N"])
    print("decode_config1", tuple(o.shape))

    for name, c in mixed_cases(W).items():
        o = run_mixed(c)
        np.savez_compressed(out / f"{name}.npz", q=_np(c.q), k=_np(c.k), v=_np(c.v),
                            max_seqlen=c.max_seqlen, cu_seqlens=_np(c.cu_seqlens),
                            kv_lens=_np(c.kv_lens), slot_ids=_np(c.slot_ids),
                            block_table=_np(c.block_table), out=_np(o),
                            block_m=mcfg["BLOCK_M"], block_n=mcfg["BLOCK_N"])
        print(name, tuple(o.shape))

    # KV-page scatter through the reference KVStorage
    cfg = types.SimpleNamespace(num_hidden_layers=1, num_attention_heads=14,
                                num_key_value_heads=2, hidden_size=896, head_dim=64)
    rng = np.random.default_rng(31)
    kv = KVStorage(cfg, max_cache_len=40 * 16, page_size=16, n_slots=6,
                   device="cpu", dtype=torch.float16)
    kv.keys[0].copy_(torch.from_numpy(rng.standard_normal(kv.keys[0].shape,
                                                          dtype=np.float32).astype(np.float16)))
    kv.values[0].copy_(torch.from_numpy(rng.standard_normal(kv.values[0].shape,
                                                            dtype=np.float32).astype(np.float16)))
    perm = torch.from_numpy(rng.permutation(kv.n_pages - 1).astype(np.int64)) + 1
    for s in range(1, 6):
        kv.block_table[s, :7] = perm[(s - 1) * 7:s * 7]
    kv.lens[1:6] = torch.tensor([0, 15, 16, 47, 111])
    k0, v0, lens0, bt0 = (kv.keys[0].clone(), kv.values[0].clone(), kv.lens.clone(),
                          kv.block_table.clone())
    slot_ids = torch.tensor([3, 1, 5, 2, 4, 0, 0])          # padded with slot 0
    B = slot_ids.shape[0]
    fused = torch.from_numpy(rng.standard_normal((1, B, 18 * 64), dtype=np.float32)
                             .astype(np.float16))
    k_proj = fused[..., 14 * 64:16 * 64].view(1, B, 2, 64)   # strided views, as the
    v_proj = fused[..., 16 * 64:18 * 64].view(1, B, 2, 64)   # split of the QKV linear
    kv.decode_update(0, slot_ids, k_proj, v_proj)
    np.savez_compressed(out / "kv_decode_update.npz", k_before=_np(k0), v_before=_np(v0),
                        lens=_np(lens0), block_table=_np(bt0), slot_ids=_np(slot_ids),
                        fused=_np(fused), k_after=_np(kv.keys[0]), v_after=_np(kv.values[0]))
    print("kv_decode_update")

    kv.keys[0].copy_(k0)
    kv.values[0].copy_(v0)
    T = 23
    pages = torch.zeros(T, dtype=torch.int64)
    offsets = torch.zeros(T, dtype=torch.int64)
    pos = torch.arange(19) + 5                               # slot 2, rows 5..23
    pages[:19] = bt0[2, pos // 16]
    offsets[:19] = pos % 16                                  # rows 19..22 pad -> page 0
    fused = torch.from_numpy(rng.standard_normal((1, T, 18 * 64), dtype=np.float32)
                             .astype(np.float16))
    k_proj = fused[..., 14 * 64:16 * 64].view(1, T, 2, 64)
    v_proj = fused[..., 16 * 64:18 * 64].view(1, T, 2, 64)
    kv.mixed_update(0, pages, offsets, k_proj, v_proj)
    np.savez_compressed(out / "kv_mixed_update.npz", k_before=_np(k0), v_before=_np(v0),
                        pages=_np(pages), offsets=_np(offsets), fused=_np(fused),
                        k_after=_np(kv.keys[0]), v_after=_np(kv.values[0]))
    print("kv_mixed_update")


if __name__ == "__main__":
    main()
