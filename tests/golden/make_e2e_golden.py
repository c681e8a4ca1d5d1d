"""Greedy tokens of the REFERENCE ENGINE on a small seeded model (golden fixture).

Run once on a CPU host where the reference project is checked out:

    python tests/golden/make_e2e_golden.py --reference <path-to-reference-checkout>

A 2-layer random-init Qwen2 with the 0.5B head layout (14 query / 2 kv heads,
head_dim 64; hidden 896, MLP 2048, vocab 4096; HF initialiser after
``torch.manual_seed(0)`` on the CPU, then fp16) gets the reference's attention
module (``attn.core.use_triton_attention``, attn/core.py:139-250) and is driven
the way the reference's scheduler modules drive it: one mixed pass over all
prompts with the reference ``AttentionMetadata`` (attn/metadata.py) and
``KVStorage`` (kv_cache/storage.py), then batched decode steps
(scheduler/decode_module.py:56-70). The reference kernels run under
``TRITON_INTERPRET=1``; its ``triton_op`` wrappers do not run in the
interpreter, so ``gqa_*_attention_op`` are pointed at the host functions
``decode_gqa_attention`` / ``mixed_gqa_attention`` with the reference's tile
configs (attn/core.py:114-116), which is what the ops call.

The fixture holds the prompts, the greedy tokens and, per step, the margin
between the two largest logits (how far each token is from a tie) and the five
largest logits with their token ids.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]

PROMPT_LENS = (5, 40, 17, 70)
N_NEW = 8
PAGE = 16


def prompts():
    rng = np.random.default_rng(2024)
    return [rng.integers(0, 4096, size=n).tolist() for n in PROMPT_LENS]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of eteboun/custom_inference_engine")
    ap.add_argument("--out", default=str(HERE / "e2e_reference_tokens.npz"))
    args = ap.parse_args()

    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    from transformers import Qwen2Config, Qwen2ForCausalLM

    import attn.core as ref_core                      # reference attention module
    from attn.metadata import AttentionMetadata       # reference metadata
    from kv_cache.storage import KVStorage            # reference KV storage

    dcfg = dict(ref_core.GQA_DECODE_CONFIG)
    mcfg = dict(ref_core.GQA_PREFILL_CONFIG)
    ref_core.gqa_decode_attention_op = (
        lambda q, k, v, lens, slot_ids, block_table:
        ref_core.decode_gqa_attention(q, k, v, lens, slot_ids, block_table, **dcfg))
    ref_core.gqa_mixed_attention_op = (
        lambda q, k, v, kv_lens, max_seqlen, cu_seqlens, slot_ids, block_table:
        ref_core.mixed_gqa_attention(q, k, v, max_seqlen=max_seqlen, cu_seqlens=cu_seqlens,
                                     kv_lens=kv_lens, slot_ids=slot_ids,
                                     block_table=block_table, **mcfg))

    cfg = Qwen2Config(hidden_size=896, intermediate_size=2048, num_hidden_layers=2,
                      num_attention_heads=14, num_key_value_heads=2, vocab_size=4096,
                      max_position_embeddings=32768, rope_theta=1000000.0,
                      rms_norm_eps=1e-6, tie_word_embeddings=True, hidden_act="silu",
                      initializer_range=0.02)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    model = Qwen2ForCausalLM(cfg).to(torch.float16).eval()
    ref_core.use_triton_attention(model)

    ps = prompts()
    B = len(ps)
    n_slots = B + 1
    kv = KVStorage(cfg, max_cache_len=1024, page_size=PAGE, n_slots=n_slots, device="cpu",
                   dtype=torch.float16)
    # slot s (1..B) owns pages 1 + 8 (s - 1) .. : 8 pages of 16 tokens each
    for s in range(1, n_slots):
        kv.block_table[s, :8] = torch.arange(1 + 8 * (s - 1), 1 + 8 * s)
    slots = list(range(1, n_slots))

    tokens = [[] for _ in range(B)]
    margins = [[] for _ in range(B)]
    top_ids = [[] for _ in range(B)]
    top_vals = [[] for _ in range(B)]

    def take(logits):
        top = torch.topk(logits.float(), 5, dim=-1)
        for i in range(B):
            tokens[i].append(int(top.indices[i, 0]))
            margins[i].append(float(top.values[i, 0] - top.values[i, 1]))
            top_ids[i].append(top.indices[i].tolist())
            top_vals[i].append(top.values[i].tolist())

    with torch.inference_mode():
        # one mixed pass over every prompt
        T = sum(len(p) for p in ps)
        md = AttentionMetadata(token_count=T, full_decode=False, device="cpu")
        md.prepare_full_graph(B)
        md.write_slot_ids(slots)
        cu = np.concatenate([[0], np.cumsum([len(p) for p in ps])]).tolist()
        md.write_cu_seqlens(cu)
        pos = [i for p in ps for i in range(len(p))]
        pages = [int(kv.block_table[s, i // PAGE]) for s, p in zip(slots, ps)
                 for i in range(len(p))]
        md.write_pages(pages)
        md.write_offsets([i % PAGE for i in pos])
        out = model(input_ids=torch.tensor([[t for p in ps for t in p]]),
                    position_ids=torch.tensor([pos]), kv_manager=kv, metadata=md,
                    use_cache=False)
        kv.mixed_advance(torch.tensor(slots), torch.tensor([len(p) for p in ps]))
        take(out.logits[0, [c - 1 for c in cu[1:]]])
        # batched decode steps
        dmd = AttentionMetadata(token_count=B, full_decode=True, device="cpu")
        dmd.prepare_full_graph(B)
        dmd.write_slot_ids(slots)
        for _ in range(N_NEW - 1):
            ids = torch.tensor([[t[-1] for t in tokens]])
            posd = kv.lens[torch.tensor(slots)].view(1, -1)
            out = model(input_ids=ids, position_ids=posd, kv_manager=kv, metadata=dmd,
                        use_cache=False)
            kv.decode_advance(slot_ids=dmd.slot_ids)
            take(out.logits[0])

    np.savez_compressed(args.out, prompt_lens=np.array(PROMPT_LENS),
                        prompts=np.array([t for p in ps for t in p]),
                        tokens=np.array(tokens), margins=np.array(margins),
                        top_ids=np.array(top_ids), top_vals=np.array(top_vals, dtype=np.float32),
                        seed=0)
    print("tokens", tokens)
    print("min margin", float(np.min(margins)))


if __name__ == "__main__":
    main()
