"""Free-running greedy generation through the reference engine's attention boundary.

The same driver runs on both sides of the end-to-end identity test
(``test_e2e_reference_engine_gpu.py``); what changes is where the top-level
``attn`` and ``kv_cache`` packages come from:

* the REFERENCE ENGINE: its own ``attn/core.py`` (``TritonQwen2Attention``, the
  ``inference::gqa_*`` Triton ops and kernels) and ``kv_cache/storage.py``,
  imported from the unmodified copy in baseline/_ref. Run as a script, in its own
  process, because both implementations register the same op names:
  ``python tests/e2e_greedy.py --reference-copy baseline/_ref --out ref.npz``;
* this package, through ``install_reference_aliases()`` (the test process).

Model: a random-init Qwen2 of the Qwen2.5-0.5B shape (hidden 896, 14 / 2 heads
of 64, MLP 4864, vocab 151936) with ``n_layers`` layers (24: the whole model),
HF's initialiser run on the GPU
after ``torch.manual_seed(0)``, fp16. Both processes build it on the same GPU
from the same seed and compare a checksum of the weights.

Schedule, as the reference's scheduler steps a batch (scheduler/scheduler.py):
mixed passes of at most ``TOKEN_BUDGET`` tokens carry one decode row for every
sequence whose prompt is done, then chunks of the remaining prompts in order
(a long prompt spans passes, its later chunks attending to K/V written by
earlier ones); once every prompt is in, batched decode passes. The model runs
eagerly, ``model(input_ids, position_ids, kv_manager=KVStorage,
metadata=AttentionMetadata, use_cache=False)`` (scheduler/decode_module.py:57-66,
scheduler/mixed_module.py:52-59), so the decoder body, the projections and the
lm_head are the same cuBLAS / PyTorch calls on both sides and only the attention
path (RoPE, K/V writes, attention kernels) differs. Every sequence stops after
``N_NEW`` tokens; each token is ``argmax`` of the fp16 logits, and the two
largest logits of every step are recorded with their token ids.
"""
from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[1]
PROMPT_LENS = (5, 40, 17, 130, 64, 1, 300, 33)
N_NEW = 32
TOKEN_BUDGET = 256
PAGE = 16


def build_model(device, n_layers: int):
    if str(REPO) not in sys.path:
        sys.path.insert(0, str(REPO))
    from custom_inference_engine_b200 import model_runner as MR

    cfg = MR.qwen2_config(num_hidden_layers=n_layers)
    return MR.random_qwen2(cfg, seed=0, device=device)


def weight_checksum(model) -> float:
    with torch.no_grad():
        return float(sum(p.double().sum().item() for p in model.parameters()))


def prompts(vocab: int):
    rng = np.random.default_rng(2025)
    return [rng.integers(0, vocab, size=n).tolist() for n in PROMPT_LENS]


def generate(model, device):
    """Greedy tokens (n_seq, N_NEW), and for every step the two best token ids
    and their logits (n_seq, N_NEW, 2)."""
    from attn.core import use_triton_attention
    from attn.metadata import AttentionMetadata
    from kv_cache.storage import KVStorage

    use_triton_attention(model)
    ps = prompts(model.config.vocab_size)
    n = len(ps)
    kv = KVStorage(model.config, max_cache_len=4096, page_size=PAGE, n_slots=n + 1,
                   device=device, dtype=torch.float16)
    g = torch.Generator().manual_seed(3)
    free = (torch.randperm(kv.n_pages - 1, generator=g) + 1).tolist()
    pages = {}
    for i, p in enumerate(ps):
        k = math.ceil((len(p) + N_NEW + 1) / PAGE)
        pages[i + 1], free = free[:k], free[k:]
        kv.block_table[i + 1, :k] = torch.tensor(pages[i + 1], device=device)

    slot_len = [0] * (n + 1)                 # host mirror of kv.lens
    fed = [0] * n                            # prompt tokens written so far
    tokens = [[] for _ in range(n)]
    top_vals = [[] for _ in range(n)]
    top_ids = [[] for _ in range(n)]

    def take(i, logits_row):
        top = torch.topk(logits_row.float(), 2)
        tokens[i].append(int(logits_row.argmax()))
        top_vals[i].append(top.values.tolist())
        top_ids[i].append(top.indices.tolist())

    with torch.inference_mode():
        while any(len(t) < N_NEW for t in tokens):
            if any(f < len(p) for f, p in zip(fed, ps)):
                # mixed pass: decode rows first, then prompt chunks
                seqs, chunks = [], []
                budget = TOKEN_BUDGET
                for i in range(n):
                    if fed[i] == len(ps[i]) and len(tokens[i]) < N_NEW:
                        seqs.append(i)
                        chunks.append([tokens[i][-1]])
                        budget -= 1
                for i in range(n):
                    if fed[i] < len(ps[i]) and budget > 0:
                        c = min(budget, len(ps[i]) - fed[i])
                        seqs.append(i)
                        chunks.append(ps[i][fed[i]:fed[i] + c])
                        budget -= c
                T = sum(len(c) for c in chunks)
                cu = np.concatenate([[0], np.cumsum([len(c) for c in chunks])]).tolist()
                pos = [slot_len[i + 1] + j for i, c in zip(seqs, chunks) for j in range(len(c))]
                pg = [pages[i + 1][(slot_len[i + 1] + j) // PAGE]
                      for i, c in zip(seqs, chunks) for j in range(len(c))]
                md = AttentionMetadata(token_count=T, full_decode=False, device=device)
                md.prepare_full_graph(len(seqs))
                md.write_slot_ids([i + 1 for i in seqs])
                md.write_cu_seqlens(cu)
                md.write_pages(pg)
                md.write_offsets([p % PAGE for p in pos])
                ids = torch.tensor([[t for c in chunks for t in c]], device=device)
                out = model(input_ids=ids, position_ids=torch.tensor([pos], device=device),
                            kv_manager=kv, metadata=md, use_cache=False)
                kv.mixed_advance(torch.tensor([i + 1 for i in seqs], device=device),
                                 torch.tensor([len(c) for c in chunks], device=device))
                for j, (i, c) in enumerate(zip(seqs, chunks)):
                    slot_len[i + 1] += len(c)
                    if fed[i] < len(ps[i]):
                        fed[i] += len(c)
                        if fed[i] < len(ps[i]):
                            continue           # prompt not finished: no token yet
                    take(i, out.logits[0, cu[j + 1] - 1])
            else:
                seqs = [i for i in range(n) if len(tokens[i]) < N_NEW]
                md = AttentionMetadata(token_count=len(seqs), full_decode=True, device=device)
                md.prepare_full_graph(len(seqs))
                md.write_slot_ids([i + 1 for i in seqs])
                ids = torch.tensor([[tokens[i][-1] for i in seqs]], device=device)
                pos = torch.tensor([[slot_len[i + 1] for i in seqs]], device=device)
                out = model(input_ids=ids, position_ids=pos, kv_manager=kv, metadata=md,
                            use_cache=False)
                kv.decode_advance(slot_ids=md.slot_ids)
                for j, i in enumerate(seqs):
                    slot_len[i + 1] += 1
                    take(i, out.logits[0, j])
    return np.array(tokens), np.array(top_ids), np.array(top_vals, dtype=np.float32)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-copy", required=True,
                    help="unmodified copy of the reference engine (baseline/_ref)")
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    ref = str(Path(args.reference_copy).resolve())
    sys.path.insert(0, ref)
    import attn.core
    assert attn.core.__file__.startswith(ref), attn.core.__file__
    dev = torch.device("cuda:0")
    model = build_model(dev, args.layers)
    toks, top_ids, top_vals = generate(model, dev)
    np.savez(args.out, tokens=toks, top_ids=top_ids, top_vals=top_vals,
             checksum=weight_checksum(model))
    return 0


if __name__ == "__main__":
    sys.exit(main())
