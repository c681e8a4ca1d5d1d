"""A paged Qwen2 runner over the CUDA attention ops: chunked prefill, greedy decode.

Drives a Hugging Face ``Qwen2ForCausalLM`` whose attention modules have been
swapped by ``attn.core.use_cuda_attention`` the way the reference's scheduler
modules drive theirs: ``model.model(input_ids, position_ids, kv_manager=...,
metadata=..., use_cache=False)`` with a ``KVStorage`` and an
``AttentionMetadata`` (scheduler/decode_module.py:57-66,
scheduler/mixed_module.py:129-132 of the reference). Prompts are prefilled through
``inference::gqa_mixed_attention`` in chunks of at most ``token_budget`` tokens;
decode steps go through ``inference::gqa_decode_attention`` and can be captured
in one CUDA graph per batch (embedding, 24 layers, lm_head, argmax and the
slot-length advance).

By default the decoder body around the attention runs through
``FusedQwen2Body`` (RMSNorm, residual adds and SiLU-mul as CUDA kernels of this
package, about 10 launches per layer); ``fused_body=False`` runs HF's modules.

This is the harness that measures Qwen2.5-0.5B-shape tokens/s and checks greedy
tokens against HF's own attention; ``serving.py`` drives it with a request
queue (Poisson arrivals, continuous batching). Every admitted slot gets enough
pages up front for its prompt plus its new tokens.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

# Qwen2.5-0.5B-Instruct architecture (the reference's model, README.md:3).
QWEN2_05B = dict(hidden_size=896, intermediate_size=4864, num_hidden_layers=24,
                 num_attention_heads=14, num_key_value_heads=2, vocab_size=151936,
                 max_position_embeddings=32768, rope_theta=1000000.0, rms_norm_eps=1e-6,
                 tie_word_embeddings=True, hidden_act="silu", initializer_range=0.02)

PAGE_SIZE = 16


def qwen2_config(**overrides):
    """Qwen2Config of the 0.5B shape; keyword overrides (layers, vocab, ...)."""
    from transformers import Qwen2Config

    kw = dict(QWEN2_05B)
    kw.update(overrides)
    return Qwen2Config(**kw)


def random_qwen2(config, seed: int = 0, device="cuda", dtype=torch.float16):
    """Random-init model: HF's own initialiser (N(0, initializer_range) weights)
    run on the device after ``torch.manual_seed(seed)``, then cast to ``dtype``."""
    from transformers import Qwen2ForCausalLM

    config._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen2ForCausalLM(config)
    return model.to(dtype).eval()


class FusedQwen2Body:
    """The Qwen2 decoder stack of ``model`` with its element-wise work in CUDA
    kernels of this package: ``inference::rms_norm`` for the first input norm,
    ``inference::add_rms_norm`` for every residual add and the norm after it
    (post-attention norm, next layer's input norm, final norm),
    ``inference::silu_and_mul`` for SiLU(gate) * up after ONE projection GEMM
    over the concatenated gate and up weights, and a rotary table indexed by
    position instead of recomputing cos / sin per pass. The attention modules
    (``TritonQwen2Attention``) and the projections are the model's own.

    It computes what HF's ``Qwen2Model.forward`` computes (same operations and
    fp16 roundings; the sum of squares of RMSNorm and the gate / up GEMM may
    accumulate in another order) in about 10 launches per layer instead of
    about 27.
    """

    def __init__(self, model, max_positions: int):
        from .attn import core  # noqa: F401  (loads the torch ops)

        m = model.model
        self.model = model
        self.embed = m.embed_tokens
        self.layers = list(m.layers)
        self.eps = float(model.config.rms_norm_eps)
        self.in_w = [layer.input_layernorm.weight for layer in self.layers]
        self.post_w = [layer.post_attention_layernorm.weight for layer in self.layers]
        self.next_w = self.in_w[1:] + [m.norm.weight]
        with torch.no_grad():
            self.gate_up = [torch.cat([layer.mlp.gate_proj.weight, layer.mlp.up_proj.weight])
                            for layer in self.layers]
            dev = self.embed.weight.device
            pos = torch.arange(max_positions, device=dev).view(1, -1)
            probe = torch.zeros(1, 1, dtype=self.embed.weight.dtype, device=dev)
            cos, sin = m.rotary_emb(probe, pos)
        self.cos, self.sin = cos[0].contiguous(), sin[0].contiguous()  # (positions, head_dim)
        for layer in self.layers:
            if layer.mlp.gate_proj.bias is not None or layer.mlp.up_proj.bias is not None:
                raise ValueError("Qwen2 MLP projections carry no bias")

    def __call__(self, input_ids, position_ids, kv, metadata):
        ops = torch.ops.inference
        h = self.embed(input_ids)
        pos = position_ids.view(-1)
        cos = self.cos.index_select(0, pos).unsqueeze(0)
        sin = self.sin.index_select(0, pos).unsqueeze(0)
        x = ops.rms_norm(h, self.in_w[0], self.eps)
        for i, layer in enumerate(self.layers):
            a, _ = layer.self_attn(x, (cos, sin), kv_manager=kv, metadata=metadata)
            x = ops.add_rms_norm(h, a, self.post_w[i], self.eps)
            y = ops.silu_and_mul(torch.nn.functional.linear(x, self.gate_up[i]))
            x = ops.add_rms_norm(h, layer.mlp.down_proj(y), self.next_w[i], self.eps)
        return x


@dataclass
class PrefillResult:
    first_tokens: list          # greedy token after each prompt
    last_logits: torch.Tensor   # (n_seq, vocab) logits at each prompt's last token
    forward_passes: int


class PagedRunner:
    """Slots, pages and forward passes of one model replica on one GPU.

    ``max_cache_len`` sizes the page pool (pages of 16 tokens; page 0 and slot 0
    are padding). Pages are handed out from a seeded random permutation, so a
    sequence's pages are scattered over the pool as in a long-running server.
    """

    def __init__(self, model, max_cache_len: int, n_slots: int, page_seed: int = 0,
                 token_budget: int = 2048, fused_body: bool = True):
        from .attn.core import use_cuda_attention
        from .kv_cache.storage import KVStorage

        self.model = model
        use_cuda_attention(model)
        self.device = next(model.parameters()).device
        self.dtype = next(model.parameters()).dtype
        self.kv = KVStorage(model.config, max_cache_len, PAGE_SIZE, n_slots, self.device,
                            self.dtype)
        g = torch.Generator().manual_seed(page_seed)
        self.free_pages = (torch.randperm(self.kv.n_pages - 1, generator=g) + 1).tolist()
        self.token_budget = token_budget
        self.host_lens = [0] * n_slots  # host mirror of kv.lens
        # fused_body: the CUDA element-wise kernels around the attention
        # (FusedQwen2Body); False runs HF's Qwen2Model modules as they are
        self.body = FusedQwen2Body(model, max_cache_len) if fused_body else None

    # ---- slots -------------------------------------------------------------
    def admit(self, slot: int, capacity_tokens: int) -> None:
        """Give ``slot`` pages for ``capacity_tokens`` tokens and an empty history."""
        if not 1 <= slot < self.kv.n_slots:
            raise ValueError(f"slot {slot} out of range (slot 0 is padding)")
        n = math.ceil(capacity_tokens / PAGE_SIZE)
        if n > len(self.free_pages):
            raise RuntimeError(f"page pool exhausted: need {n}, {len(self.free_pages)} free")
        pages, self.free_pages = self.free_pages[:n], self.free_pages[n:]
        self.kv.block_table[slot].zero_()
        self.kv.block_table[slot, :n] = torch.tensor(pages, dtype=torch.long)
        self.kv.lens[slot] = 0
        self.host_lens[slot] = 0

    def release(self, slot: int) -> None:
        """Return ``slot``'s pages to the pool and clear its history."""
        n = int((self.kv.block_table[slot] != 0).sum())
        pages = self.kv.block_table[slot, :n].tolist()
        self.free_pages.extend(int(p) for p in pages)
        self.kv.block_table[slot].zero_()
        self.kv.lens[slot] = 0
        self.host_lens[slot] = 0

    # ---- forward -----------------------------------------------------------
    def _hidden(self, input_ids, position_ids, metadata):
        # the attention lengths of this pass, once for all layers
        lens = self.kv.lens[metadata.slot_ids]
        metadata.attn_lens = lens + 1 if metadata.full_decode else lens
        if self.body is not None:
            return self.body(input_ids, position_ids, self.kv, metadata)
        out = self.model.model(input_ids=input_ids, position_ids=position_ids,
                               attention_mask={"full_attention": None}, kv_manager=self.kv,
                               metadata=metadata, use_cache=False)
        return out.last_hidden_state

    def mixed_metadata(self, slots, chunks):
        """AttentionMetadata of one mixed pass: sequence i appends ``chunks[i]``
        tokens to slot ``slots[i]`` at positions host_lens[slot] onward."""
        from .attn.metadata import AttentionMetadata

        T = sum(chunks)
        md = AttentionMetadata(token_count=T, full_decode=False, device=self.device)
        md.prepare_full_graph(len(slots))
        md.write_slot_ids(slots)
        cu = [0]
        pages, offsets, positions = [], [], []
        bt = self.kv.block_table
        rows = bt[torch.tensor(slots)].cpu()
        for i, (s, c) in enumerate(zip(slots, chunks)):
            start = self.host_lens[s]
            pos = list(range(start, start + c))
            positions += pos
            pages += [int(rows[i, p // PAGE_SIZE]) for p in pos]
            offsets += [p % PAGE_SIZE for p in pos]
            cu.append(cu[-1] + c)
        md.write_cu_seqlens(cu)
        md.write_pages(pages)
        md.write_offsets(offsets)
        return md, positions, cu

    def mixed_step(self, slots, token_chunks) -> list:
        """One mixed pass: sequence i appends ``token_chunks[i]`` (a decode row is
        a chunk of one token) to slot ``slots[i]``; returns the greedy token after
        each chunk's last row."""
        chunks = [len(c) for c in token_chunks]
        with torch.inference_mode():
            md, positions, cu = self.mixed_metadata(slots, chunks)
            ids = torch.tensor([[t for c in token_chunks for t in c]], dtype=torch.long,
                               device=self.device)
            pos = torch.tensor([positions], dtype=torch.long, device=self.device)
            hidden = self._hidden(ids, pos, md)
            self.kv.mixed_advance(torch.tensor(slots, dtype=torch.long, device=self.device),
                                  torch.tensor(chunks, dtype=torch.long, device=self.device))
            rows = torch.tensor([c - 1 for c in cu[1:]], device=self.device)
            tokens = self.model.lm_head(hidden[0, rows]).argmax(-1).tolist()
        for s, c in zip(slots, chunks):
            self.host_lens[s] += c
        return tokens

    def prefill(self, slots, prompts) -> PrefillResult:
        """Write every prompt into its slot through mixed passes of at most
        ``token_budget`` tokens (a long prompt spans several passes, continuing
        from its slot's length); returns the greedy token after each prompt."""
        remaining = [list(p) for p in prompts]
        done_logits = [None] * len(slots)
        passes = 0
        with torch.inference_mode():
            while any(remaining):
                budget = self.token_budget
                sel, chunks, toks = [], [], []
                for i, r in enumerate(remaining):
                    if r and budget > 0:
                        c = min(len(r), budget)
                        sel.append(i)
                        chunks.append(c)
                        toks += r[:c]
                        budget -= c
                batch_slots = [slots[i] for i in sel]
                md, positions, cu = self.mixed_metadata(batch_slots, chunks)
                ids = torch.tensor([toks], dtype=torch.long, device=self.device)
                pos = torch.tensor([positions], dtype=torch.long, device=self.device)
                hidden = self._hidden(ids, pos, md)
                slot_t = torch.tensor(batch_slots, dtype=torch.long, device=self.device)
                len_t = torch.tensor(chunks, dtype=torch.long, device=self.device)
                self.kv.mixed_advance(slot_t, len_t)
                last_rows = []
                for j, i in enumerate(sel):
                    self.host_lens[slots[i]] += chunks[j]
                    remaining[i] = remaining[i][chunks[j]:]
                    if not remaining[i]:
                        last_rows.append((i, cu[j + 1] - 1))
                if last_rows:
                    rows = torch.tensor([r for _, r in last_rows], device=self.device)
                    logits = self.model.lm_head(hidden[0, rows]).float()
                    for (i, _), lg in zip(last_rows, logits):
                        done_logits[i] = lg
                passes += 1
        last = torch.stack(done_logits)
        return PrefillResult(first_tokens=last.argmax(-1).tolist(), last_logits=last,
                             forward_passes=passes)

    def decode_graph(self, slots, first_tokens, capture: bool = True) -> "DecodeGraph":
        return DecodeGraph(self, slots, first_tokens, capture)


class DecodeGraph:
    """One greedy decode step for a fixed batch of slots: the tokens of the
    previous step in, the next tokens out (``tokens``, device (B,)), every slot
    one position longer. Captured in a CUDA graph unless ``capture`` is False."""

    def __init__(self, runner: PagedRunner, slots, first_tokens, capture: bool = True):
        from .attn.metadata import AttentionMetadata

        self.runner = runner
        self.slots = list(slots)
        B = len(self.slots)
        dev = runner.device
        self.md = AttentionMetadata(token_count=B, full_decode=True, device=dev)
        self.md.prepare_full_graph(B)
        self.md.write_slot_ids(self.slots)
        self.tokens = torch.tensor(first_tokens, dtype=torch.long, device=dev)
        self.logits = None
        self.graph = None
        if capture:
            # the tokens this warm-up produces are discarded: undo its writes
            saved_lens = runner.kv.lens.clone()
            saved_tokens = self.tokens.clone()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side), torch.inference_mode():
                self._step()
            torch.cuda.current_stream().wait_stream(side)
            runner.kv.lens.copy_(saved_lens)
            self.tokens.copy_(saved_tokens)
            self.graph = torch.cuda.CUDAGraph()
            with torch.inference_mode(), torch.cuda.graph(self.graph):
                self._step()
            runner.kv.lens.copy_(saved_lens)
            self.tokens.copy_(saved_tokens)

    def _step(self):
        kv = self.runner.kv
        ids = self.tokens.view(1, -1)
        pos = kv.lens[self.md.slot_ids].view(1, -1)
        hidden = self.runner._hidden(ids, pos, self.md)
        self.logits = self.runner.model.lm_head(hidden[0])
        self.tokens.copy_(self.logits.argmax(-1))
        kv.decode_advance(self.md.slot_ids)

    def step(self) -> torch.Tensor:
        if self.graph is not None:
            self.graph.replay()
        else:
            with torch.inference_mode():
                self._step()
        for s in self.slots:
            self.runner.host_lens[s] += 1
        return self.tokens
