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

import numpy as np
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
                 token_budget: int = 2048, fused_body: bool = True, mixed_graphs: bool = True,
                 block_table_dtype=torch.int64, fused_lm_head: bool = True,
                 fused_mixed_attention: bool = True):
        from .attn.core import use_cuda_attention
        from .kv_cache.storage import KVStorage

        self.model = model
        use_cuda_attention(model)
        # fused_mixed_attention: the metadata of this runner's mixed passes asks
        # for RoPE, K/V write and attention as one call per layer (no piecewise
        # splitter runs over this runner)
        self.fused_mixed_attention = fused_mixed_attention
        self.device = next(model.parameters()).device
        self.dtype = next(model.parameters()).dtype
        self.kv = KVStorage(model.config, max_cache_len, PAGE_SIZE, n_slots, self.device,
                            self.dtype, block_table_dtype=block_table_dtype)
        g = torch.Generator().manual_seed(page_seed)
        self.free_pages = (torch.randperm(self.kv.n_pages - 1, generator=g) + 1).tolist()
        self.token_budget = token_budget
        self.host_lens = [0] * n_slots  # host mirror of kv.lens
        self.host_pages = {}            # slot -> its pages (host mirror of the block-table row)
        # fused_body: the CUDA element-wise kernels around the attention
        # (FusedQwen2Body); False runs HF's Qwen2Model modules as they are
        self.body = FusedQwen2Body(model, max_cache_len) if fused_body else None
        # mixed_graphs: mixed passes replay a CUDA graph per token bucket (the
        # reference's FullMixedModule); False runs them eagerly
        self.use_mixed_graphs = mixed_graphs and self.device.type == "cuda"
        # fused_lm_head: decode steps take the greedy token from one pass over the
        # lm_head weight (inference::lm_head_argmax) and keep no logits; False
        # runs the lm_head GEMM, keeps the logits and takes their argmax
        self.fused_lm_head = fused_lm_head
        self.mixed_buckets = sorted({b for b in MIXED_TOKEN_BUCKETS if b < token_budget}
                                    | {token_budget})
        self._mixed_graphs = {}
        self._graph_pool = None

    # ---- slots -------------------------------------------------------------
    def admit(self, slot: int, capacity_tokens: int) -> None:
        """Give ``slot`` pages for ``capacity_tokens`` tokens and an empty history."""
        if not 1 <= slot < self.kv.n_slots:
            raise ValueError(f"slot {slot} out of range (slot 0 is padding)")
        n = math.ceil(capacity_tokens / PAGE_SIZE)
        if n > len(self.free_pages):
            raise RuntimeError(f"page pool exhausted: need {n}, {len(self.free_pages)} free")
        pages, self.free_pages = self.free_pages[:n], self.free_pages[n:]
        self.host_pages[slot] = np.asarray(pages, dtype=np.int64)
        self.kv.block_table[slot].zero_()
        self.kv.block_table[slot, :n] = torch.from_numpy(self.host_pages[slot])
        self.kv.lens[slot] = 0
        self.host_lens[slot] = 0

    def release(self, slot: int) -> None:
        """Return ``slot``'s pages to the pool and clear its history."""
        self.free_pages.extend(int(p) for p in self.host_pages.pop(slot, ()))
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

    def placement(self, slots, chunks):
        """Positions, pages and in-page offsets (numpy, one per token) and
        cu_seqlens of a mixed pass in which sequence i appends ``chunks[i]``
        tokens to slot ``slots[i]`` at positions host_lens[slot] onward."""
        T = int(sum(chunks))
        ch = np.asarray(chunks, dtype=np.int64)
        cu = np.concatenate([[0], np.cumsum(ch)])
        seq = np.repeat(np.arange(len(slots)), ch)          # sequence of every token
        starts = np.asarray([self.host_lens[s] for s in slots], dtype=np.int64)
        positions = starts[seq] + np.arange(T, dtype=np.int64) - cu[seq]
        pages = np.empty(T, dtype=np.int64)
        for i, s in enumerate(slots):
            pages[cu[i]:cu[i + 1]] = self.host_pages[s][positions[cu[i]:cu[i + 1]] // PAGE_SIZE]
        offsets = positions % PAGE_SIZE
        return positions, pages, offsets, cu

    def mixed_metadata(self, slots, chunks):
        """AttentionMetadata of one mixed pass (see ``placement``)."""
        from .attn.metadata import AttentionMetadata

        positions, pages, offsets, cu = self.placement(slots, chunks)
        md = AttentionMetadata(token_count=int(cu[-1]), full_decode=False, device=self.device)
        md.fuse_mixed_attention = self.fused_mixed_attention
        md.prepare_full_graph(len(slots))
        md.write_slot_ids(slots)
        md.write_cu_seqlens(cu)
        md.write_pages(pages)
        md.write_offsets(offsets)
        return md, positions, cu.tolist()

    def mixed_graph(self, tokens: int) -> "MixedGraph":
        """The captured mixed pass of the smallest token bucket >= ``tokens``."""
        b = next(x for x in self.mixed_buckets if x >= tokens)
        if b not in self._mixed_graphs:
            if self._graph_pool is None:
                self._graph_pool = torch.cuda.graph_pool_handle()
            self._mixed_graphs[b] = MixedGraph(self, b, self.kv.n_slots - 1, self._graph_pool)
        return self._mixed_graphs[b]

    def capture_mixed_graphs(self) -> None:
        """Capture every token bucket's mixed pass now (capture takes tens of
        milliseconds; do it before anything is timed)."""
        if self.use_mixed_graphs:
            for b in self.mixed_buckets:
                self.mixed_graph(b)

    def mixed_logits(self, slots, token_chunks):
        """One mixed pass (sequence i appends ``token_chunks[i]`` to slot
        ``slots[i]``); returns the logits at each chunk's last row (n, vocab),
        from a captured graph when ``mixed_graphs`` is on."""
        chunks = [len(c) for c in token_chunks]
        flat = [t for c in token_chunks for t in c]
        with torch.inference_mode():
            if self.use_mixed_graphs and len(slots) <= self.kv.n_slots - 1 and \
                    sum(chunks) <= self.mixed_buckets[-1]:
                logits = self.mixed_graph(sum(chunks)).run(slots, chunks, flat)
            else:
                md, positions, cu = self.mixed_metadata(slots, chunks)
                ids = torch.tensor([flat], dtype=torch.long, device=self.device)
                pos = torch.from_numpy(positions).view(1, -1).to(self.device)
                hidden = self._hidden(ids, pos, md)
                self.kv.mixed_advance(torch.tensor(slots, dtype=torch.long, device=self.device),
                                      torch.tensor(chunks, dtype=torch.long, device=self.device))
                rows = torch.tensor([c - 1 for c in cu[1:]], device=self.device)
                logits = self.model.lm_head(hidden[0, rows])
        for s, c in zip(slots, chunks):
            self.host_lens[s] += c
        return logits

    def mixed_step(self, slots, token_chunks) -> list:
        """One mixed pass: sequence i appends ``token_chunks[i]`` (a decode row is
        a chunk of one token) to slot ``slots[i]``; returns the greedy token after
        each chunk's last row."""
        return self.mixed_logits(slots, token_chunks).argmax(-1).tolist()

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
                sel, chunks = [], []
                for i, r in enumerate(remaining):
                    if r and budget > 0:
                        c = min(len(r), budget)
                        sel.append(i)
                        chunks.append(c)
                        budget -= c
                batch_slots = [slots[i] for i in sel]
                logits = self.mixed_logits(batch_slots, [remaining[i][:c] for i, c in zip(sel, chunks)])
                for j, i in enumerate(sel):
                    remaining[i] = remaining[i][chunks[j]:]
                    if not remaining[i]:
                        done_logits[i] = logits[j].float()
                passes += 1
        last = torch.stack(done_logits)
        return PrefillResult(first_tokens=last.argmax(-1).tolist(), last_logits=last,
                             forward_passes=passes)

    def decode_graph(self, slots, first_tokens, capture: bool = True) -> "DecodeGraph":
        return DecodeGraph(self, slots, first_tokens, capture)


class DecodeGraph:
    """One greedy decode step for a fixed batch of slots: the tokens of the
    previous step in, the next tokens out (``tokens``, device (B,)), every slot
    one position longer. Captured in a CUDA graph unless ``capture`` is False.
    ``logits`` holds the step's logits only when the runner's ``fused_lm_head``
    is off."""

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
        lm_head = self.runner.model.lm_head
        if self.runner.fused_lm_head and lm_head.bias is None:
            self.tokens.copy_(torch.ops.inference.lm_head_argmax(hidden[0], lm_head.weight))
        else:
            self.logits = lm_head(hidden[0])
            self.tokens.copy_(torch.ops.inference.argmax_rows(self.logits))
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


MIXED_TOKEN_BUCKETS = (64, 128, 256, 512, 1024, 2048)


class MixedGraph:
    """One mixed pass of up to ``max_seqs`` sequences and ``tokens`` tokens,
    captured in a CUDA graph (the reference's FullMixedModule): the metadata,
    token ids, positions, last-row indices and the length advance live in
    static buffers written before each replay. Tokens past the pass's own are
    padding the reference's way: page 0, offset 0, position 0, outside every
    sequence (cu_seqlens repeats its last value); absent sequences are slot 0
    with no tokens. ``run`` returns the logits at each sequence's last row."""

    def __init__(self, runner, tokens: int, max_seqs: int, pool=None):
        from .attn.metadata import AttentionMetadata

        self.runner = runner
        self.tokens = tokens
        self.max_seqs = max_seqs
        dev = runner.device
        self.md = AttentionMetadata(token_count=tokens, full_decode=False, device=dev)
        self.md.fuse_mixed_attention = runner.fused_mixed_attention
        self.md.prepare_full_graph(max_seqs)
        z = lambda n: torch.zeros(n, dtype=torch.long, device=dev)
        self.ids, self.pos = z((1, tokens)), z((1, tokens))
        self.last_rows, self.adv_slots, self.adv_lens = z(max_seqs), z(max_seqs), z(max_seqs)
        self.logits = None
        saved = runner.kv.lens.clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.inference_mode():
            self._pass()
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.inference_mode(), torch.cuda.graph(self.graph, pool=pool):
            self._pass()
        runner.kv.lens.copy_(saved)

    def _pass(self):
        r = self.runner
        hidden = r._hidden(self.ids, self.pos, self.md)
        self.logits = r.model.lm_head(hidden[0, self.last_rows])
        r.kv.mixed_advance(self.adv_slots, self.adv_lens)

    def run(self, slots, chunks, flat_tokens):
        n, T = len(slots), int(sum(chunks))
        positions, pages, offsets, cu = self.runner.placement(slots, chunks)
        md = self.md
        md.write_slot_ids(slots)
        md.write_cu_seqlens(cu)
        md.write_pages(pages)
        md.write_offsets(offsets)
        ids = np.zeros(self.tokens, dtype=np.int64)
        ids[:T] = flat_tokens
        pos = np.zeros(self.tokens, dtype=np.int64)
        pos[:T] = positions
        small = np.zeros((3, self.max_seqs), dtype=np.int64)
        small[0, :n] = cu[1:] - 1
        small[1, :n] = slots
        small[2, :n] = chunks
        self.ids.copy_(torch.from_numpy(ids).view(1, -1))
        self.pos.copy_(torch.from_numpy(pos).view(1, -1))
        small_d = torch.from_numpy(small).to(self.ids.device)
        self.last_rows.copy_(small_d[0])
        self.adv_slots.copy_(small_d[1])
        self.adv_lens.copy_(small_d[2])
        self.graph.replay()
        return self.logits[:n]
