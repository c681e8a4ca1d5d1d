"""Continuous-batching serving loop over the paged runner: Poisson arrivals,
chunked prefill mixed with decode rows, CUDA-graphed decode steps.

This is the request path of the reference's serving benchmark reduced to what
measures tokens/s on the attention ops (the reference's Scheduler,
scheduler/scheduler.py:307-640, and benchmark/serve.py; metric definitions of
benchmark/metrics.py:54-75, 159-200):

* every step gives each decoding request one token of the ``token_budget``
  and fills the rest with prefill chunks of the requests still reading their
  prompt, oldest first (scheduler.py:568-605); requests whose planned arrival
  time has passed are admitted into free slots with what budget is left
  (scheduler.py:372-433);
* a step with prefill work is ONE mixed pass through
  ``inference::gqa_mixed_attention`` (decode rows are chunks of one token),
  replayed from the CUDA graph of the smallest token bucket that holds it; a
  step with only decode rows replays the CUDA graph of the smallest batch
  bucket that holds them (rows beyond the batch use the padding slot 0);
* a request finishes after ``max_new`` tokens (the end-of-sequence id of the
  benchmark is one argmax never produces), and its slot and pages are freed.

Differences from the reference, on purpose: pages for a request's prompt and
all its new tokens are reserved at admission (a request waits until they are
free), so there is no preemption; requests are timed on one thread against a
wall clock instead of through futures from a client thread.
"""
from __future__ import annotations

import bisect
import math
import time
from collections import deque
from dataclasses import dataclass, field

import numpy as np

DECODE_BUCKETS = (1, 2, 4, 8, 16, 24, 32)


@dataclass
class Request:
    rid: int
    prompt: list
    max_new: int
    planned: float                    # planned arrival, seconds after the start
    slot: int = 0
    pos: int = 0                      # prompt tokens already in the KV pages
    arrival: float = float("nan")     # admission time
    new_tokens: list = field(default_factory=list)
    t_first: float = float("nan")
    t_end: float = float("nan")

    @property
    def prefilled(self) -> bool:
        return self.pos >= len(self.prompt)


def poisson_requests(n: int, rate: float, seed: int, vocab: int, median_prompt: float = 512.0,
                     sigma: float = 0.5, max_prompt: int = 4096, min_new: int = 64,
                     max_new: int = 512):
    """``n`` requests: exponential gaps of mean 1/rate (benchmark/workload.py:173-186),
    lognormal prompt lengths (median ``median_prompt``, capped), uniform random
    prompt ids, output lengths uniform in [min_new, max_new]."""
    rng = np.random.default_rng(seed)
    arrivals = np.cumsum(rng.exponential(1.0 / rate, size=n))
    lens = np.clip(np.round(np.exp(rng.normal(np.log(median_prompt), sigma, size=n))), 1,
                   max_prompt).astype(int)
    outs = rng.integers(min_new, max_new + 1, size=n)
    return [Request(rid=i, prompt=rng.integers(0, vocab, size=int(lens[i])).tolist(),
                    max_new=int(outs[i]), planned=float(arrivals[i])) for i in range(n)]


class DecodeBuckets:
    """One captured greedy decode step per batch bucket of ``runner``."""

    def __init__(self, runner, max_batch: int, buckets=DECODE_BUCKETS):
        from .model_runner import DecodeGraph

        self.runner = runner
        self.sizes = [b for b in buckets if b < max_batch] + [max_batch]
        self.sizes = sorted(set(self.sizes))
        self.graphs = {b: DecodeGraph(runner, [0] * b, [0] * b, capture=True)
                       for b in self.sizes}

    def step(self, slots, tokens) -> list:
        n = len(slots)
        b = self.sizes[bisect.bisect_left(self.sizes, n)]
        g = self.graphs[b]
        g.md.write_slot_ids(slots)
        g.tokens[:n].copy_(g.tokens.new_tensor(tokens))
        g.tokens[n:].zero_()
        g.graph.replay()
        out = g.tokens[:n].tolist()
        for s in slots:
            self.runner.host_lens[s] += 1
        return out


def serve(engine, requests, n_slots: int, token_budget: int, clock=time.perf_counter,
          sleep=time.sleep):
    """Runs ``requests`` (sorted by planned arrival) to completion.

    ``engine`` provides ``free_pages`` (list), ``admit(slot, tokens)``,
    ``release(slot)``, ``mixed_step(slots, token_chunks) -> next tokens`` and
    ``decode_step(slots, tokens) -> next tokens``. Returns the requests with
    their timestamps (seconds after the start) and the step counts."""
    pool = len(engine.free_pages)
    for r in requests:
        if math.ceil((len(r.prompt) + r.max_new) / 16) > pool:
            raise ValueError(f"request {r.rid} needs more pages than the pool holds ({pool})")
    pending = deque(sorted(requests, key=lambda r: r.planned))
    running = {}                 # slot -> request, in admission order
    free_slots = list(range(1, n_slots))
    steps = {"mixed": 0, "decode": 0}
    t0 = clock()
    while pending or running:
        now = clock() - t0
        decoding = [s for s, r in running.items() if r.prefilled]
        budget = token_budget - len(decoding)
        plan = []                # (slot, chunk of prompt tokens)
        for s, r in running.items():
            if r.prefilled or budget <= 0:
                continue
            c = min(budget, len(r.prompt) - r.pos)
            plan.append((s, r.prompt[r.pos:r.pos + c]))
            budget -= c
        while pending and pending[0].planned <= now and free_slots and budget > 0:
            r = pending[0]
            need = math.ceil((len(r.prompt) + r.max_new) / 16)
            if need > len(engine.free_pages):
                break
            pending.popleft()
            s = free_slots.pop(0)
            engine.admit(s, len(r.prompt) + r.max_new)
            r.slot, r.arrival = s, now
            running[s] = r
            c = min(budget, len(r.prompt))
            plan.append((s, r.prompt[:c]))
            budget -= c
        if not running:
            sleep(max(0.0, pending[0].planned - (clock() - t0)))
            continue
        if plan:
            slots = decoding + [s for s, _ in plan]
            chunks = [[running[s].new_tokens[-1]] for s in decoding] + [c for _, c in plan]
            out = engine.mixed_step(slots, chunks)
            steps["mixed"] += 1
        else:
            slots = decoding
            chunks = None
            out = engine.decode_step(slots, [running[s].new_tokens[-1] for s in slots])
            steps["decode"] += 1
        t = clock() - t0
        for i, (s, tok) in enumerate(zip(slots, out)):
            r = running[s]
            if not r.prefilled:
                r.pos += len(chunks[i])
                if not r.prefilled:
                    continue     # more prompt to read: the token is not a prediction
            r.new_tokens.append(int(tok))
            if len(r.new_tokens) == 1:
                r.t_first = t
            if len(r.new_tokens) >= r.max_new:
                r.t_end = t
                del running[s]
                engine.release(s)
                free_slots.append(s)
                free_slots.sort()
    return requests, steps


def summarize(requests, trim: float = 0.05) -> dict:
    """benchmark/metrics.py:159-200: drop ``trim`` of the requests at each end
    (by planned arrival); tok/s = new tokens / (last end - first planned);
    TTFT = first token - planned, TPOT = (end - first) / (tokens - 1)."""
    ordered = sorted(requests, key=lambda r: r.planned)
    cut = int(len(ordered) * trim)
    m = ordered[cut:len(ordered) - cut]
    start = min(r.planned for r in m)
    end = max(r.t_end for r in m)
    tokens = sum(len(r.new_tokens) for r in m)
    ttft = np.array([r.t_first - r.planned for r in m])
    tpot = np.array([(r.t_end - r.t_first) / (len(r.new_tokens) - 1) for r in m
                     if len(r.new_tokens) > 1])
    pct = lambda a, q: float(np.percentile(a, q)) if len(a) else float("nan")
    return {"n_measured": len(m), "duration_s": end - start, "tok_s": tokens / (end - start),
            "first_planned_s": start, "last_end_s": end,
            "req_s": len(m) / (end - start), "new_tokens": tokens,
            "ttft_ms": {"mean": 1e3 * float(ttft.mean()), "p50": 1e3 * pct(ttft, 50),
                        "p99": 1e3 * pct(ttft, 99)},
            "tpot_ms": {"mean": 1e3 * float(tpot.mean()) if len(tpot) else float("nan"),
                        "p50": 1e3 * pct(tpot, 50), "p99": 1e3 * pct(tpot, 99)}}


class RunnerEngine:
    """``serve``'s engine on a ``PagedRunner``: mixed passes and decode steps
    from CUDA graphs captured per token bucket and per batch bucket."""

    def __init__(self, runner, n_slots: int):
        self.runner = runner
        self.buckets = DecodeBuckets(runner, n_slots - 1)
        runner.capture_mixed_graphs()

    @property
    def free_pages(self):
        return self.runner.free_pages

    def admit(self, slot, tokens):
        self.runner.admit(slot, tokens)

    def release(self, slot):
        self.runner.release(slot)

    def mixed_step(self, slots, chunks):
        return self.runner.mixed_step(slots, chunks)

    def decode_step(self, slots, tokens):
        return self.buckets.step(slots, tokens)
