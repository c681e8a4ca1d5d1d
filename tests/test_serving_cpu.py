"""The continuous-batching loop (serving.serve) on a fake engine and a fake
clock: token budget per step, chunked prefill, decode-only steps, admission
by planned arrival, completion after max_new tokens, and the benchmark
metrics (5 % trim, tok/s over first planned .. last end)."""
import math

import pytest

from custom_inference_engine_b200 import serving as SV


class FakeClock:
    def __init__(self):
        self.t = 0.0

    def __call__(self):
        return self.t

    def sleep(self, dt):
        self.t += dt


class FakeEngine:
    """Next token = (last input token + 1) % 1000; every step costs 1 ms."""

    def __init__(self, clock, n_pages=10_000):
        self.clock = clock
        self.free_pages = list(range(1, n_pages))
        self.owned = {}
        self.steps = []

    def admit(self, slot, tokens):
        n = math.ceil(tokens / 16)
        self.owned[slot], self.free_pages = self.free_pages[:n], self.free_pages[n:]

    def release(self, slot):
        self.free_pages += self.owned.pop(slot)

    def mixed_step(self, slots, chunks):
        assert len(set(slots)) == len(slots)
        self.steps.append(("mixed", list(slots), [len(c) for c in chunks]))
        self.clock.t += 1e-3
        return [(c[-1] + 1) % 1000 for c in chunks]

    def decode_step(self, slots, tokens):
        self.steps.append(("decode", list(slots), [1] * len(slots)))
        self.clock.t += 1e-3
        return [(t + 1) % 1000 for t in tokens]


def _run(reqs, n_slots=5, budget=64, n_pages=10_000):
    clock = FakeClock()
    eng = FakeEngine(clock, n_pages)
    out, steps = SV.serve(eng, reqs, n_slots=n_slots, token_budget=budget, clock=clock,
                          sleep=clock.sleep)
    return out, steps, eng


def test_every_request_completes_with_its_tokens():
    reqs = SV.poisson_requests(12, rate=200.0, seed=1, vocab=1000, median_prompt=40,
                               max_prompt=150, min_new=3, max_new=9)
    out, steps, eng = _run(reqs)
    for r in out:
        assert len(r.new_tokens) == r.max_new
        # the fake model continues the prompt: first token = last prompt id + 1
        want = [(r.prompt[-1] + 1 + i) % 1000 for i in range(r.max_new)]
        assert r.new_tokens == want
        assert r.planned <= r.arrival <= r.t_first <= r.t_end
    assert not eng.owned and len(eng.free_pages) == 9_999  # every page came back
    assert steps["mixed"] > 0 and steps["decode"] > 0


def test_budget_and_step_kinds():
    reqs = SV.poisson_requests(10, rate=1000.0, seed=2, vocab=1000, median_prompt=100,
                               max_prompt=300, min_new=2, max_new=5)
    out, steps, eng = _run(reqs, n_slots=4, budget=48)
    for kind, slots, chunks in eng.steps:
        assert sum(chunks) <= 48
        assert len(slots) <= 3               # slot 0 is padding
        if kind == "decode":
            assert all(c == 1 for c in chunks)
    # prompts longer than the budget are read over several mixed passes
    assert any(max(ch) == 48 for k, _, ch in eng.steps if k == "mixed")


def test_admission_waits_for_arrival_and_pages():
    reqs = [SV.Request(0, [1] * 20, 4, planned=0.0), SV.Request(1, [2] * 20, 4, planned=5.0)]
    out, _, eng = _run(reqs)
    assert out[1].arrival >= 5.0                      # not before its planned time
    assert out[0].t_end < 5.0                         # the first finished long before
    # a pool too small for both at once serialises them
    reqs = [SV.Request(0, [1] * 40, 8, planned=0.0), SV.Request(1, [2] * 40, 8, planned=0.0)]
    out, _, eng = _run(reqs, n_pages=5)
    assert out[1].arrival >= out[0].t_end


def test_summarize_trims_and_defines_rates():
    reqs = []
    for i in range(20):
        r = SV.Request(i, [0], 5, planned=float(i))
        r.t_first, r.t_end = i + 0.5, i + 1.0
        r.new_tokens = [1] * 5
        reqs.append(r)
    m = SV.summarize(reqs, trim=0.05)                 # drops one request at each end
    assert m["n_measured"] == 18
    assert m["duration_s"] == pytest.approx(19.0 - 1.0)  # planned 1 .. end of #18 (19)
    assert m["tok_s"] == pytest.approx(18 * 5 / 18.0)
    assert m["ttft_ms"]["mean"] == pytest.approx(500.0)
    assert m["tpot_ms"]["mean"] == pytest.approx(125.0)


def test_request_larger_than_the_pool_is_rejected():
    reqs = [SV.Request(0, [1] * 400, 8, planned=0.0)]
    with pytest.raises(ValueError):
        _run(reqs, n_pages=5)
