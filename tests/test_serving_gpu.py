"""Requests served through the continuous-batching loop (Poisson arrivals,
chunked prefill mixed with decode rows, bucketed CUDA-graph decode steps) on
a small random-init Qwen2 of the 0.5B head layout produce the greedy tokens of
the same model with Hugging Face's own attention, each prompt alone."""
import pytest
import torch

from custom_inference_engine_b200 import model_runner as MR
from custom_inference_engine_b200 import serving as SV

pytestmark = pytest.mark.gpu


def test_served_tokens_match_hf_greedy(cuda_device):
    cfg = MR.qwen2_config(num_hidden_layers=2, vocab_size=4096, intermediate_size=2048)
    model = MR.random_qwen2(cfg, seed=0, device=cuda_device)
    reqs = SV.poisson_requests(6, rate=400.0, seed=5, vocab=4096, median_prompt=60,
                               max_prompt=200, min_new=4, max_new=10)
    n_slots = 5                                   # 4 real slots: admission has to wait
    runner = MR.PagedRunner(model, max_cache_len=4096, n_slots=n_slots, token_budget=64)
    engine = SV.RunnerEngine(runner, n_slots)
    out, steps = SV.serve(engine, reqs, n_slots=n_slots, token_budget=64)
    assert steps["mixed"] > 0 and steps["decode"] > 0
    with torch.inference_mode():
        for r in out:
            seq = list(r.prompt)
            for _ in range(r.max_new):
                ids = torch.tensor([seq], device=cuda_device)
                seq.append(int(model(input_ids=ids).logits[0, -1].float().argmax()))
            assert r.new_tokens == seq[len(r.prompt):], r.rid
    m = SV.summarize(out, trim=0.0)
    assert m["new_tokens"] == sum(r.max_new for r in reqs) and m["tok_s"] > 0
