"""The reference engine's CUDA-graph modules run unchanged over this package's ops.

``DecodeModule`` (scheduler/decode_module.py:8-48), ``FullMixedModule``
(scheduler/mixed_module.py:180-214) and ``PiecewiseMixedModule``
(scheduler/mixed_module.py:216-249, with the splitter and backend of
piecewise/utils.py and piecewise/backend.py) are the reference's own code, from
the unmodified copy in baseline/_ref. They are built over a seeded random-init
2-layer Qwen2 of the 0.5B shape whose attention modules are this package's
``TritonQwen2Attention`` and whose KV cache is this package's ``KVStorage``:
each one compiles its forward with ``torch.compile(fullgraph=True)`` (Dynamo
raises on a graph break) and captures CUDA graphs in the reference's way
(DecodeModule and FullMixedModule: the whole forward; PiecewiseMixedModule:
the pieces between the attention groups, with a dynamic batch).

Requests are served through them the way the reference scheduler uses them: a
prefill pass, a mixed pass that carries two decode rows and a new prompt, then
greedy decode steps (DecodeModule). The greedy tokens must equal those of this
package's ``PagedRunner`` (HF decoder body, eager passes) on the same model.
Inductor is asked to round fp16 intermediates as eager PyTorch does
(``emulate_precision_casts``), so the compiled decoder body computes what the
eager one computes and the comparison is about the attention path.
"""
import math

import numpy as np
import pytest
import torch

from custom_inference_engine_b200 import model_runner as MR

pytestmark = pytest.mark.gpu

N_SLOTS = 5          # slot 0 is padding
BATCH = 4            # decode / full-mixed batch size
TOKENS = 256         # token count of the mixed modules
N_DECODE = 8
PROMPT_LENS = {"A": 5, "B": 40, "C": 130}


@pytest.fixture(scope="module")
def setup(reference_modules, cuda_device):
    import torch._inductor.config as inductor_config

    saved = inductor_config.emulate_precision_casts
    inductor_config.emulate_precision_casts = True
    cfg = MR.qwen2_config(num_hidden_layers=2)
    model = MR.random_qwen2(cfg, seed=0, device=cuda_device)
    rng = np.random.default_rng(11)
    prompts = {k: rng.integers(0, cfg.vocab_size, size=n).tolist()
               for k, n in PROMPT_LENS.items()}
    yield reference_modules, model, prompts
    inductor_config.emulate_precision_casts = saved


def _give_pages(kv, slots, lens, seed):
    """Scattered pages for each slot, as the reference scheduler hands them out
    (page 0 is never given to a real slot)."""
    g = torch.Generator().manual_seed(seed)
    free = (torch.randperm(kv.n_pages - 1, generator=g) + 1).tolist()
    for s, n in zip(slots, lens):
        k = math.ceil(n / kv.page_size)
        kv.block_table[s].zero_()
        kv.block_table[s, :k] = torch.tensor(free[:k], device=kv.block_table.device)
        free = free[k:]
        kv.lens[s] = 0


def _serve(mixed, decode, kv, prompts):
    """Prefill A, B; one mixed pass with A's and B's decode rows and prompt C;
    then greedy decode steps for all three."""
    total = {s: len(p) + N_DECODE + 4 for s, p in zip((1, 2, 3), prompts.values())}
    kv.reset([1, 2, 3, 4])
    _give_pages(kv, list(total), list(total.values()), seed=5)
    out = {1: [], 2: [], 3: []}
    t = mixed.forward([prompts["A"], prompts["B"]], [1, 2])
    out[1].append(t[0])
    out[2].append(t[1])
    t = mixed.forward([[out[1][-1]], [out[2][-1]], prompts["C"]], [1, 2, 3])
    for s, tok in zip((1, 2, 3), t):
        out[s].append(tok)
    for _ in range(N_DECODE):
        for s, tok in zip((1, 2, 3), decode.forward([1, 2, 3])):
            out[s].append(tok)
    return out


def _paged_runner(model, prompts):
    runner = MR.PagedRunner(model, max_cache_len=4096, n_slots=N_SLOTS, token_budget=TOKENS,
                            fused_body=False, mixed_graphs=False)
    for s, p in zip((1, 2, 3), prompts.values()):
        runner.admit(s, len(p) + N_DECODE + 4)
    out = {1: [], 2: [], 3: []}
    t = runner.mixed_step([1, 2], [prompts["A"], prompts["B"]])
    out[1].append(t[0])
    out[2].append(t[1])
    t = runner.mixed_step([1, 2, 3], [[out[1][-1]], [out[2][-1]], prompts["C"]])
    for s, tok in zip((1, 2, 3), t):
        out[s].append(tok)
    graph = runner.decode_graph([1, 2, 3], [out[s][-1] for s in (1, 2, 3)], capture=False)
    for _ in range(N_DECODE):
        for s, tok in zip((1, 2, 3), graph.step().tolist()):
            out[s].append(tok)
    return out


def test_reference_graph_modules_serve_the_runners_tokens(setup, cuda_device):
    from kv_cache.storage import KVStorage   # this package's, through the aliases

    R, model, prompts = setup
    from attn.core import use_triton_attention

    use_triton_attention(model)
    want = _paged_runner(model, prompts)

    kv = KVStorage(model.config, max_cache_len=4096, page_size=16, n_slots=N_SLOTS,
                   device=cuda_device, dtype=torch.float16)
    pool = torch.cuda.graph_pool_handle()
    decode = R.decode_module.DecodeModule(model, kv, BATCH, pool)
    full = R.mixed_module.FullMixedModule(model, kv, BATCH, TOKENS, pool)
    buffer = torch.zeros((1, TOKENS, kv.num_q_heads, kv.head_dim), dtype=model.dtype,
                         device=cuda_device)
    piecewise = R.mixed_module.PiecewiseMixedModule(model, kv, TOKENS, buffer, pool)

    got_full = _serve(full, decode, kv, prompts)
    got_piecewise = _serve(piecewise, decode, kv, prompts)
    assert got_full == want, (got_full, want)
    assert got_piecewise == want, (got_piecewise, want)

    from custom_inference_engine_b200 import native
    assert native.device_errors(cuda_device.index or 0) == 0
