"""Greedy tokens of the reference engine, free-running, on the same GPU.

The reference engine (its own attention module, Triton kernels and KV storage,
unmodified, from baseline/_ref) and this package generate from the same seeded
random-init Qwen2 of the Qwen2.5-0.5B shape, driven by the same schedule of
mixed passes (chunked prefill with decode rows) and decode passes
(``tests/e2e_greedy.py``): 8 prompts of 1-300 tokens, 32 new tokens each, every
token fed back. The reference runs in a child process (the two register the
same op names) on the same GPU, so the decoder body, projections and lm_head
are the same cuBLAS and PyTorch calls on both sides and only the attention path
differs: its outputs agree within fp16 rounding, not bit for bit (the two
sides sum the fp32 dot products in different orders).

* 4 layers: the tokens are identical.
* 24 layers (the whole model): rounding differences pass through 24 layers,
  and a sequence may turn at a step where the reference's two best logits are
  within one fp16 ulp of each other (equal, or adjacent fp16 values). Each
  sequence must match token for token up to its first difference, which may
  only be such a tie with the same two candidates on both sides; later tokens
  of a sequence that turned follow a different history and are not compared.
  The test prints where sequences turned.
"""
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def _ulp16(x: float) -> float:
    """Spacing of fp16 values at |x| (normal range)."""
    return float(np.spacing(np.float16(abs(x))))


@pytest.mark.parametrize("layers", [4, 24])
def test_free_running_greedy_tokens_follow_the_reference_engine(layers, reference_modules,
                                                                cuda_device, tmp_path):
    import e2e_greedy
    from conftest import REFERENCE_COPY

    out = tmp_path / "reference_engine.npz"
    run = subprocess.run([sys.executable, str(HERE / "e2e_greedy.py"), "--reference-copy",
                          str(REFERENCE_COPY), "--layers", str(layers), "--out", str(out)],
                         capture_output=True, text=True, timeout=1200)
    assert run.returncode == 0, run.stderr[-4000:]
    ref = np.load(out)

    model = e2e_greedy.build_model(cuda_device, layers)
    assert e2e_greedy.weight_checksum(model) == float(ref["checksum"])
    tokens, ids, vals = e2e_greedy.generate(model, cuda_device)
    want, rids, rvals = ref["tokens"], ref["top_ids"], ref["top_vals"]
    assert tokens.shape == want.shape == (len(e2e_greedy.PROMPT_LENS), e2e_greedy.N_NEW)

    turned = []
    for s in range(tokens.shape[0]):
        diff = np.flatnonzero(tokens[s] != want[s])
        if not len(diff):
            continue
        t = int(diff[0])
        margin = float(rvals[s, t, 0] - rvals[s, t, 1])
        turned.append((s, t, margin, float(vals[s, t, 0] - vals[s, t, 1])))
        assert layers == 24, f"{layers} layers: sequence {s} differs at step {t} (margin {margin})"
        assert margin <= _ulp16(rvals[s, t, 0]), (s, t, margin)
        assert sorted(ids[s, t].tolist()) == sorted(rids[s, t].tolist()), (s, t)
    n_same = tokens.shape[0] - len(turned)
    print(f"\n{layers} layers: {n_same} of {tokens.shape[0]} sequences identical over "
          f"{tokens.shape[1]} tokens; turned at fp16 ties (sequence, step, reference margin, "
          f"ours): {turned}")
    from custom_inference_engine_b200 import native
    assert native.device_errors(0) == 0
