"""The fused last-token lm_head + argmax (cie_lm_head_argmax, inference::lm_head_argmax).

It replaces the lm_head GEMM + argmax of the reference's decode and mixed
modules (scheduler/decode_module.py:103-107, scheduler/mixed_module.py:58-65).
Its tokens must be exactly torch.argmax of the logits it computes (first
index of the maximum, NaN largest), those logits must be a fp16 GEMM's within
fp16 rounding of the fp32 dot products, and wherever a cuBLAS GEMM's logits
give another token, the two candidates must be within one fp16 ulp there
(the same tie, rounded the other way).
"""
import pytest
import torch

from custom_inference_engine_b200 import cabi, native
from custom_inference_engine_b200 import model_runner as MR

native.load_ops()  # torch.ops.inference.* (also when this file runs alone)

pytestmark = pytest.mark.gpu
VOCAB, HIDDEN = 151936, 896


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    native.device_errors(0, clear=True)
    yield
    assert native.device_errors(0, clear=True) == 0


def _ulp16(x):
    return torch.from_numpy(__import__("numpy").spacing(x.abs().cpu().half().numpy())).float()


def _check(hidden, weight):
    tokens, logits = cabi.lm_head_argmax(hidden, weight, logits=True)
    torch.cuda.synchronize()
    # the tokens are torch.argmax of the kernel's own logits, bit for bit
    assert torch.equal(tokens, logits.argmax(dim=-1))
    ref = hidden @ weight.t()                       # cuBLAS fp16 GEMM, fp32 accumulation
    exact = (hidden.float() @ weight.float().t())   # fp32 dot products
    # one fp16 rounding of the fp32 dot product (plus slack for the fp32
    # summation order)
    err = (logits.float() - exact).abs()
    assert bool((err <= 0.5 * _ulp16(exact).to(err.device) + 1e-4).all()), float(err.max())
    assert (logits.float() - ref.float()).abs().max().item() <= 4e-3
    want = ref.argmax(dim=-1)
    for b in torch.nonzero(tokens != want).flatten().tolist():
        a, c = int(tokens[b]), int(want[b])
        gap = (ref[b, c].float() - ref[b, a].float()).abs()
        assert gap <= _ulp16(ref[b, c].float().reshape(1)).item(), (b, a, c, float(gap))
    return tokens, logits


@pytest.mark.parametrize("batch", [1, 5, 64, 70])
def test_qwen2_head_against_cublas(batch, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(batch)
    w = (torch.randn(VOCAB, HIDDEN, generator=g, device=cuda_device) * 0.02).half()
    h = torch.randn(batch, HIDDEN, generator=g, device=cuda_device).half()
    tokens, _ = _check(h, w)
    op = torch.ops.inference.lm_head_argmax(h, w)
    assert torch.equal(op, tokens)
    # strided hidden rows (a view of a wider buffer)
    wide = torch.zeros(batch, HIDDEN + 64, dtype=torch.float16, device=cuda_device)
    wide[:, :HIDDEN] = h
    assert torch.equal(torch.ops.inference.lm_head_argmax(wide[:, :HIDDEN], w), tokens)


@pytest.mark.parametrize("vocab,hidden", [(1000, 64), (129, 1024), (128, 896)])
def test_other_shapes(vocab, hidden, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(vocab)
    w = (torch.randn(vocab, hidden, generator=g, device=cuda_device) * 0.05).half()
    h = torch.randn(17, hidden, generator=g, device=cuda_device).half()
    _check(h, w)


def test_maximum_at_every_range_edge(cuda_device):
    """The maximum placed on 128-row chunk edges, on the vocab's last rows and on
    the first and last rows of every range of an even split into 148 or 132
    parts is found (each position in its own hidden row)."""
    hidden = 64
    g = torch.Generator(device=cuda_device).manual_seed(11)
    w = (torch.randn(VOCAB, hidden, generator=g, device=cuda_device) * 0.02).half()
    units = (VOCAB + 15) // 16
    pos = {0, 127, 128, 1023, 1024, 1039, 1040, VOCAB - 17, VOCAB - 16, VOCAB - 1}
    for grid in (148, 132):
        for c in range(grid):
            pos.add(units * c // grid * 16)
            pos.add(min(units * (c + 1) // grid * 16, VOCAB) - 1)
    pos = sorted(pos)
    eye = torch.eye(hidden, dtype=torch.float16, device=cuda_device)
    for i0 in range(0, len(pos), hidden):
        rows = pos[i0:i0 + hidden]
        w2 = w.clone()
        for i, r in enumerate(rows):
            w2[r] = 4 * eye[i]      # logit 4 for h row i, about 0.02 everywhere else
        h = eye[:len(rows)].contiguous()
        tokens, logits = cabi.lm_head_argmax(h, w2, logits=True)
        assert torch.equal(tokens, logits.argmax(dim=-1))
        assert tokens.tolist() == rows


def test_ties_nan_and_zero_rows(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(3)
    w = (torch.randn(4096, HIDDEN, generator=g, device=cuda_device) * 0.02).half()
    h = torch.randn(6, HIDDEN, generator=g, device=cuda_device).half()
    w[3000] = w[77] * 4            # row 1: a clear maximum at 77, repeated at 3000
    w[77] = w[3000]
    h[1] = w[77].float().sign().half()
    h[2] = 0                       # all logits +-0: the first index wins
    w[2500] = float("nan")         # every row's logit 2500 is NaN: NaN counts as largest
    tokens, logits = cabi.lm_head_argmax(h, w, logits=True)
    assert torch.equal(tokens, logits.argmax(dim=-1))
    assert int(tokens[2]) == 2500 and int(tokens[0]) == 2500
    w[2500] = 0
    tokens, logits = cabi.lm_head_argmax(h, w, logits=True)
    assert torch.equal(tokens, logits.argmax(dim=-1))
    assert int(tokens[1]) == 77
    assert int(tokens[2]) == 0


def test_decode_steps_with_the_fused_head(cuda_device):
    """The runner's decode graph gives the same greedy tokens with the fused
    lm_head + argmax as with the lm_head GEMM + argmax."""
    cfg = MR.qwen2_config(num_hidden_layers=2)
    model = MR.random_qwen2(cfg, seed=0, device=cuda_device)
    prompts = [list(range(11, 11 + n)) for n in (5, 40, 130, 1)]
    toks = {}
    for fused in (True, False):
        runner = MR.PagedRunner(model, max_cache_len=2048, n_slots=5, token_budget=256,
                                fused_lm_head=fused)
        slots = [1, 2, 3, 4]
        for s, p in zip(slots, prompts):
            runner.admit(s, len(p) + 12)
        pre = runner.prefill(slots, prompts)
        graph = runner.decode_graph(slots, pre.first_tokens, capture=True)
        toks[fused] = [graph.step().tolist() for _ in range(10)]
        assert (graph.logits is None) == fused
    assert toks[True] == toks[False]
