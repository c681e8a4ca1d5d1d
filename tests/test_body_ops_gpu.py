"""The Qwen2 body kernels (include/cie_model_ops.h, torch ops inference::rms_norm,
add_rms_norm, silu_and_mul) against the Hugging Face modules they replace.

SiLU-mul and the residual add follow torch's arithmetic exactly and must give
the same bits. RMSNorm's sum of squares is reduced in another order than
torch's: the normalised value may then round one fp16 ulp apart in rare
elements, which the multiplication by the weight (|w| up to ~1.3 here) can
turn into two ulps of the output.
"""
import pytest
import torch

from custom_inference_engine_b200 import model_runner as MR

pytestmark = pytest.mark.gpu

HIDDEN = 896


@pytest.fixture(scope="module")
def ops(cuda_device):
    from custom_inference_engine_b200.attn import core  # noqa: F401  (loads the ops)
    return torch.ops.inference


def _hf_norm(weight, eps=1e-6):
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RMSNorm
    n = Qwen2RMSNorm(weight.shape[0], eps=eps).to(weight.device, torch.float16)
    with torch.no_grad():
        n.weight.copy_(weight)
    return n


def _ulps(a, b):
    """Distance in fp16 ulps (same-sign finite values)."""
    ia = a.view(torch.int16).to(torch.int32)
    ib = b.view(torch.int16).to(torch.int32)
    return (ia - ib).abs()


@pytest.mark.parametrize("rows", [1, 5, 64, 2048])
def test_rms_norm_matches_hf(ops, cuda_device, rows):
    g = torch.Generator(device=cuda_device).manual_seed(rows)
    x = torch.randn(1, rows, HIDDEN, generator=g, device=cuda_device).half() * 3
    w = (1 + 0.1 * torch.randn(HIDDEN, generator=g, device=cuda_device)).half()
    ref = _hf_norm(w)(x)
    out = ops.rms_norm(x, w, 1e-6)
    d = _ulps(out, ref)
    exact = (d == 0).float().mean().item()
    assert int(d.max()) <= 2 and exact >= 0.99, (int(d.max()), exact)


def test_add_rms_norm_matches_residual_then_hf_norm(ops, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(3)
    h = torch.randn(1, 77, HIDDEN, generator=g, device=cuda_device).half()
    delta = torch.randn(1, 77, HIDDEN, generator=g, device=cuda_device).half()
    w = (1 + 0.1 * torch.randn(HIDDEN, generator=g, device=cuda_device)).half()
    want_h = h + delta
    want = _hf_norm(w)(want_h)
    out = ops.add_rms_norm(h, delta, w, 1e-6)
    assert torch.equal(h, want_h)            # residual stream updated in place, exact
    d = _ulps(out, want)
    exact = (d == 0).float().mean().item()
    assert int(d.max()) <= 2 and exact >= 0.99, (int(d.max()), exact)


def test_rms_norm_row_strided_input(ops, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(4)
    wide = torch.randn(1, 9, HIDDEN + 64, generator=g, device=cuda_device).half()
    x = wide[..., :HIDDEN]
    w = torch.randn(HIDDEN, generator=g, device=cuda_device).half()
    assert torch.equal(ops.rms_norm(x, w, 1e-6), ops.rms_norm(x.contiguous(), w, 1e-6))


@pytest.mark.parametrize("rows", [1, 64, 1000])
def test_silu_and_mul_is_bit_exact(ops, cuda_device, rows):
    g = torch.Generator(device=cuda_device).manual_seed(rows)
    gu = (torch.randn(1, rows, 2 * 4864, generator=g, device=cuda_device) * 4).half()
    gate, up = gu.split(4864, dim=-1)
    want = torch.nn.functional.silu(gate) * up
    assert torch.equal(ops.silu_and_mul(gu), want)


def test_rotary_table_equals_per_pass_rotary(cuda_device):
    cfg = MR.qwen2_config(num_hidden_layers=1, vocab_size=256, intermediate_size=256)
    model = MR.random_qwen2(cfg, seed=0, device=cuda_device)
    body = MR.FusedQwen2Body(model, max_positions=4096)
    pos = torch.tensor([[0, 1, 17, 600, 4095, 2048]], device=cuda_device)
    probe = torch.zeros(1, 1, dtype=torch.float16, device=cuda_device)
    cos, sin = model.model.rotary_emb(probe, pos)
    assert torch.equal(body.cos[pos[0]], cos[0]) and torch.equal(body.sin[pos[0]], sin[0])


@pytest.mark.parametrize("rows,n", [(64, 151936), (3, 4096), (5, 1001)])
def test_argmax_rows_matches_torch(ops, cuda_device, rows, n):
    """The greedy argmax over the vocabulary gives torch.argmax's index: the
    first of equal maxima (values 0..3 make ties everywhere), also for a row
    of -inf and on a row-strided view."""
    g = torch.Generator(device=cuda_device).manual_seed(n)
    x = torch.randint(0, 4, (rows, n), generator=g, device=cuda_device).half()
    x[-1].fill_(float("-inf"))
    assert torch.equal(ops.argmax_rows(x), x.argmax(-1))
    y = torch.randn(rows, n + 8, generator=g, device=cuda_device).half()[:, :n]
    assert torch.equal(ops.argmax_rows(y), y.argmax(-1))
