"""cie_decode_attention_noalloc against cie_decode_attention.

The no-allocation entry point serves callers that cannot allocate device
memory (an FFI host holding only device pointers, or a process whose HBM is
already fully reserved for weights and the KV pool). It must give the same
output as the workspace-taking entry point, call after call, although every
call reuses the same built-in scratch array. This file is collected last so
that a failure here never hides the other tests.
"""
import pytest
import torch

from custom_inference_engine_b200 import cabi, native
from custom_inference_engine_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _case(lens, seed, dev):
    c = W.make_decode_case(lens, seed=seed)
    return [t.to(dev) for t in (c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)]


def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    """Both entry points launch the same kernels with the same split count, so
    their outputs are compared bit for bit. The calls run large, small, large:
    the small call's partials cover only the start of the scratch, with the
    previous call's partials left beyond them, so a read outside the call's own
    region would show up as a difference."""
    native.device_errors(0, clear=True)
    cases = [(_case([4096] * 3 + [5, 800], 42, cuda_device), 0),       # ~59 splits per row
             (_case([1, 300, 17, 0], 41, cuda_device), 2),
             (_case([1, 300, 17, 0, 4096, 1024, 33, 2000], 43, cuda_device), 8)]
    for args, splits in cases:
        S = splits or cabi.decode_default_splits(args[4].shape[0], 0)
        assert cabi.decode_workspace_bytes(args[4].shape[0], 14, 64, S) > 0
        for _ in range(2):
            got = cabi.decode_attention_noalloc(*args, num_splits=splits)
            want = cabi.decode_attention(*args, num_splits=splits)
            torch.cuda.synchronize()
            assert torch.equal(got, want)
    assert native.device_errors(0) == 0


def test_noalloc_rejects_requests_beyond_its_scratch(cuda_device):
    args = _case([64] * 4, 43, cuda_device)
    with pytest.raises(RuntimeError, match="WORKSPACE"):
        cabi.decode_attention_noalloc(*args, num_splits=400)
