"""The reference engine's graph modules trace over this package's ops (CPU).

``DecodeModule`` and ``FullMixedModule`` compile their forward with
``torch.compile(fullgraph=True, dynamic=False)`` (scheduler/decode_module.py:38-48,
scheduler/mixed_module.py:196-206 of the reference), and ``PiecewiseMixedModule``
splits the traced graph at every ``torch.ops.inference.gqa_mixed_attention.default``
node, grouped with the node of its ``kv_lens`` argument (piecewise/utils.py:5-23).
Here Dynamo traces the reference modules' own ``_forward`` methods (the
reference's code, unchanged, from baseline/_ref) over a 2-layer Qwen2 whose
attention is this package's ``TritonQwen2Attention``, with the ops' fake
kernels standing in for the CUDA ones: no graph break may occur, and the
reference splitter must find one attention group per layer. The GPU test
(``test_reference_modules_gpu.py``) compiles, captures and runs them.
"""
import pytest
import torch

N_LAYERS = 3


class _Traced(Exception):
    pass


def _capture_backend(graphs):
    def backend(gm, example_inputs):
        graphs.append(gm)

        def never_run(*args):
            raise _Traced
        return never_run
    return backend


@pytest.fixture(scope="module")
def small_model():
    from custom_inference_engine_b200 import model_runner as MR

    cfg = MR.qwen2_config(num_hidden_layers=N_LAYERS, vocab_size=512, intermediate_size=256)
    return MR.random_qwen2(cfg, seed=0, device="cpu")


def _trace(fn):
    graphs = []
    compiled = torch.compile(fn, fullgraph=True, dynamic=False,
                             backend=_capture_backend(graphs))
    with torch.inference_mode(), pytest.raises(_Traced):
        compiled()
    assert len(graphs) == 1
    return graphs[0]


def _targets(gm):
    return [n.target for n in gm.graph.nodes if n.op == "call_function"]


def _kv(model, reference_modules):
    import kv_cache.storage as storage   # resolved to this package by the fixture

    from custom_inference_engine_b200.kv_cache.storage import KVStorage
    assert storage.KVStorage is KVStorage
    return KVStorage(model.config, max_cache_len=256, page_size=16, n_slots=5,
                     device=torch.device("cpu"), dtype=torch.float16)


def test_decode_module_forward_traces_as_one_graph(reference_modules, small_model):
    import attn.metadata
    from attn.core import use_triton_attention

    R = reference_modules
    use_triton_attention(small_model)
    d = R.decode_module.DecodeModule.__new__(R.decode_module.DecodeModule)
    d.model, d.kv_cache, d.batch_size = small_model, _kv(small_model, R), 4
    d.metadata = attn.metadata.AttentionMetadata(token_count=4, device="cpu", full_decode=True)
    d.metadata.prepare_full_graph(4)
    d.static_token = torch.zeros((1, 4), dtype=torch.long)
    d.static_position_ids = torch.zeros((1, 4), dtype=torch.long)
    gm = _trace(d._forward)
    fused = torch.ops.inference.rope_kv_decode_attention.default
    assert _targets(gm).count(fused) == N_LAYERS


@pytest.mark.parametrize("fuse_rope", [True, False])
def test_mixed_module_forward_splits_at_every_attention(reference_modules, small_model,
                                                        fuse_rope):
    import attn.metadata
    from attn.core import TritonQwen2Attention, use_triton_attention

    R = reference_modules
    use_triton_attention(small_model)
    m = R.mixed_module.MixedModule.__new__(R.mixed_module.MixedModule)
    m.model, m.kv_cache, m.token_count = small_model, _kv(small_model, R), 64
    m.metadata = attn.metadata.AttentionMetadata(token_count=64, device="cpu", full_decode=False)
    m.metadata.prepare_full_graph(4)
    m.static_input_ids = torch.zeros((1, 64), dtype=torch.long)
    m.static_position_ids = torch.zeros((1, 64), dtype=torch.long)
    saved = TritonQwen2Attention.fuse_rope
    TritonQwen2Attention.fuse_rope = fuse_rope
    try:
        gm = _trace(m._forward)
    finally:
        TritonQwen2Attention.fuse_rope = saved
    attn_op = torch.ops.inference.gqa_mixed_attention.default
    assert _targets(gm).count(attn_op) == N_LAYERS
    write = (torch.ops.inference.rope_kv_mixed_update.default if fuse_rope
             else torch.ops.inference.kv_mixed_update.default)
    assert _targets(gm).count(write) == N_LAYERS   # K and V of a layer in one op

    pw = R.piecewise_utils
    split = pw.split(gm, pw.create_partition(gm))
    pieces = list(split.named_children())
    assert len(pieces) == 2 * N_LAYERS + 1
    for i, (name, sub) in enumerate(pieces):
        # even pieces are compiled + captured, odd ones are the eager
        # kv_lens gather + attention groups
        assert pw.is_graph_piece(sub) == (i % 2 == 0), name
        if i % 2:
            ops = [n.target for n in sub.graph.nodes if n.op == "call_function"]
            assert ops.count(attn_op) == 1
            assert len(ops) <= 3, ops   # the gather of kv_lens (and its index) + the op
