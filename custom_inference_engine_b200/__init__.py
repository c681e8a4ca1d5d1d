"""B200-native (sm_100a) paged GQA attention for the custom inference engine.

The package mirrors the reference engine's attention boundary:

* ``custom_inference_engine_b200.attn.core`` -- host functions and the
  ``inference::gqa_decode_attention`` / ``inference::gqa_mixed_attention``
  torch ops (same schemas as the reference ``triton_op`` wrappers), plus
  ``TritonQwen2Attention`` / ``use_triton_attention``;
* ``custom_inference_engine_b200.attn.metadata`` -- ``AttentionMetadata``;
* ``custom_inference_engine_b200.kv_cache.storage`` -- ``KVStorage`` whose
  ``decode_update`` / ``mixed_update`` run the CUDA KV-page scatter.

All compute runs in hand-written CUDA kernels inside ``libcie_attention.so``
(C ABI, declared in ``include/cie_attention.h``); ``_cie_torch_ops.so``
registers the torch ops on top of it. There is no CPU fallback: importing
the ops without the built libraries raises.
"""

__all__ = ["native", "install_reference_aliases"]

# Top-level module names under which the reference engine imports its attention
# boundary (scheduler/decode_module.py:3-6, scheduler/mixed_module.py:4-8,
# scheduler/scheduler.py:9-11).
REFERENCE_MODULES = ("attn", "attn.core", "attn.metadata", "kv_cache", "kv_cache.storage")


def install_reference_aliases() -> None:
    """Make the reference engine's ``import attn.core`` / ``attn.metadata`` /
    ``kv_cache.storage`` resolve to this package's modules.

    The reference's scheduler, graph modules and piecewise backend import the
    attention boundary as top-level packages. After this call those imports
    return the very module objects of ``custom_inference_engine_b200.attn`` and
    ``.kv_cache`` (one ``TritonQwen2Attention`` class, one op registration), so
    the reference code runs unchanged on the CUDA ops. Raises ``RuntimeError``
    if another ``attn`` / ``kv_cache`` (the reference's own Triton one) is
    already imported: the two register the same ``inference::*`` op names.
    """
    import importlib
    import sys

    for name in REFERENCE_MODULES:
        mod = importlib.import_module(f"{__name__}.{name}")
        present = sys.modules.get(name)
        if present is not None and present is not mod:
            raise RuntimeError(f"module {name!r} is already imported from "
                               f"{getattr(present, '__file__', '?')}")
        sys.modules[name] = mod
