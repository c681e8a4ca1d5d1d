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

__all__ = ["native"]
