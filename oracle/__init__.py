"""CPU oracle for the paged GQA attention hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this
directory: it is the checker used by ``tests/``, by
``__graft_entry__.smoke()`` and by the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py``. The product path runs the CUDA
extension and fails loudly when it is missing.
"""
from .attention import (  # noqa: F401
    GROUP,
    HEAD_DIM,
    H_KV,
    H_Q,
    PAGE_SIZE,
    SCALE,
    decode_attention_blockwise,
    decode_attention_fp32,
    decode_update_ref,
    mixed_attention_blockwise,
    mixed_attention_fp32,
    mixed_update_ref,
    rope_ref,
    valid_token_rows,
)
