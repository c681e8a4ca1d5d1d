"""Loaders for the package's two native libraries.

``lib()`` returns the ctypes handle of ``libcie_attention.so`` (the C ABI in
``include/cie_attention.h``) with argument types declared; ``load_ops()``
registers the ``inference::*`` torch ops from ``_cie_torch_ops.so`` and their
fake (meta) implementations for Dynamo. Both raise ``NativeLibraryMissing``
when the libraries have not been built: there is no CPU or Python fallback
for any op of this package.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libcie_attention.so"
OPS_PATH = PKG / "_cie_torch_ops.so"


class NativeLibraryMissing(RuntimeError):
    """The CUDA extension of this package is not built (run ``__graft_entry__.build()``)."""


c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_ptr = ctypes.c_void_p
c_size = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/cie_attention.h and include/cie_model_ops.h
SIGNATURES = {
    "cie_version": (c_int, []),
    "cie_status_string": (ctypes.c_char_p, [c_int]),
    "cie_last_error_message": (ctypes.c_char_p, []),
    "cie_read_device_errors": (c_int, [c_int, ctypes.POINTER(ctypes.c_uint), c_int]),
    "cie_decode_default_splits": (c_int, [c_int, c_int]),
    "cie_decode_workspace_bytes": (c_size, [c_int, c_int, c_int, c_int]),
    "cie_decode_attention": (c_int, [c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr,
                                     c_size, c_int, c_int, c_int, c_int, c_int, c_i64, c_i64,
                                     c_i64, c_i64, c_i64, c_int, c_ptr]),
    "cie_decode_attention_noalloc": (c_int, [c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr,
                                             c_int, c_int, c_int, c_int, c_int, c_i64, c_i64,
                                             c_i64, c_i64, c_i64, c_int, c_ptr]),
    "cie_mixed_workspace_bytes": (c_size, [c_int, c_i64, c_int, c_int, c_int]),
    "cie_mixed_attention": (c_int, [c_ptr, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_ptr,
                                    c_ptr, c_ptr, c_size, c_int, c_i64, c_int, c_int, c_int,
                                    c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_int, c_ptr]),
    "cie_kv_decode_update": (c_int, [c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_int,
                                     c_int, c_int, c_int, c_i64, c_i64, c_i64, c_i64, c_i64,
                                     c_i64, c_i64, c_i64, c_i64, c_ptr]),
    "cie_kv_mixed_update": (c_int, [c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_int,
                                    c_int, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                    c_i64, c_ptr]),
    "cie_rope_kv_decode_update": (c_int, [c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_ptr,
                                          c_ptr, c_ptr, c_ptr, c_int, c_int, c_int, c_int, c_int,
                                          c_i64, c_i64, c_i64, c_i64, c_i64, c_ptr]),
    "cie_rope_kv_mixed_update": (c_int, [c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_ptr,
                                         c_ptr, c_ptr, c_i64, c_int, c_int, c_int, c_int, c_i64,
                                         c_i64, c_i64, c_ptr]),
    "cie_rope_kv_decode_attention": (c_int, [c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr,
                                             c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_size, c_int,
                                             c_int, c_int, c_int, c_int, c_i64, c_i64, c_i64,
                                             c_i64, c_i64, c_int, c_ptr]),
    "cie_rope_kv_mixed_workspace_bytes": (c_size, [c_int, c_i64, c_int, c_int, c_int, c_int]),
    "cie_rope_kv_mixed_attention": (c_int, [c_ptr, c_i64, c_ptr, c_ptr, c_i64, c_ptr, c_ptr,
                                            c_ptr, c_ptr, c_i64, c_ptr, c_ptr, c_ptr, c_ptr,
                                            c_ptr, c_ptr, c_size, c_int, c_i64, c_int, c_int,
                                            c_int, c_int, c_i64, c_i64, c_i64, c_i64, c_i64,
                                            c_int, c_ptr]),
}
# the int32-block-table variants take the same arguments
for _name in ("cie_decode_attention", "cie_mixed_attention", "cie_kv_decode_update",
              "cie_rope_kv_decode_update", "cie_rope_kv_decode_attention",
              "cie_rope_kv_mixed_attention"):
    SIGNATURES[_name + "_bt32"] = SIGNATURES[_name]
SIGNATURES.update({
    # include/cie_model_ops.h
    "cie_rms_norm": (c_int, [c_ptr, c_ptr, c_ptr, c_ptr, c_i64, c_int, c_i64, c_i64, c_i64,
                             ctypes.c_float, c_ptr]),
    "cie_silu_mul": (c_int, [c_ptr, c_ptr, c_ptr, c_i64, c_int, c_i64, c_i64, c_i64, c_ptr]),
    "cie_argmax_workspace_bytes": (c_size, [c_i64]),
    "cie_argmax_rows": (c_int, [c_ptr, c_i64, c_int, c_i64, c_ptr, c_ptr, c_size, c_ptr]),
    "cie_lm_head_argmax_workspace_bytes": (c_size, [c_int, c_i64, c_int]),
    "cie_lm_head_argmax": (c_int, [c_ptr, c_i64, c_ptr, c_i64, c_int, c_int, c_i64, c_ptr,
                                   c_i64, c_ptr, c_ptr, c_size, c_ptr]),
})

CIE_OK = 0
STATUS = {
    0: "CIE_OK",
    -1: "CIE_ERR_INVALID_ARGUMENT",
    -2: "CIE_ERR_UNSUPPORTED",
    -3: "CIE_ERR_OVERFLOW",
    -4: "CIE_ERR_ALIGNMENT",
    -5: "CIE_ERR_WORKSPACE",
    -6: "CIE_ERR_CUDA",
}

_lock = threading.Lock()
_lib = None
_ops_loaded = False


def lib() -> ctypes.CDLL:
    """The C-ABI library with ctypes signatures applied (loaded once)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise NativeLibraryMissing(
                    f"{LIB_PATH.name} is not built; run __graft_entry__.build()")
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(status: int, what: str = "cie call") -> None:
    """Raise RuntimeError for a non-zero C-ABI status, with the library's message."""
    if status != CIE_OK:
        msg = lib().cie_last_error_message().decode(errors="replace")
        raise RuntimeError(f"{what}: {STATUS.get(status, status)}: {msg}")


def device_errors(device: int = 0, clear: bool = True) -> int:
    """Device error bits (cie_device_error_bits) of ``device``; synchronises it."""
    bits = ctypes.c_uint(0)
    check(lib().cie_read_device_errors(device, ctypes.byref(bits), 1 if clear else 0),
          "cie_read_device_errors")
    return int(bits.value)


def load_ops() -> None:
    """Register the ``inference::*`` torch ops (CUDA kernels + fake kernels)."""
    global _ops_loaded
    with _lock:
        if _ops_loaded:
            return
        if not OPS_PATH.exists() or not LIB_PATH.exists():
            raise NativeLibraryMissing(
                f"{OPS_PATH.name} / {LIB_PATH.name} not built; run __graft_entry__.build()")
        torch.ops.load_library(str(OPS_PATH))
        _register_fakes()
        _ops_loaded = True


def _register_fakes() -> None:
    @torch.library.register_fake("inference::gqa_decode_attention")
    def _decode_fake(q, k, v, lens, slot_ids, block_table):
        return torch.empty_like(q)

    @torch.library.register_fake("inference::gqa_decode_attention_splits")
    def _decode_splits_fake(q, k, v, lens, slot_ids, block_table, num_splits):
        return torch.empty_like(q)

    @torch.library.register_fake("inference::gqa_mixed_attention")
    def _mixed_fake(q, k, v, max_seqlen, cu_seqlens, kv_lens, slot_ids, block_table):
        return torch.empty_like(q)

    @torch.library.register_fake("inference::kv_decode_update")
    def _dec_upd_fake(k_cache, v_cache, lens, slot_ids, block_table, k_new, v_new):
        return None

    @torch.library.register_fake("inference::kv_mixed_update")
    def _mix_upd_fake(k_cache, v_cache, pages, offsets, k_new, v_new):
        return None

    def _rope_out(qkv, k_cache):
        hkv, d = k_cache.shape[1], k_cache.shape[3]
        hq = qkv.shape[-1] // d - 2 * hkv
        return qkv.new_empty((1, qkv.shape[1], hq, d))

    @torch.library.register_fake("inference::rope_kv_decode_update")
    def _rope_dec_fake(qkv, cos, sin, k_cache, v_cache, lens, slot_ids, block_table):
        return _rope_out(qkv, k_cache)

    @torch.library.register_fake("inference::rope_kv_mixed_update")
    def _rope_mix_fake(qkv, cos, sin, k_cache, v_cache, pages, offsets):
        return _rope_out(qkv, k_cache)

    @torch.library.register_fake("inference::rope_kv_mixed_attention")
    def _rope_mix_attn_fake(qkv, cos, sin, k_cache, v_cache, pages, offsets, max_seqlen,
                            cu_seqlens, kv_lens, slot_ids, block_table):
        return _rope_out(qkv, k_cache)

    @torch.library.register_fake("inference::rope_kv_decode_attention")
    def _rope_dec_attn_fake(qkv, cos, sin, k_cache, v_cache, lens, slot_ids, block_table):
        return _rope_out(qkv, k_cache)

    @torch.library.register_fake("inference::rms_norm")
    def _rms_fake(x, weight, eps):
        return torch.empty_like(x, memory_format=torch.contiguous_format)

    @torch.library.register_fake("inference::add_rms_norm")
    def _add_rms_fake(residual, delta, weight, eps):
        return torch.empty_like(residual, memory_format=torch.contiguous_format)

    @torch.library.register_fake("inference::argmax_rows")
    def _argmax_fake(x):
        return x.new_empty(x.shape[:-1], dtype=torch.long)

    @torch.library.register_fake("inference::lm_head_argmax")
    def _lm_head_argmax_fake(hidden, weight):
        return hidden.new_empty(hidden.shape[:-1], dtype=torch.long)

    @torch.library.register_fake("inference::silu_and_mul")
    def _silu_mul_fake(gate_up):
        return gate_up.new_empty((*gate_up.shape[:-1], gate_up.shape[-1] // 2))


def stream_ptr(stream=None) -> int:
    """Raw cudaStream_t of ``stream`` (default: torch's current stream)."""
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream)
