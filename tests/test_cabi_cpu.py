"""The C-ABI library loads without a GPU, exports every symbol the header
declares, and rejects bad arguments on the host before launching anything."""
import ctypes
import re
from pathlib import Path

import pytest

from custom_inference_engine_b200 import native

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))


def declared_functions():
    names = set()
    for header in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(cie_[a-z_0-9]+)\s*\(", text))
    return sorted(names)


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    for must in ("cie_decode_attention", "cie_mixed_attention", "cie_kv_decode_update",
                 "cie_kv_mixed_update", "cie_decode_workspace_bytes", "cie_rms_norm",
                 "cie_silu_mul"):
        assert must in names


def test_every_declared_symbol_is_exported():
    handle = ctypes.CDLL(str(native.LIB_PATH))
    for name in declared_functions():
        assert hasattr(handle, name), name
    assert set(declared_functions()) == set(native.SIGNATURES)


def test_host_only_queries():
    lib = native.lib()
    assert lib.cie_version() >= 1
    assert lib.cie_status_string(-2) == b"unsupported shape"
    assert lib.cie_decode_workspace_bytes(256, 14, 64, 1) == 0
    assert lib.cie_decode_workspace_bytes(8, 14, 64, 4) == 8 * 4 * 14 * 66 * 4
    assert lib.cie_decode_default_splits(0, -1) == 1
    assert lib.cie_decode_default_splits(256, -1) == 1
    assert lib.cie_decode_default_splits(8, -1) == 32    # 37 rounded down to a power of two
    assert lib.cie_decode_default_splits(12, -1) == 24   # 24 is 3/2 of 16: kept
    assert lib.cie_decode_default_splits(32, -1) == 8    # 9 -> 8
    assert lib.cie_decode_default_splits(96, -1) == 3
    assert lib.cie_decode_default_splits(1, -1) == 64   # capped: the merge outgrows the gain


def _decode(**kw):
    args = dict(q=1 << 20, k=1 << 21, v=1 << 22, lens=1 << 23, slot_ids=1 << 24, bt=1 << 25,
                o=1 << 26, ws=None, ws_bytes=0, batch=4, hq=14, hkv=2, d=64, page=16,
                n_pages=100, n_slots=5, bt_stride=100, pstride=2048, hstride=1024, splits=1,
                stream=None)
    args.update(kw)
    return native.lib().cie_decode_attention(*args.values())


@pytest.mark.parametrize("kw,status", [
    (dict(q=None), -1),
    (dict(batch=-1), -1),
    (dict(d=128), -2),
    (dict(page=32), -2),
    (dict(hq=16), -2),
    (dict(hkv=3, hq=21), -2),
    (dict(n_pages=1 << 31), -3),
    (dict(pstride=2000), -1),
    (dict(pstride=2052, hstride=1026), -4),
    (dict(k=(1 << 21) + 2), -4),
    (dict(splits=4), -5),
])
def test_decode_argument_checks(kw, status):
    assert _decode(**kw) == status
    assert native.lib().cie_last_error_message()


def test_decode_empty_batch_is_a_no_op():
    assert _decode(batch=0, q=None) == 0


def test_mixed_and_update_argument_checks():
    lib = native.lib()
    p = 1 << 20
    def mixed(**kw):
        a = dict(q=p, k=p, v=p, max_seqlen=16, cu=p, kvl=p, slots=p, bt=p, o=p, ws=None,
                 ws_bytes=0, batch=2, T=16, hq=14, hkv=2, d=64, page=16, n_pages=10, n_slots=3,
                 bt_stride=10, pstride=2048, hstride=1024, splits=1, stream=None)
        a.update(kw)
        return lib.cie_mixed_attention(*a.values())
    assert mixed(d=128) == -2
    assert mixed(q=None) == -1
    assert mixed(max_seqlen=0) == 0
    for splits in (0, 1, 4):
        assert mixed(splits=splits) == -5        # the plan always needs workspace
    assert mixed(splits=17) == -1
    assert mixed(batch=2049, T=4096, max_seqlen=16) == -2

    def plan_bytes(batch, T, hkv, splits, sms=148):
        # header | items (2 x int4) | split counters | records of 2 x 128 rows x 66 fp32
        r256 = lambda x: (x + 255) // 256 * 256
        units = hkv * ((T + 35) // 36 + batch)
        if splits >= 1:
            items, split, rec = splits * units, (units if splits > 1 else 0), \
                (splits * units if splits > 1 else 0)
        else:  # automatic plan: 3/2 x SMs slots
            slots = (sms * 3 + 1) // 2
            items, split, rec = units + slots, slots, 2 * slots
        return 256 + r256(items * 32) + r256(split * 4) + rec * 256 * 66 * 4
    for args in ((4, 2048, 2, 1), (4, 2048, 2, 3), (4, 2048, 2, 0), (32, 2048, 2, 0),
                 (1, 1, 2, 16)):
        assert lib.cie_mixed_workspace_bytes(*args, -1) == plan_bytes(*args)
    assert lib.cie_mixed_workspace_bytes(4, 2048, 2, 0, -1) < 32 << 20
    assert lib.cie_kv_mixed_update(None, p, p, p, p, p, 4, 2, 64, 16, 10, 2048, 1024, 1152, 64,
                                   1152, 64, None) == -1
    # fused RoPE + KV write: qkv row 1152, cos/sin row 64, pool strides 2048 / 1024
    assert lib.cie_rope_kv_mixed_update(p, 1152, p, p, 64, p, p, p, p, p, 0, 14, 2, 64, 16, 10,
                                        2048, 1024, None) == 0  # nothing to do
    assert lib.cie_rope_kv_mixed_update(p, 1152, p, p, 64, p, p, p, None, p, 4, 14, 2, 64, 16,
                                        10, 2048, 1024, None) == -1
    assert lib.cie_rope_kv_mixed_update(p, 1152, p, p, 64, p, p, p, p, p, 4, 14, 2, 128, 16,
                                        10, 2048, 1024, None) == -2
    assert lib.cie_rope_kv_mixed_update(p, 1000, p, p, 64, p, p, p, p, p, 4, 14, 2, 64, 16,
                                        10, 2048, 1024, None) == -1   # rows overlap
    assert lib.cie_rope_kv_mixed_update(p + 2, 1152, p, p, 64, p, p, p, p, p, 4, 14, 2, 64, 16,
                                        10, 2048, 1024, None) == -4   # misaligned
    assert lib.cie_rope_kv_decode_update(p, 1152, p, p, 64, p, p, p, None, p, p, 4, 14, 2, 64,
                                         16, 10, 3, 10, 2048, 1024, None) == -1
    assert lib.cie_kv_decode_update(p, p, p, p, p, p, p, 4, 2, 64, 16, 10, 3, 10, 100, 1024,
                                    1152, 64, 1152, 64, None) == -1


def test_body_kernel_argument_checks():
    """RMSNorm / SiLU-mul entry points reject bad arguments on the host."""
    lib = native.lib()
    p = 1 << 20
    rms = lambda h=p, d=None, w=p, o=p, rows=4, hidden=896, hs=896, ds=896, os_=896, eps=1e-6: \
        lib.cie_rms_norm(h, d, w, o, rows, hidden, hs, ds, os_, eps, None)
    assert rms(rows=0) == 0
    assert rms(h=None) == -1
    assert rms(rows=-1) == -1
    assert rms(hidden=900, hs=900, os_=900) == -2
    assert rms(h=p + 2) == -4
    assert rms(hs=900) == -4
    assert rms(d=p + 8) == -4
    assert rms(hs=888) == -1
    assert rms(eps=-1.0) == -1
    silu = lambda g=p, u=p + 9728, o=p, rows=4, n=4864, gs=9728, us=9728, os_=4864: \
        lib.cie_silu_mul(g, u, o, rows, n, gs, us, os_, None)
    assert silu(rows=0) == 0
    assert silu(g=None) == -1
    assert silu(n=4860, os_=4860) == -2
    assert silu(u=p + 2) == -4
    assert silu(os_=4800) == -1


def test_fused_decode_and_argmax_argument_checks():
    """cie_rope_kv_decode_attention and cie_argmax_rows reject bad arguments
    on the host."""
    lib = native.lib()
    p = 1 << 20

    def fused(**kw):
        a = dict(qkv=p, qkv_tok=1152, cos=p, sin=p, cs_tok=64, k=p, v=p, lens=p, slots=p, bt=p,
                 o=p, ws=None, ws_bytes=0, batch=4, hq=14, hkv=2, d=64, page=16, n_pages=100,
                 n_slots=5, bt_stride=100, pstride=2048, hstride=1024, splits=1, stream=None)
        a.update(kw)
        return lib.cie_rope_kv_decode_attention(*a.values())
    assert fused(batch=0) == 0
    assert fused(qkv=None) == -1
    assert fused(qkv_tok=1000) == -1          # rows overlap
    assert fused(qkv=p + 2) == -4
    assert fused(d=128) == -2
    assert fused(splits=4) == -5              # the split path needs workspace
    assert lib.cie_argmax_workspace_bytes(64) == 64 * 16 * 8
    assert lib.cie_argmax_rows(p, 0, 10, 10, p, None, 0, None) == 0
    assert lib.cie_argmax_rows(p, 4, 10, 10, p, None, 0, None) == -5
    assert lib.cie_argmax_rows(p + 1, 4, 10, 10, p, p, 1 << 10, None) == -4
    assert lib.cie_argmax_rows(p, 4, 10, 8, p, p, 1 << 10, None) == -1


def test_noalloc_checks_arguments_before_its_scratch_limit():
    """cie_decode_attention_noalloc reports a bad argument with the status
    cie_decode_attention gives it; CIE_ERR_WORKSPACE only for a valid request
    that is too large for the built-in scratch."""
    lib = native.lib()

    def noalloc(**kw):
        a = dict(q=1 << 20, k=1 << 21, v=1 << 22, lens=1 << 23, slot_ids=1 << 24, bt=1 << 25,
                 o=1 << 26, batch=4, hq=14, hkv=2, d=64, page=16, n_pages=100, n_slots=5,
                 bt_stride=100, pstride=2048, hstride=1024, splits=1, stream=None)
        a.update(kw)
        return lib.cie_decode_attention_noalloc(*a.values())
    assert noalloc(batch=0) == 0
    assert noalloc(q=None, splits=5000) == -1      # null pointer, not a scratch overflow
    assert noalloc(splits=5000) == -1              # num_splits > 4096 is invalid
    assert noalloc(d=128, splits=400) == -2
    assert noalloc(k=(1 << 21) + 2, splits=400) == -4
    assert noalloc(splits=400) == -5               # valid, but 4 x 400 splits > 4 MiB


def test_bt32_variants_check_arguments_like_the_int64_ones():
    """The int32-block-table entry points reject what the int64 ones reject."""
    lib = native.lib()
    p = 1 << 20
    args = [p, p, p, p, p, p, p, None, 0, 4, 14, 2, 64, 16, 100, 5, 100, 2048, 1024]
    assert lib.cie_decode_attention_bt32(None, *args[1:], 1, None) == -1
    bad = list(args)
    bad[12] = 128   # head_dim
    assert lib.cie_decode_attention_bt32(*bad, 1, None) == -2
    assert lib.cie_decode_attention_bt32(*args, 4, None) == -5   # split path without workspace
    assert lib.cie_kv_decode_update_bt32(p, p, p, p, None, p, p, 4, 2, 64, 16, 10, 3, 10, 2048,
                                         1024, 1152, 64, 1152, 64, None) == -1


def test_rope_kv_mixed_attention_argument_checks():
    """The one-call RoPE + K/V write + mixed attention rejects bad arguments
    on the host: missing pages, a workspace without room for the rotated q."""
    lib = native.lib()
    p = 1 << 20

    def call(**kw):
        a = dict(qkv=p, qkv_tok=1152, cos=p, sin=p, cs_tok=64, k=p, v=p, pages=p, offsets=p,
                 max_seqlen=16, cu=p, kvl=p, slots=p, bt=p, o=p, ws=p, ws_bytes=0, batch=2,
                 T=16, hq=14, hkv=2, d=64, page=16, n_pages=10, n_slots=3, bt_stride=10,
                 pstride=2048, hstride=1024, splits=0, stream=None)
        a.update(kw)
        return lib.cie_rope_kv_mixed_attention(*a.values())
    assert call(pages=None) == -1
    assert call(d=128) == -2
    need = lib.cie_rope_kv_mixed_workspace_bytes(2, 16, 14, 2, 0, -1)
    assert need >= lib.cie_mixed_workspace_bytes(2, 16, 2, 0, -1) + 16 * 14 * 64 * 2
    assert call(ws_bytes=need - 1) == -5
    assert call(qkv_tok=1000, ws_bytes=need) == -1      # qkv rows overlap
    assert call(batch=0, T=0) == 0
