"""The C-ABI library loads and exports what include/*.h declares (CPU only).

Also checks the argument validation paths that return before any CUDA call,
and the pure-host size helpers.
"""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = {}
    inc = os.path.join(ROOT, "include")
    for f in sorted(os.listdir(inc)):
        if not f.endswith(".h"):
            continue
        src = open(os.path.join(inc, f)).read()
        for m in re.finditer(r"^M27B_API\s+[^;(]*?\b(\w+)\s*\(", src, re.M):
            names[m.group(1)] = f
    return names


def test_headers_declare_the_api():
    names = declared_functions()
    for fn in ("m27b_act_quant", "m27b_qmv", "m27b_qmv_swiglu", "m27b_qmv_argmax", "m27b_repack", "m27b_dequant_rows"):
        assert fn in names


def test_library_exports_every_declared_symbol(m27b):
    lib = ctypes.CDLL(m27b.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_version(m27b):
    assert "sm_100a" in m27b.version()


def test_size_helpers(m27b):
    L = m27b.lib()
    assert L.m27b_act_bytes(m27b.Q8_K, 5120) == 20 * 292
    assert L.m27b_act_bytes(m27b.Q8_0, 1024) == 32 * 34
    assert L.m27b_act_bytes(m27b.Q8_K, 5000) == 0
    assert L.m27b_act_bytes(m27b.Q4_K, 5120) == 0
    assert L.m27b_act_type_for(m27b.Q4_K) == m27b.Q8_K
    assert L.m27b_act_type_for(m27b.Q6_K | m27b.LAYOUT_PLANAR) == m27b.Q8_K
    assert L.m27b_act_type_for(m27b.Q8_0) == m27b.Q8_0
    assert L.m27b_act_type_for(1) == 0
    # repacked q6_K rows: 4-block tiles of 848 bytes; q8_0 rows: codes then the d plane padded to 16 B
    assert L.m27b_repacked_bytes(m27b.Q6_K, 20, 3) == 3 * 5 * 848  # 4-block tiles of 848 bytes
    assert L.m27b_repacked_bytes(m27b.Q6_K, 68, 1) == 17 * 848
    assert L.m27b_repacked_bytes(m27b.Q6_K, 17, 1) == 5 * 848  # padded to whole tiles
    assert L.m27b_repacked_bytes(m27b.Q8_0, 32, 5) == 5 * (32 * 32 + 64)
    assert L.m27b_repacked_bytes(m27b.Q4_K, 20, 1) == 0


def _view(m27b, ptr, t, rb, rc):
    return ctypes.byref(m27b.WeightView(ptr, t, rb, rc))


@pytest.mark.parametrize("case,needle", [
    ("null_view", "null WeightView"),
    ("null_ptr", "null weight pointer"),
    ("unaligned", "16-byte aligned"),
    ("empty", "empty weight"),
    ("raw_q6K", "must be repacked"),
    ("bad_type", "unsupported weight type"),
    ("bad_flags", "unknown layout flags"),
    ("iq4xs_odd_blocks", "even number of blocks"),
    ("f16_ragged_row", "multiple of 8"),
    ("f16_with_q8_acts", "fp32 activations"),
])
def test_qmv_rejects_bad_views(m27b, case, needle):
    v = {
        "null_view": None,
        "null_ptr": _view(m27b, None, m27b.Q4_K, 20, 8),
        "unaligned": _view(m27b, 0x1008, m27b.Q4_K, 20, 8),
        "empty": _view(m27b, 0x1000, m27b.Q4_K, 0, 8),
        "raw_q6K": _view(m27b, 0x1000, m27b.Q6_K, 20, 8),
        "bad_type": _view(m27b, 0x1000, 2, 20, 8),  # q4_0: not on this path
        "bad_flags": _view(m27b, 0x1000, m27b.Q4_K | 0x200, 20, 8),
        "iq4xs_odd_blocks": _view(m27b, 0x1000, m27b.IQ4_XS, 3, 8),
        "f16_ragged_row": _view(m27b, 0x1000, m27b.F16, 20, 8),
        "f16_with_q8_acts": _view(m27b, 0x1000, m27b.F16, 64, 8),
    }[case]
    ok, msg = m27b.call_raw("m27b_qmv", v, ctypes.c_void_p(0x2000), 1, ctypes.c_void_p(0x3000), 8, None, None)
    assert not ok and needle in msg, msg


@pytest.mark.parametrize("ntok", [0, 17, -1])
def test_qmv_rejects_bad_token_counts(m27b, ntok):
    v = _view(m27b, 0x1000, m27b.Q4_K, 20, 8)
    ok, msg = m27b.call_raw("m27b_qmv", v, ctypes.c_void_p(0x2000), ntok, ctypes.c_void_p(0x3000), 8, None, None)
    assert not ok and "n_tok" in msg


def test_swiglu_rejects_mismatched_shapes(m27b):
    g = _view(m27b, 0x1000, m27b.Q4_K, 20, 8)
    u = _view(m27b, 0x2000, m27b.Q4_K, 20, 9)
    ok, msg = m27b.call_raw("m27b_qmv_swiglu", g, u, ctypes.c_void_p(0x3000), 1, ctypes.c_void_p(0x4000), 8, None)
    assert not ok and "same type and shape" in msg


def test_act_quant_rejects_bad_k(m27b):
    ok, msg = m27b.call_raw("m27b_act_quant", ctypes.c_void_p(0x1000), 300, 1, 300, m27b.Q8_K, ctypes.c_void_p(0x2000), None)
    assert not ok and "multiple of the block size" in msg
    ok, msg = m27b.call_raw("m27b_act_quant", ctypes.c_void_p(0x1000), 256, 1, 100, m27b.Q8_K, ctypes.c_void_p(0x2000), None)
    assert not ok and "ldx" in msg


def test_repack_rejects_other_types(m27b):
    ok, msg = m27b.call_raw("m27b_repack", ctypes.c_void_p(0x1000), m27b.Q4_K, 20, 4, ctypes.c_void_p(0x2000), None)
    assert not ok and "only raw q6_K and q8_0" in msg
    ok, msg = m27b.call_raw("m27b_repack", ctypes.c_void_p(0x1000), m27b.Q6_K, 20, 4, ctypes.c_void_p(0x2008), None)
    assert not ok and "16-byte aligned" in msg


def test_missing_library_fails_loudly(m27b, monkeypatch, tmp_path):
    monkeypatch.setattr(m27b, "_lib", None)
    monkeypatch.setattr(m27b, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(m27b.M27BError):
        m27b.lib()
