"""ctypes wrapper over ``liboracle.so`` — the CPU oracle (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module.  It restates ggml's CPU semantics for the quantized
matvec path (see ``ggml_semantics.c`` for the algorithm and the reference
file:line each piece follows) and is the checker the CUDA path is held to.
"""
import ctypes
import os

import numpy as np

from . import build as _build

F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, IQ4_XS = 0, 1, 8, 12, 13, 14, 15, 23
QK = 256
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
         Q8_K: (256, 292), IQ4_XS: (256, 136)}
FLOAT_TYPES = (F32, F16)

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.LIB
        if not os.path.exists(path):
            _build.build_oracle()
        L = ctypes.CDLL(path)
        vp, i64, fp = ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p
        for name in ("orc_dequantize_row_q4_K", "orc_dequantize_row_q5_K", "orc_dequantize_row_q6_K",
                     "orc_dequantize_row_q8_0", "orc_dequantize_row_iq4_xs", "orc_dequantize_row_f16",
                     "orc_quantize_row_q8_K", "orc_quantize_row_q8_0", "orc_quantize_row_q4_K",
                     "orc_quantize_row_q5_K", "orc_quantize_row_q6_K", "orc_quantize_row_iq4_xs",
                     "orc_quantize_row_f16"):
            getattr(L, name).argtypes = [vp, vp, i64]
            getattr(L, name).restype = None
        for name in ("orc_vec_dot_q4_K_q8_K", "orc_vec_dot_q5_K_q8_K", "orc_vec_dot_q6_K_q8_K",
                     "orc_vec_dot_iq4_xs_q8_K", "orc_vec_dot_q8_0_q8_0", "orc_vec_dot_f16_f32",
                     "orc_vec_dot_f32_f32"):
            getattr(L, name).argtypes = [i64, vp, vp]
            getattr(L, name).restype = ctypes.c_float
        L.orc_matvec.argtypes = [ctypes.c_int, vp, i64, i64, vp, ctypes.c_int, fp, ctypes.c_int]
        L.orc_matvec.restype = ctypes.c_int
        L.orc_quantize_rows.argtypes = [ctypes.c_int, vp, i64, i64, vp, ctypes.c_int]
        L.orc_quantize_rows.restype = ctypes.c_int
        L.orc_dequantize_rows.argtypes = [ctypes.c_int, vp, i64, i64, fp]
        L.orc_dequantize_rows.restype = ctypes.c_int
        L.orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.orc_fp16_to_fp32.restype = ctypes.c_float
        L.orc_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.orc_fp32_to_fp16.restype = ctypes.c_uint16
        L.orc_max_threads.restype = ctypes.c_int
        L.orc_argmax.argtypes = [fp, i64]
        L.orc_argmax.restype = ctypes.c_int64
        L.orc_simd_level.restype = ctypes.c_int
        L.orc_simd_level.argtypes = []
        L.orc_matvec_q4K_simd.argtypes = [vp, i64, i64, vp, ctypes.c_int, fp, ctypes.c_int, ctypes.c_int]
        L.orc_matvec_q4K_simd.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


def row_bytes(qtype, k):
    be, bb = BLOCK[qtype]
    assert k % be == 0, (qtype, k)
    return k // be * bb


def max_threads():
    return lib().orc_max_threads()


def quantize_weights(qtype, x, nthreads=0):
    """fp32 [rows, k] -> uint8 [rows, row_bytes] in ggml type ``qtype``."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    out = np.empty((rows, row_bytes(qtype, k)), dtype=np.uint8)
    assert lib().orc_quantize_rows(qtype, _p(x), rows, k, _p(out), nthreads) == 0
    return out


def dequantize(qtype, w, k):
    """uint8 [rows, row_bytes] -> fp32 [rows, k]."""
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1, row_bytes(qtype, k))
    out = np.empty((w.shape[0], k), dtype=np.float32)
    assert lib().orc_dequantize_rows(qtype, _p(w), w.shape[0], k, _p(out)) == 0
    return out


def quantize_q8_K(x):
    """fp32 [n, k] (k % 256 == 0) -> uint8 [n, k/256*292] activation blocks."""
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    n, k = x.shape
    out = np.empty((n, row_bytes(Q8_K, k)), dtype=np.uint8)
    for t in range(n):
        lib().orc_quantize_row_q8_K(_p(x[t]), _p(out[t]), k)
    return out


def quantize_q8_0(x):
    """fp32 [n, k] (k % 32 == 0) -> uint8 [n, k/32*34] activation blocks."""
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    n, k = x.shape
    out = np.empty((n, row_bytes(Q8_0, k)), dtype=np.uint8)
    for t in range(n):
        lib().orc_quantize_row_q8_0(_p(x[t]), _p(out[t]), k)
    return out


def act_type_for(qtype):
    """Activation format a weight type's dot product takes: q8_0 for q8_0,
    fp32 rows for f16 / f32 (converted inside the dot), q8_K otherwise."""
    return Q8_0 if qtype == Q8_0 else (F32 if qtype in FLOAT_TYPES else Q8_K)


def quantize_act(qtype, x):
    if qtype in FLOAT_TYPES:
        return np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32).view(np.uint8)
    return quantize_q8_0(x) if qtype == Q8_0 else quantize_q8_K(x)


def matvec(qtype, w, k, xq, nthreads=0):
    """y[t, r] = W[r] . x[t] with ggml dot-product semantics; xq from quantize_act."""
    w = np.ascontiguousarray(w).view(np.uint8)
    rows = w.size // row_bytes(qtype, k)
    xq = np.ascontiguousarray(np.atleast_2d(xq))
    if xq.dtype != np.uint8:
        xq = xq.view(np.uint8)
    ntok = xq.shape[0]
    y = np.empty((ntok, rows), dtype=np.float32)
    assert lib().orc_matvec(qtype, _p(w), rows, k, _p(xq), ntok, _p(y), nthreads) == 0
    return y


SIMD_NAMES = {0: "scalar", 1: "AVX2 (vpmaddubsw + vpmaddwd)", 2: "AVX-512 VNNI (vpdpbusd)"}


def simd_level():
    """Instruction set of the vectorised q4_K matvec on this CPU (see SIMD_NAMES)."""
    return int(lib().orc_simd_level())


def matvec_q4K_simd(w, k, xq, nthreads=0, level=-1):
    """q4_K matvec with the vectorised dot product (the timed CPU baseline);
    equal bit for bit to matvec(Q4_K, ...).  Returns (y, level used)."""
    w = np.ascontiguousarray(w).view(np.uint8)
    rows = w.size // row_bytes(Q4_K, k)
    xq = np.ascontiguousarray(np.atleast_2d(xq))
    if xq.dtype != np.uint8:
        xq = xq.view(np.uint8)
    ntok = xq.shape[0]
    y = np.empty((ntok, rows), dtype=np.float32)
    lv = lib().orc_matvec_q4K_simd(_p(w), rows, k, _p(xq), ntok, _p(y), nthreads, level)
    return y, lv


def argmax(v):
    v = np.ascontiguousarray(v, dtype=np.float32)
    return int(lib().orc_argmax(_p(v), v.size))


def fp16_to_fp32(h):
    return lib().orc_fp16_to_fp32(int(h))


def fp32_to_fp16(f):
    return lib().orc_fp32_to_fp16(float(f))


def rms_norm(x, eps=1e-6):
    """RMSNorm with weight 1.0 in fp32 (sum of squares accumulated in fp64 then rounded)."""
    x = np.asarray(x, dtype=np.float32)
    ms = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True)
    return (x / np.sqrt(ms + eps).astype(np.float32)).astype(np.float32)


def silu_mul(g, u):
    g = np.asarray(g, dtype=np.float32)
    return (g / (1.0 + np.exp(-g.astype(np.float64))).astype(np.float32) * u).astype(np.float32)


def ffn(gate_w, up_w, down_w, hidden, k_in, k_ffn, down_type=Q6_K, gate_type=Q4_K):
    """down(silu(gate.x) * up.x) for RMSNormed hidden rows, ggml semantics per matvec."""
    x = rms_norm(hidden)
    xq = quantize_act(gate_type, x)
    g = matvec(gate_type, gate_w, k_in, xq)
    u = matvec(gate_type, up_w, k_in, xq)
    a = silu_mul(g, u)
    aq = quantize_act(down_type, a)
    return matvec(down_type, down_w, k_ffn, aq)


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
