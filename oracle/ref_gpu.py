"""ctypes wrapper over oracle/_ref/libref_gpu.so — the reference executor's
own quantizer and batch-1 matvec kernels compiled for sm_100a (comparison arm;
test and benchmark infrastructure only, see ref_gpu_harness.cu).

The reference quantizes activations to q8_1 (32-value blocks, 36 bytes) and
reads raw GGUF blocks; its results differ from ggml's q8_K semantics at the
~1e-2 level, so it is a timing comparison, not a parity oracle."""
import ctypes
import os

from . import build as _build

_lib = None
Q8_0, Q4_K, Q6_K = 8, 12, 14
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210, Q8_0: 34}
BLOCK_ELEMS = {Q4_K: 256, Q6_K: 256, Q8_0: 32}


def available():
    return os.path.exists(_build.REF_GPU)


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise RuntimeError("oracle/_ref/libref_gpu.so is not built (needs the reference checkout at build time)")
        L = ctypes.CDLL(_build.REF_GPU)
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        L.refgpu_quant_q8_1.argtypes = [vp, vp, i32, vp]
        L.refgpu_quant_q8_1.restype = i32
        L.refgpu_matvec.argtypes = [i32, vp, vp, vp, i32, i32, vp]
        L.refgpu_matvec.restype = i32
        _lib = L
    return _lib


def q8_1_bytes(k):
    return k // 32 * 36


def quant_q8_1(x_ptr, q8_ptr, n, stream_ptr):
    rc = lib().refgpu_quant_q8_1(ctypes.c_void_p(x_ptr), ctypes.c_void_p(q8_ptr), n, ctypes.c_void_p(stream_ptr))
    if rc != 0:
        raise RuntimeError(f"refgpu_quant_q8_1: CUDA error {rc}")


def matvec(qtype, w_ptr, q8_ptr, y_ptr, rb, rows, stream_ptr):
    rc = lib().refgpu_matvec(qtype, ctypes.c_void_p(w_ptr), ctypes.c_void_p(q8_ptr), ctypes.c_void_p(y_ptr), rb, rows,
                             ctypes.c_void_p(stream_ptr))
    if rc != 0:
        raise RuntimeError(f"refgpu_matvec: CUDA error {rc}")
