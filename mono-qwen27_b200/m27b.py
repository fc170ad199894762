"""ctypes binding of libm27b.so, the C ABI declared in include/m27b_qmv.h.

This is the Python mirror of the reference's matvec seam (WeightView +
quantize/matvec calls, src/mono27b_executor.cu:1989-2261) used by the tests and
the benchmark.  PyTorch only provides device memory and streams; every
computation goes through the CUDA library.  There is no fallback: if
libm27b.so is missing or fails to load, every call raises.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libm27b.so")

# ggml type codes (reference include/mono27b_gguf.h:28-44; IQ4_XS = 23)
F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, IQ4_XS = 0, 1, 8, 12, 13, 14, 15, 23
LAYOUT_PLANAR = 0x100
MAX_TOKENS = 16
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
         Q8_K: (256, 292), IQ4_XS: (256, 136)}

ERR_CAP = 512


class WeightView(ctypes.Structure):
    """Same layout as the reference's WeightView (include/mono27b_config.h:63-68)."""
    _fields_ = [("ptr", ctypes.c_void_p), ("ggml_type", ctypes.c_uint32), ("row_blocks", ctypes.c_uint32),
                ("row_count", ctypes.c_uint32)]


class M27BError(RuntimeError):
    pass


_lib = None


def lib():
    """Load libm27b.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise M27BError(f"libm27b.so is not built ({LIB_PATH}); run __graft_entry__.build()")
    L = ctypes.CDLL(LIB_PATH)
    vp, u32, i32, sz, cp = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_size_t, ctypes.c_char_p
    fp, b = ctypes.c_float, ctypes.c_bool
    wvp = ctypes.POINTER(WeightView)
    sig = {
        "m27b_version": (cp, []),
        "m27b_device_status": (b, [ctypes.POINTER(ctypes.c_int), i32, cp, sz]),
        "m27b_act_bytes": (sz, [u32, i32]),
        "m27b_act_type_for": (u32, [u32]),
        "m27b_act_quant": (b, [vp, i32, i32, i32, u32, vp, vp, cp, sz]),
        "m27b_act_quant_gated": (b, [vp, vp, i32, i32, i32, u32, vp, vp, cp, sz]),
        "m27b_act_quant_swiglu": (b, [vp, vp, i32, i32, i32, u32, vp, vp, cp, sz]),
        "m27b_act_quant_rmsnorm": (b, [vp, vp, fp, i32, i32, i32, u32, vp, vp, cp, sz]),
        "m27b_repacked_bytes": (sz, [u32, u32, u32]),
        "m27b_repack": (b, [vp, u32, u32, u32, vp, vp, cp, sz]),
        "m27b_qmv": (b, [wvp, vp, i32, vp, i32, vp, vp, cp, sz]),
        "m27b_qmv_swiglu": (b, [wvp, wvp, vp, i32, vp, i32, vp, cp, sz]),
        "m27b_qmv_argmax": (b, [wvp, vp, i32, vp, i32, vp, u32, vp, cp, sz]),
        "m27b_qmv_f32": (b, [wvp, vp, i32, i32, vp, vp, i32, vp, vp, cp, sz]),
        "m27b_qmv_f32_rmsnorm": (b, [wvp, wvp, vp, i32, vp, fp, i32, vp, vp, i32, vp, vp, cp, sz]),
        "m27b_dequant_rows": (b, [wvp, vp, i32, vp, i32, vp, cp, sz]),
        "m27b_hbm_read_probe": (b, [vp, sz, vp, cp, sz]),
        "m27b_hbm_read_probe_shape": (b, [vp, sz, i32, i32, i32, i32, vp, cp, sz]),
        "m27b_qmv_mma_split_part_bytes": (sz, [wvp, i32]),
        "m27b_qmv_mma_split_count_bytes": (sz, [wvp]),
        "m27b_qmv_mma_split": (b, [wvp, vp, i32, vp, i32, vp, vp, vp, vp, cp, sz]),
        "m27b_qmv_q6k_mma_part_bytes": (sz, [wvp]),
        "m27b_qmv_q6k_mma_count_bytes": (sz, [wvp]),
        "m27b_qmv_q6k_mma": (b, [wvp, vp, i32, vp, i32, vp, vp, vp, vp, cp, sz]),
        "m27b_qmv_q6k_mma_argmax": (b, [wvp, vp, i32, vp, i32, vp, u32, vp, cp, sz]),
        "m27b_qmv_q6k_stream_part_bytes": (sz, [wvp]),
        "m27b_qmv_q6k_stream_count_bytes": (sz, [wvp]),
        "m27b_qmv_q6k_stream": (b, [wvp, vp, vp, vp, vp, vp, vp, cp, sz]),
        "m27b_qmv_q6k_ksplit_part_bytes": (sz, [wvp]),
        "m27b_qmv_q6k_ksplit_count_bytes": (sz, [wvp]),
        "m27b_qmv_q6k_ksplit": (b, [wvp, vp, i32, vp, i32, vp, vp, vp, vp, cp, sz]),
        "m27b_allreduce_norm_quant": (b, [vp, i32, i32, vp, vp, vp, fp, i32, vp, vp, ctypes.c_ulonglong, vp, cp, sz]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def version():
    return lib().m27b_version().decode()


def device_status(clear=True):
    """The device status word (0 = every bounded kernel wait completed)."""
    v = ctypes.c_int(0)
    err = ctypes.create_string_buffer(ERR_CAP)
    _check(lib().m27b_device_status(ctypes.byref(v), 1 if clear else 0, err, ERR_CAP), err, "m27b_device_status")
    return v.value


def row_bytes(qtype, k):
    be, bb = BLOCK[qtype & 0xff]
    assert k % be == 0
    return k // be * bb


def act_type_for(qtype):
    """q8_0 for q8_0 weights, q8_K for the 256-value types, 0 (fp32 rows) for f16 / f32."""
    b = qtype & 0xff
    return Q8_0 if b == Q8_0 else (0 if b in (F16, F32) else Q8_K)


def act_bytes(act_type, k):
    return lib().m27b_act_bytes(act_type, k)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(stream):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _check(ok, err, what):
    if not ok:
        raise M27BError(f"{what}: {err.value.decode(errors='replace')}")


class QWeight:
    """A quantized (or f16 / f32) weight matrix resident on the device.

    Holds the device bytes (a torch uint8 tensor) and the WeightView the C ABI
    consumes.  q6_K and q8_0 are repacked to the planar layout on upload; for
    f16 / f32 row_blocks counts values, as in the reference loader.
    """

    def __init__(self, raw_u8, qtype, k, rows, device="cuda", stream=None, keep_raw=False):
        import torch
        self.qtype, self.k, self.rows = qtype, k, rows
        be = BLOCK[qtype][0]
        self.row_blocks = k // be
        raw = torch.as_tensor(raw_u8).reshape(-1)
        if raw.dtype != torch.uint8:
            raw = raw.view(torch.uint8)
        assert raw.numel() == rows * row_bytes(qtype, k), (raw.numel(), rows, row_bytes(qtype, k))
        raw_dev = raw.to(device) if raw.device.type != "cuda" else raw
        if qtype in (Q6_K, Q8_0):
            n = lib().m27b_repacked_bytes(qtype, self.row_blocks, rows)
            self.data = torch.empty(n, dtype=torch.uint8, device=raw_dev.device)
            err = ctypes.create_string_buffer(ERR_CAP)
            _check(lib().m27b_repack(_ptr(raw_dev), qtype, self.row_blocks, rows, _ptr(self.data), _stream(stream), err,
                                     ERR_CAP), err, "m27b_repack")
            self.view = WeightView(self.data.data_ptr(), qtype | LAYOUT_PLANAR, self.row_blocks, rows)
            self.raw = raw_dev if keep_raw else None
        else:
            self.data = raw_dev.contiguous()
            self.view = WeightView(self.data.data_ptr(), qtype, self.row_blocks, rows)
            self.raw = self.data
        self.nbytes = rows * row_bytes(qtype, k)  # stored GGUF bytes (algorithmic)

    @property
    def act_type(self):
        return act_type_for(self.qtype)


def act_quant(x, act_type, out=None, stream=None, gate=None, norm_w=None, eps=None):
    """Quantize fp32 rows x [n, k] (device) to q8_K / q8_0 blocks (device uint8)."""
    import torch
    x = x if x.dim() == 2 else x.reshape(1, -1)
    n, k = x.shape
    nb = act_bytes(act_type, k)
    if nb == 0:
        raise M27BError(f"act_quant: bad k={k} for type {act_type}")
    if out is None:
        out = torch.empty(n * nb, dtype=torch.uint8, device=x.device)
    err = ctypes.create_string_buffer(ERR_CAP)
    L = lib()
    if gate is not None:
        ok = L.m27b_act_quant_gated(_ptr(x), _ptr(gate), k, n, x.stride(0), act_type, _ptr(out), _stream(stream), err,
                                    ERR_CAP)
    elif eps is not None:
        ok = L.m27b_act_quant_rmsnorm(_ptr(x), _ptr(norm_w), ctypes.c_float(eps), k, n, x.stride(0), act_type, _ptr(out),
                                      _stream(stream), err, ERR_CAP)
    else:
        ok = L.m27b_act_quant(_ptr(x), k, n, x.stride(0), act_type, _ptr(out), _stream(stream), err, ERR_CAP)
    _check(ok, err, "m27b_act_quant")
    return out


def allreduce_norm_quant(words, nsrc, src_stride, ss_words, epoch, k, x_out, xq, norm_w=None, eps=1e-6, wait_ns=0,
                         stream=None):
    """The fused all-reduce's consumer (include/m27b_allreduce.h): sum the nsrc
    ranks' epoch-tagged words (device int64 tensors, value bits low, epoch
    high) once they carry *epoch (device uint32), then RMSNorm + q8_K into xq."""
    err = ctypes.create_string_buffer(ERR_CAP)
    ok = lib().m27b_allreduce_norm_quant(_ptr(words), nsrc, src_stride, _ptr(ss_words), _ptr(epoch), _ptr(norm_w),
                                         ctypes.c_float(eps), k, _ptr(x_out), _ptr(xq), ctypes.c_ulonglong(wait_ns),
                                         _stream(stream), err, ERR_CAP)
    _check(ok, err, "m27b_allreduce_norm_quant")
    return xq


def qmv_q6k_ksplit(w, xq, n_tok, y, residual=None, part=None, count=None, stream=None, ldy=None):
    """q6_K x n_tok (5..16) tokens with K split across CTAs (m27b_qmv_q6k_ksplit);
    part / count scratch are allocated here (counters zeroed) unless given."""
    import torch
    L = lib()
    if part is None:
        part = torch.empty(max(16, L.m27b_qmv_q6k_ksplit_part_bytes(ctypes.byref(w.view))), dtype=torch.uint8,
                           device="cuda")
    if count is None:
        count = torch.zeros(max(16, L.m27b_qmv_q6k_ksplit_count_bytes(ctypes.byref(w.view))), dtype=torch.uint8,
                            device="cuda")
    err = ctypes.create_string_buffer(ERR_CAP)
    _check(L.m27b_qmv_q6k_ksplit(ctypes.byref(w.view), _ptr(xq), n_tok, _ptr(y),
                                 ldy if ldy is not None else w.view.row_count, _ptr(residual), _ptr(part), _ptr(count),
                                 _stream(stream), err, ERR_CAP), err, "m27b_qmv_q6k_ksplit")
    return y


def qmv_mma_split(w, xq, n_tok, y, residual=None, part=None, count=None, stream=None, ldy=None):
    """q4_K x n_tok (5..16) tokens on the tensor cores with K split across CTAs
    (m27b_qmv_mma_split); part / count scratch are allocated here (counters
    zeroed) unless given."""
    import torch
    L = lib()
    if part is None:
        part = torch.empty(max(16, L.m27b_qmv_mma_split_part_bytes(ctypes.byref(w.view), n_tok)), dtype=torch.uint8,
                           device="cuda")
    if count is None:
        count = torch.zeros(max(16, L.m27b_qmv_mma_split_count_bytes(ctypes.byref(w.view))), dtype=torch.uint8,
                            device="cuda")
    err = ctypes.create_string_buffer(ERR_CAP)
    _check(L.m27b_qmv_mma_split(ctypes.byref(w.view), _ptr(xq), n_tok, _ptr(y),
                                ldy if ldy is not None else w.view.row_count, _ptr(residual), _ptr(part), _ptr(count),
                                _stream(stream), err, ERR_CAP), err, "m27b_qmv_mma_split")
    return y


def qmv_q6k_mma(w, xq, n_tok, y, residual=None, part=None, count=None, stream=None, ldy=None, split=True):
    """q6_K x n_tok (1..8) tokens on the tensor cores (m27b_qmv_q6k_mma); with
    split, K-split scratch is allocated here (counters zeroed) unless given."""
    import torch
    L = lib()
    if split and part is None:
        part = torch.empty(max(16, L.m27b_qmv_q6k_mma_part_bytes(ctypes.byref(w.view))), dtype=torch.uint8,
                           device="cuda")
    if split and count is None:
        count = torch.zeros(max(16, L.m27b_qmv_q6k_mma_count_bytes(ctypes.byref(w.view))), dtype=torch.uint8,
                            device="cuda")
    err = ctypes.create_string_buffer(ERR_CAP)
    _check(L.m27b_qmv_q6k_mma(ctypes.byref(w.view), _ptr(xq), n_tok, _ptr(y),
                              ldy if ldy is not None else w.view.row_count, _ptr(residual), _ptr(part), _ptr(count),
                              _stream(stream), err, ERR_CAP), err, "m27b_qmv_q6k_mma")
    return y


def qmv_q6k_mma_argmax(w, xq, n_tok, best, logits=None, row_offset=0, stream=None, ldl=None):
    """q6_K x n_tok (1..8) tokens on the tensor cores with the argmax epilogue
    (m27b_qmv_q6k_mma_argmax)."""
    err = ctypes.create_string_buffer(ERR_CAP)
    ldl = ldl if ldl is not None else w.rows
    _check(lib().m27b_qmv_q6k_mma_argmax(ctypes.byref(w.view), _ptr(xq), n_tok, _ptr(logits), ldl, _ptr(best),
                                         row_offset, _stream(stream), err, ERR_CAP), err, "m27b_qmv_q6k_mma_argmax")
    return best


def qmv_q6k_stream(w, xq, y, residual=None, part=None, count=None, stream=None):
    """q6_K x one token with the items cut evenly over warps
    (m27b_qmv_q6k_stream); part / count scratch are allocated here (counters
    zeroed) unless given."""
    import torch
    L = lib()
    if part is None:
        part = torch.empty(max(16, L.m27b_qmv_q6k_stream_part_bytes(ctypes.byref(w.view))), dtype=torch.uint8,
                           device="cuda")
    if count is None:
        count = torch.zeros(max(16, L.m27b_qmv_q6k_stream_count_bytes(ctypes.byref(w.view))), dtype=torch.uint8,
                            device="cuda")
    err = ctypes.create_string_buffer(ERR_CAP)
    _check(L.m27b_qmv_q6k_stream(ctypes.byref(w.view), _ptr(xq), _ptr(y), _ptr(residual), _ptr(part), _ptr(count),
                                 _stream(stream), err, ERR_CAP), err, "m27b_qmv_q6k_stream")
    return y


def hbm_read_probe(buf, shape=None, stream=None):
    """One streaming read of the device tensor `buf` (see
    m27b_hbm_read_probe_shape); shape = (warps, stages, chunk, ctas_per_sm)
    or None for the default one."""
    err = ctypes.create_string_buffer(ERR_CAP)
    n = buf.numel() * buf.element_size()
    if shape is None:
        ok = lib().m27b_hbm_read_probe(_ptr(buf), n, _stream(stream), err, ERR_CAP)
    else:
        ok = lib().m27b_hbm_read_probe_shape(_ptr(buf), n, *[int(v) for v in shape], _stream(stream), err, ERR_CAP)
    _check(ok, err, "m27b_hbm_read_probe")


def act_quant_swiglu(gate, up, act_type, out=None, stream=None):
    """Quantize silu(gate) * up (device rows [n, k]) to q8_K / q8_0 blocks."""
    import torch
    n, k = up.shape
    nb = act_bytes(act_type, k)
    if out is None:
        out = torch.empty(n * nb, dtype=torch.uint8, device=up.device)
    err = ctypes.create_string_buffer(ERR_CAP)
    _check(lib().m27b_act_quant_swiglu(_ptr(gate), _ptr(up), k, n, up.stride(0), act_type, _ptr(out), _stream(stream),
                                       err, ERR_CAP), err, "m27b_act_quant_swiglu")
    return out


def qmv(w, xq, n_tok, y, residual=None, stream=None, ldy=None):
    err = ctypes.create_string_buffer(ERR_CAP)
    ldy = ldy if ldy is not None else w.rows
    _check(lib().m27b_qmv(ctypes.byref(w.view), _ptr(xq), n_tok, _ptr(y), ldy, _ptr(residual), _stream(stream), err,
                          ERR_CAP), err, "m27b_qmv")
    return y


def qmv_swiglu(gate, up, xq, n_tok, y, stream=None, ldy=None):
    err = ctypes.create_string_buffer(ERR_CAP)
    ldy = ldy if ldy is not None else gate.rows
    _check(lib().m27b_qmv_swiglu(ctypes.byref(gate.view), ctypes.byref(up.view), _ptr(xq), n_tok, _ptr(y), ldy,
                                 _stream(stream), err, ERR_CAP), err, "m27b_qmv_swiglu")
    return y


def qmv_argmax(w, xq, n_tok, best, logits=None, row_offset=0, stream=None, ldl=None):
    err = ctypes.create_string_buffer(ERR_CAP)
    ldl = ldl if ldl is not None else w.rows
    _check(lib().m27b_qmv_argmax(ctypes.byref(w.view), _ptr(xq), n_tok, _ptr(logits), ldl, _ptr(best), row_offset,
                                 _stream(stream), err, ERR_CAP), err, "m27b_qmv_argmax")
    return best


def qmv_f32(w, x, n_tok, y, residual=None, xq_scratch=None, norm_w=None, eps=None, up=None, stream=None, ldy=None):
    """y = W . q8(x) (+ residual) from fp32 rows x [n_tok, k] (device); with eps
    given, x is RMSNormed (weights norm_w) first; with `up`, SwiGLU epilogue."""
    err = ctypes.create_string_buffer(ERR_CAP)
    L = lib()
    ldx = x.stride(0) if x.dim() == 2 else x.shape[-1]
    ldy = ldy if ldy is not None else w.view.row_count
    if eps is None and up is None:
        ok = L.m27b_qmv_f32(ctypes.byref(w.view), _ptr(x), ldx, n_tok, _ptr(xq_scratch), _ptr(y), ldy, _ptr(residual),
                            _stream(stream), err, ERR_CAP)
        _check(ok, err, "m27b_qmv_f32")
    else:
        ok = L.m27b_qmv_f32_rmsnorm(ctypes.byref(w.view), ctypes.byref(up.view) if up is not None else None, _ptr(x),
                                    ldx, _ptr(norm_w), ctypes.c_float(1e-6 if eps is None else eps), n_tok,
                                    _ptr(xq_scratch), _ptr(y), ldy, _ptr(residual), _stream(stream), err, ERR_CAP)
        _check(ok, err, "m27b_qmv_f32_rmsnorm")
    return y


def argmax_key_index(key):
    return 0xffffffff - (int(key) & 0xffffffff)


def dequant_rows(w, rows_dev, out, stream=None, view=None):
    err = ctypes.create_string_buffer(ERR_CAP)
    v = view if view is not None else w.view
    k = v.row_blocks * BLOCK[v.ggml_type & 0xff][0]
    _check(lib().m27b_dequant_rows(ctypes.byref(v), _ptr(rows_dev), rows_dev.numel(), _ptr(out), k, _stream(stream), err,
                                   ERR_CAP), err, "m27b_dequant_rows")
    return out


def call_raw(name, *args):
    """Call a C-ABI function with an error buffer appended; returns (ok, message)."""
    err = ctypes.create_string_buffer(ERR_CAP)
    ok = getattr(lib(), name)(*args, err, ERR_CAP)
    return bool(ok), err.value.decode(errors="replace")


# --------------------------------------------------------------------------
# decode attention (include/m27b_attn.h)


def _attn_lib():
    L = lib()
    if getattr(L, "_attn_sigs", False):
        return L
    vp, i32, sz, cp, fp, b = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_float, ctypes.c_bool
    L.m27b_attn_part_bytes.restype = sz
    L.m27b_attn_part_bytes.argtypes = [i32, i32, i32]
    L.m27b_attn_decode.restype = b
    L.m27b_attn_decode.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, fp, vp, vp, vp, cp, sz]
    L.m27b_attn_decode_noalloc.restype = b
    L.m27b_attn_decode_noalloc.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, fp, vp, vp, cp, sz]
    L.m27b_attn_noalloc_scratch_bytes.restype = sz
    L.m27b_attn_noalloc_scratch_bytes.argtypes = []
    L._attn_sigs = True
    return L


def attn_part_bytes(n_q, head_dim, splits):
    return _attn_lib().m27b_attn_part_bytes(n_q, head_dim, splits)


def attn_decode(q, k_cache, v_cache, pos, n_q, n_kv, head_dim, splits, scale, part, out, stream=None):
    """Decode attention of n_q heads over cache positions [0, pos[0]] (all device tensors)."""
    err = ctypes.create_string_buffer(ERR_CAP)
    ok = _attn_lib().m27b_attn_decode(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(pos), n_q, n_kv, head_dim, splits,
                                      ctypes.c_float(scale), _ptr(part), _ptr(out), _stream(stream), err, ERR_CAP)
    _check(ok, err, "m27b_attn_decode")
    return out


def attn_noalloc_scratch_bytes():
    """Capacity of m27b_attn_decode_noalloc's static scratch, as compiled into the library."""
    return _attn_lib().m27b_attn_noalloc_scratch_bytes()


def attn_decode_noalloc(q, k_cache, v_cache, pos, n_q, n_kv, head_dim, splits, scale, out, stream=None):
    """m27b_attn_decode with the library's static scratch (no scratch argument, no allocation)."""
    err = ctypes.create_string_buffer(ERR_CAP)
    ok = _attn_lib().m27b_attn_decode_noalloc(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(pos), n_q, n_kv, head_dim,
                                              splits, ctypes.c_float(scale), _ptr(out), _stream(stream), err, ERR_CAP)
    _check(ok, err, "m27b_attn_decode_noalloc")
    return out


# --------------------------------------------------------------------------
# decode engine (include/m27b_engine.h)


class ModelConfig(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("hidden", ctypes.c_int), ("ffn", ctypes.c_int), ("n_head", ctypes.c_int),
                ("n_kv_head", ctypes.c_int), ("head_dim", ctypes.c_int), ("vocab", ctypes.c_int), ("n_rot", ctypes.c_int),
                ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float), ("max_ctx", ctypes.c_int),
                ("tp_rank", ctypes.c_int), ("tp_size", ctypes.c_int), ("weight_type", ctypes.c_uint32),
                ("attn_interval", ctypes.c_int), ("ssm_d_inner", ctypes.c_int), ("ssm_d_state", ctypes.c_int),
                ("ssm_dt_rank", ctypes.c_int), ("ssm_n_group", ctypes.c_int), ("ssm_conv_kern", ctypes.c_int)]


class Partition(ctypes.Structure):
    _fields_ = [("q_lo", ctypes.c_int), ("n_q", ctypes.c_int), ("kv_lo", ctypes.c_int), ("n_kv", ctypes.c_int),
                ("f_lo", ctypes.c_int), ("n_f", ctypes.c_int), ("v_lo", ctypes.c_int), ("n_v", ctypes.c_int)]


QWEN27 = dict(n_layers=64, hidden=5120, ffn=17408, n_head=24, n_kv_head=4, head_dim=256, vocab=248320, n_rot=64,
              rope_theta=1e7, rms_eps=1e-6)
# the BASELINE cfg4 draft: a 0.6B-shaped q8_0 model (hidden 1024, FFN 3072,
# 28 layers; 16 query / 8 kv heads of 128, the target's vocabulary)
DRAFT = dict(n_layers=28, hidden=1024, ffn=3072, n_head=16, n_kv_head=8, head_dim=128, vocab=248320, n_rot=64,
             rope_theta=1e6, rms_eps=1e-6, weight_type=8)
# the reference's hybrid layout (include/mono27b_config.h:43-50; every 4th layer attention)
HYBRID = dict(attn_interval=4, ssm_d_inner=6144, ssm_d_state=128, ssm_dt_rank=48, ssm_n_group=16, ssm_conv_kern=4)


def model_config(max_ctx=1024, tp_rank=0, tp_size=1, **kw):
    d = dict(QWEN27)
    d.update(kw)
    return ModelConfig(max_ctx=max_ctx, tp_rank=tp_rank, tp_size=tp_size, **d)


def _engine_lib():
    L = lib()
    if getattr(L, "_engine_sigs", False):
        return L
    vp, cp, sz, i32, u32, b = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32, ctypes.c_bool
    sig = {
        "m27b_engine_partition": (b, [ctypes.POINTER(ModelConfig), ctypes.POINTER(Partition), cp, sz]),
        "m27b_nccl_unique_id": (b, [vp, cp, sz]),
        "m27b_engine_create": (b, [ctypes.POINTER(ModelConfig), ctypes.POINTER(vp), cp, sz]),
        "m27b_engine_set_nccl": (b, [vp, vp, cp, sz]),
        "m27b_engine_enable_p2p": (b, [vp, cp, sz]),
        "m27b_engine_load_tensor": (b, [vp, cp, u32, u32, u32, vp, cp, sz]),
        "m27b_engine_random_weights": (b, [vp, ctypes.c_uint64, ctypes.c_float, cp, sz]),
        "m27b_engine_weight_bytes_per_token": (sz, [vp]),
        "m27b_engine_reset": (b, [vp, cp, sz]),
        "m27b_engine_decode_step": (b, [vp, i32, i32, ctypes.POINTER(ctypes.c_int), vp, cp, sz]),
        "m27b_engine_generate": (b, [vp, i32, i32, i32, vp, cp, sz]),
        "m27b_engine_verify": (b, [vp, vp, i32, i32, vp, vp, cp, sz]),
        "m27b_engine_hidden": (b, [vp, vp, cp, sz]),
        "m27b_engine_stream": (vp, [vp]),
        "m27b_engine_destroy": (None, [vp]),
        "m27b_engine_create_sharing": (b, [vp, i32, ctypes.POINTER(vp), cp, sz]),
        "m27b_engine_speculative_generate": (b, [vp, vp, vp, i32, i32, i32, vp, ctypes.POINTER(SpecStats), cp, sz]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    L._engine_sigs = True
    return L


def partition(cfg):
    p = Partition()
    err = ctypes.create_string_buffer(ERR_CAP)
    _check(_engine_lib().m27b_engine_partition(ctypes.byref(cfg), ctypes.byref(p), err, ERR_CAP), err,
           "m27b_engine_partition")
    return p


def nccl_unique_id():
    buf = ctypes.create_string_buffer(128)
    err = ctypes.create_string_buffer(ERR_CAP)
    _check(_engine_lib().m27b_nccl_unique_id(buf, err, ERR_CAP), err, "m27b_nccl_unique_id")
    return buf.raw


class Engine:
    """One tensor-parallel rank of the decode engine on the current device."""

    def __init__(self, cfg):
        self.cfg = cfg
        self.L = _engine_lib()
        self.h = ctypes.c_void_p()
        self._call("m27b_engine_create", ctypes.byref(cfg), ctypes.byref(self.h))

    def _call(self, name, *args):
        err = ctypes.create_string_buffer(ERR_CAP)
        _check(getattr(self.L, name)(*args, err, ERR_CAP), err, name)

    def set_nccl(self, uid):
        buf = ctypes.create_string_buffer(bytes(uid), 128)
        self._call("m27b_engine_set_nccl", self.h, buf)

    def enable_p2p(self):
        """Fused NVLink all-reduce instead of NCCL (tp_size > 1; after set_nccl)."""
        self._call("m27b_engine_enable_p2p", self.h)

    def load_tensor(self, name, ggml_type, row_elems, row_count, data):
        import numpy as np
        a = np.ascontiguousarray(data)
        self._call("m27b_engine_load_tensor", self.h, name.encode(), ggml_type, row_elems, row_count,
                   ctypes.c_void_p(a.ctypes.data))

    def load_blob(self, blob, source=1):
        """Load a .m27b blob's entries of `source` (a Blob, or a path)."""
        b = blob if isinstance(blob, Blob) else Blob(blob)
        engine_load_blob(self, b, source)

    def random_weights(self, seed=0, sigma=0.02):
        self._call("m27b_engine_random_weights", self.h, seed, ctypes.c_float(sigma))

    def weight_bytes_per_token(self):
        return self.L.m27b_engine_weight_bytes_per_token(self.h)

    def decode_step(self, token, pos, logits=False):
        import numpy as np
        nxt = ctypes.c_int(-1)
        lg = np.empty(self.cfg.vocab, dtype=np.float32) if logits else None
        self._call("m27b_engine_decode_step", self.h, int(token), int(pos), ctypes.byref(nxt),
                   ctypes.c_void_p(lg.ctypes.data) if logits else None)
        return (nxt.value, lg) if logits else nxt.value

    def reset(self):
        """Start a new sequence: the DeltaNet states return to zero (attention needs nothing)."""
        self._call("m27b_engine_reset", self.h)

    def generate(self, token, pos, n):
        """Greedy tokens of steps pos..pos+n-1 (step i consumes step i-1's token), all on the device."""
        import numpy as np
        out = np.empty(n, dtype=np.int32)
        self._call("m27b_engine_generate", self.h, int(token), int(pos), int(n), ctypes.c_void_p(out.ctypes.data))
        return out

    def verify(self, tokens, pos, logits=False):
        """Greedy next token after each of `tokens` (at positions pos, pos+1, ...), one pass."""
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = np.empty(len(t), dtype=np.int32)
        lg = np.empty((len(t), self.cfg.vocab), dtype=np.float32) if logits else None
        self._call("m27b_engine_verify", self.h, ctypes.c_void_p(t.ctypes.data), len(t), int(pos),
                   ctypes.c_void_p(nxt.ctypes.data), ctypes.c_void_p(lg.ctypes.data) if logits else None)
        return (nxt, lg) if logits else nxt

    def stream(self):
        """The engine's cudaStream_t as an integer handle."""
        return self.L.m27b_engine_stream(self.h)

    def hidden(self):
        import numpy as np
        out = np.empty(self.cfg.hidden, dtype=np.float32)
        self._call("m27b_engine_hidden", self.h, ctypes.c_void_p(out.ctypes.data))
        return out

    def close(self):
        if self.h:
            self.L.m27b_engine_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# --------------------------------------------------------------------------
# .m27b blobs (include/m27b_blob.h)

SOURCE_TARGET, SOURCE_DRAFT = 1, 2
ROLE_NONE, ROLE_TARGET_MATVEC, ROLE_DRAFT_MATVEC, ROLE_OUTPUT_HEAD = 0, 1, 2, 3


class BlobHeader(ctypes.Structure):
    _fields_ = [("magic", ctypes.c_uint32), ("schema_version", ctypes.c_uint32), ("section_count", ctypes.c_uint32),
                ("reserved0", ctypes.c_uint32), ("file_bytes", ctypes.c_uint64), ("tensor_table_offset", ctypes.c_uint64),
                ("section_table_offset", ctypes.c_uint64), ("tokenizer_offset", ctypes.c_uint64),
                ("tokenizer_bytes", ctypes.c_uint64), ("max_ctx_hint", ctypes.c_uint32),
                ("target_layers", ctypes.c_uint32), ("draft_layers", ctypes.c_uint32), ("target_arch", ctypes.c_char * 16),
                ("draft_arch", ctypes.c_char * 16), ("target_quant", ctypes.c_char * 16),
                ("draft_quant", ctypes.c_char * 16)]


class WeightEntry(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 64), ("ggml_type", ctypes.c_uint32), ("source_model", ctypes.c_uint32),
                ("role", ctypes.c_uint32), ("row_elems", ctypes.c_uint32), ("row_count", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32), ("data_offset", ctypes.c_uint64), ("data_bytes", ctypes.c_uint64)]


class PackTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("ggml_type", ctypes.c_uint32), ("source", ctypes.c_uint32),
                ("role", ctypes.c_uint32), ("row_elems", ctypes.c_uint32), ("row_count", ctypes.c_uint32),
                ("data", ctypes.c_void_p), ("bytes", ctypes.c_uint64)]


class PackInfo(ctypes.Structure):
    _fields_ = [("max_ctx_hint", ctypes.c_uint32), ("target_layers", ctypes.c_uint32), ("draft_layers", ctypes.c_uint32),
                ("target_arch", ctypes.c_char_p), ("draft_arch", ctypes.c_char_p), ("target_quant", ctypes.c_char_p),
                ("draft_quant", ctypes.c_char_p), ("vocab_size", ctypes.c_uint32), ("bos_id", ctypes.c_uint32),
                ("eos_id", ctypes.c_uint32), ("im_start_id", ctypes.c_uint32), ("im_end_id", ctypes.c_uint32)]


def _blob_lib():
    L = lib()
    if getattr(L, "_blob_sigs", False):
        return L
    vp, cp, sz, b = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_bool
    L.m27b_blob_pack.restype = b
    L.m27b_blob_pack.argtypes = [cp, ctypes.POINTER(PackInfo), ctypes.POINTER(PackTensor), sz, cp, sz]
    L.m27b_blob_open.restype = b
    L.m27b_blob_open.argtypes = [cp, ctypes.POINTER(vp), cp, sz]
    L.m27b_blob_header.restype = ctypes.POINTER(BlobHeader)
    L.m27b_blob_header.argtypes = [vp]
    L.m27b_blob_count.restype = sz
    L.m27b_blob_count.argtypes = [vp]
    L.m27b_blob_entry.restype = b
    L.m27b_blob_entry.argtypes = [vp, sz, ctypes.POINTER(WeightEntry), ctypes.POINTER(vp), cp, sz]
    L.m27b_blob_close.restype = None
    L.m27b_blob_close.argtypes = [vp]
    L.m27b_engine_load_blob.restype = b
    L.m27b_engine_load_blob.argtypes = [vp, vp, ctypes.c_uint32, cp, sz]
    L._blob_sigs = True
    return L


def blob_pack(path, tensors, max_ctx_hint=8192, target_layers=0, draft_layers=0, target_arch="qwen35",
              draft_arch="dflash-draft", target_quant="q4_k_m", draft_quant="q8_0", vocab_size=1, bos_id=0, eos_id=0,
              im_start_id=0, im_end_id=0):
    """Write a .m27b blob.  tensors: iterable of dicts with name, ggml_type,
    data (numpy bytes in GGUF layout or fp32), row_elems, row_count and
    optionally source (default target) and role (default: output head for
    output.weight, target/draft matvec for quantized 2-D tensors, 0 otherwise)."""
    import numpy as np
    keep, arr = [], []
    for t in tensors:
        d = np.ascontiguousarray(t["data"])
        keep.append(d)
        src = t.get("source", SOURCE_TARGET)
        role = t.get("role")
        if role is None:
            if t["name"] == "output.weight":
                role = ROLE_OUTPUT_HEAD
            elif t["ggml_type"] != F32 and t["row_count"] > 1:
                role = ROLE_TARGET_MATVEC if src == SOURCE_TARGET else ROLE_DRAFT_MATVEC
            else:
                role = ROLE_NONE
        arr.append(PackTensor(t["name"].encode(), t["ggml_type"], src, role, t["row_elems"], t["row_count"],
                              ctypes.c_void_p(d.ctypes.data), d.nbytes))
    tarr = (PackTensor * len(arr))(*arr)
    info = PackInfo(max_ctx_hint, target_layers, draft_layers, target_arch.encode(), draft_arch.encode(),
                    target_quant.encode(), draft_quant.encode(), vocab_size, bos_id, eos_id, im_start_id, im_end_id)
    err = ctypes.create_string_buffer(ERR_CAP)
    _check(_blob_lib().m27b_blob_pack(str(path).encode(), ctypes.byref(info), tarr, len(arr), err, ERR_CAP), err,
           "m27b_blob_pack")


class Blob:
    """A mapped, validated .m27b blob."""

    def __init__(self, path):
        self.L = _blob_lib()
        self.h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(ERR_CAP)
        _check(self.L.m27b_blob_open(str(path).encode(), ctypes.byref(self.h), err, ERR_CAP), err, "m27b_blob_open")

    @property
    def header(self):
        return self.L.m27b_blob_header(self.h).contents

    def __len__(self):
        return self.L.m27b_blob_count(self.h)

    def entry(self, i):
        """(WeightEntry, payload as a read-only numpy uint8 view of the mapping)."""
        import numpy as np
        e = WeightEntry()
        p = ctypes.c_void_p()
        err = ctypes.create_string_buffer(ERR_CAP)
        _check(self.L.m27b_blob_entry(self.h, i, ctypes.byref(e), ctypes.byref(p), err, ERR_CAP), err,
               "m27b_blob_entry")
        buf = (ctypes.c_uint8 * e.data_bytes).from_address(p.value)
        return e, np.frombuffer(buf, dtype=np.uint8)

    def entries(self):
        return [self.entry(i) for i in range(len(self))]

    def close(self):
        if self.h:
            self.L.m27b_blob_close(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def engine_load_blob(engine, blob, source=SOURCE_TARGET):
    err = ctypes.create_string_buffer(ERR_CAP)
    _check(_blob_lib().m27b_engine_load_blob(engine.h, blob.h, source, err, ERR_CAP), err, "m27b_engine_load_blob")


# --------------------------------------------------------------------------
# speculative decoding (draft engine + target engine, greedy)


class SpecStats(ctypes.Structure):
    """M27BSpecStats (include/m27b_engine.h)."""
    _fields_ = [("iterations", ctypes.c_int), ("proposed", ctypes.c_int), ("accepted", ctypes.c_int),
                ("prefill_ms", ctypes.c_double), ("draft_ms", ctypes.c_double), ("verify_ms", ctypes.c_double)]


def speculative_generate(target, draft, prompt, n_new, k=7):
    """Greedy speculative decoding through m27b_engine_speculative_generate
    (the loop runs in the library): the draft proposes k tokens, the target
    verifies k + 1 in one pass and keeps the longest agreeing prefix plus its
    own next token.  Lossless: equals the target's greedy decoding of
    `prompt`.  Both engines must start empty; returns (tokens, stats)."""
    import numpy as np
    p = np.ascontiguousarray(prompt, dtype=np.int32)
    out = np.empty(n_new, dtype=np.int32)
    st = SpecStats()
    err = ctypes.create_string_buffer(ERR_CAP)
    _check(_engine_lib().m27b_engine_speculative_generate(target.h, draft.h, ctypes.c_void_p(p.ctypes.data), len(p),
                                                          int(n_new), int(k), ctypes.c_void_p(out.ctypes.data),
                                                          ctypes.byref(st), err, ERR_CAP),
           err, "m27b_engine_speculative_generate")
    stats = {f: getattr(st, f) for f, _ in SpecStats._fields_}
    return [int(t) for t in out], stats


M27B_VERIFY_MAX = 16
