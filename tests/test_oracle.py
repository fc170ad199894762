"""The CPU oracle pinned against golden vectors (CPU only).

The oracle restates ggml's q4_K / q5_K / q6_K / IQ4_XS / q8_0 / q8_K / f16
semantics; these tests pin it against gguf 0.19.0's dequantizers and q8_0
quantizer (committed fixtures), against the reference's own q4_K known-answer
values, and check its integer dot-product formulation against the pinned
dequantization.
"""
import os
import subprocess

import numpy as np
import pytest

import _data as D

F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, IQ4_XS = 0, 1, 8, 12, 13, 14, 15, 23


@pytest.mark.parametrize("name,qt", [("q4K", Q4_K), ("q6K", Q6_K), ("q80", Q8_0), ("q5K", Q5_K),
                                     ("iq4xs", IQ4_XS), ("f16", F16)])
def test_dequant_matches_gguf_bit_exact(orc, golden, name, qt):
    k = int(golden[name + "_k"])
    got = orc.dequantize(qt, golden[name + "_raw"], k)
    want = golden[name + "_deq"]
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q8_0_quantize_matches_gguf_bit_exact(orc, golden):
    got = orc.quantize_q8_0(golden["q80_x"])
    assert np.array_equal(got, golden["q80_q"])


def test_q4K_known_answer_from_reference(orc, golden):
    block = np.zeros(144, dtype=np.uint8)
    block[:32] = golden["kat_block"]  # d, dmin, scales[12], qs[0..15]
    out = orc.dequantize(Q4_K, block, 256)[0]
    # printed with 9 significant digits, which round-trips a float32 exactly
    want = golden["kat_values"].astype(np.float32)
    assert np.array_equal(out[:16], want)


def test_reference_kat_binary_agrees(orc):
    """The reference's own official_dequant.c, built from source, prints the same values."""
    from oracle import build as ob
    exe = ob.build_reference_kat()
    if not exe or not os.path.exists(exe):
        pytest.skip("reference KAT program not built (reference checkout absent)")
    vals = np.array([float(v) for v in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()])
    block = np.zeros(144, dtype=np.uint8)
    block[:32] = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))["kat_block"]
    out = orc.dequantize(Q4_K, block, 256)[0][:8]
    assert np.array_equal(out, vals.astype(np.float32))


def test_fp16_conversions_round_trip(orc):
    for h in list(range(0, 0x7c00, 97)) + [0x0001, 0x03ff, 0x0400, 0x7bff, 0x8001, 0xfbff]:
        f = orc.fp16_to_fp32(h)
        assert f == np.float32(np.uint16(h).view(np.float16))
        assert orc.fp32_to_fp16(f) == h
    rng = np.random.default_rng(5)
    xs = np.concatenate([rng.standard_normal(4000) * s for s in (1e-7, 1e-5, 1e-2, 1, 100, 6e4)]).astype(np.float32)
    for x in xs:
        assert orc.fp32_to_fp16(float(x)) == int(np.float16(x).view(np.uint16)), x


def _q8K_fields(raw):
    b = raw.reshape(-1, 292)
    d = b[:, 0:4].copy().view(np.float32).ravel()
    qs = b[:, 4:260].view(np.int8)
    bs = b[:, 260:292].copy().view(np.int16)
    return d, qs, bs


def test_q8_K_quantizer_rules(orc):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((3, 512)).astype(np.float32)
    x[1, 256:] = 0.0                      # all-zero block
    x[2, 10] = -5.0                        # negative maximum, and a tie of equal magnitude later
    x[2, 20] = 5.0
    q = orc.quantize_q8_K(x)
    for t in range(3):
        d, qs, bs = _q8K_fields(q[t])
        for b in range(2):
            xb = x[t, 256 * b:256 * (b + 1)]
            if not np.any(xb):
                assert d[b] == 0 and not qs[b].any() and not bs[b].any()
                continue
            i = int(np.argmax(np.abs(xb)))  # first index of largest magnitude
            iscale = np.float32(-127.0) / xb[i]
            want = np.minimum(127, np.rint(iscale * xb)).astype(np.int8)
            assert np.array_equal(qs[b], want)
            assert d[b] == np.float32(1.0) / iscale
            assert np.array_equal(bs[b], qs[b].astype(np.int32).reshape(16, 16).sum(1))
    d, qs, _ = _q8K_fields(q[2])
    assert d[0] > 0 and qs[0][10] == -127 and qs[0][20] == 127  # first maximum (-5) sets the sign


@pytest.mark.parametrize("qt,k", [(Q4_K, 1024), (Q6_K, 1024), (Q8_0, 512), (Q5_K, 1024), (IQ4_XS, 1024),
                                  (F16, 200), (F32, 200)])
def test_vec_dot_equals_dequantized_dot(orc, qt, k):
    """The integer vec_dot equals sum(dequant(W) * dequant(x)) up to fp32 rounding
    (f16: x rounded to fp16 first, as ggml converts it to the weight's type)."""
    rng = np.random.default_rng(7)
    w = orc.quantize_weights(qt, (rng.standard_normal((16, k)) * 0.02).astype(np.float32))
    x = rng.standard_normal((2, k)).astype(np.float32)
    xq = orc.quantize_act(qt, x)
    y = orc.matvec(qt, w, k, xq)
    wd = orc.dequantize(qt, w, k).astype(np.float64)
    if qt in (F16, F32):
        xd = (x.astype(np.float16) if qt == F16 else x).astype(np.float64)
    elif qt == Q8_0:
        xb = xq.reshape(2, -1, 34)
        xd = (xb[:, :, 2:].view(np.int8).astype(np.float64) *
              xb[:, :, 0:2].copy().view(np.float16).astype(np.float64)).reshape(2, k)
    else:
        xd = []
        for t in range(2):
            d, qs, _ = _q8K_fields(xq[t])
            xd.append((qs.astype(np.float64) * d[:, None].astype(np.float64)).ravel())
        xd = np.array(xd)
    ref = xd @ wd.T
    assert orc.rel_l2(y, ref) < 1e-6


def test_weight_quantizers_are_accurate(orc):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((32, 512)) * 0.02).astype(np.float32)
    for qt, tol in ((Q4_K, 0.09), (Q5_K, 0.045), (Q6_K, 0.025), (IQ4_XS, 0.11), (Q8_0, 0.008), (F16, 5e-4)):
        w = orc.quantize_weights(qt, x)
        assert orc.rel_l2(orc.dequantize(qt, w, 512), x) < tol


def test_matvec_threads_do_not_change_results(orc):
    rng = np.random.default_rng(9)
    w = orc.quantize_weights(Q4_K, (rng.standard_normal((64, 512)) * 0.02).astype(np.float32))
    xq = orc.quantize_q8_K(rng.standard_normal((1, 512)).astype(np.float32))
    a = orc.matvec(Q4_K, w, 512, xq, nthreads=1)
    b = orc.matvec(Q4_K, w, 512, xq, nthreads=4)
    assert np.array_equal(a, b)


def test_iq4_xs_codebook_and_scale_fields(orc):
    """IQ4_XS field layout: ls = 4 bits of scales_l | 2 bits of scales_h, the
    multiplier ls - 32, low nibbles the first 16 values of a sub-block."""
    blk = np.zeros(136, np.uint8)
    blk[0:2] = np.array([1.0], np.float16).view(np.uint8)
    # sub-block 0: ls = 0x21 (33 -> multiplier 1); sub-block 1: ls = 0x1e (30 -> -2)
    blk[4] = 0x1 | (0xe << 4)
    blk[2:4] = np.array([0x2 | (0x1 << 2)], np.uint16).view(np.uint8)
    blk[8] = 0x0 | (0xf << 4)    # sub-block 0, element 0: code 0; element 16: code 15
    blk[8 + 16] = 0x8            # sub-block 1, element 0: code 8
    v = orc.dequantize(IQ4_XS, blk[None], 256)[0]
    assert v[0] == -127 and v[16] == 113 and v[1] == -127
    assert v[32] == -2 * 1 and v[33] == -2 * -127
    assert np.all(v[64:] == -32 * -127)  # stored ls 0: multiplier -32, code 0: codebook -127


def test_simd_q4K_matvec_equals_scalar_oracle(orc):
    """The vectorised q4_K . q8_K (the timed CPU baseline) gives the scalar
    oracle's results bit for bit, at every instruction-set level this CPU has
    (extreme codes and scales included)."""
    rng = np.random.default_rng(21)
    for rows, k, ntok in ((37, 256, 1), (300, 5120, 3), (64, 17408, 2)):
        w = D.random_valid_blocks(orc.Q4_K, rows, k, 5 + rows)
        wb = w.reshape(rows, -1, 144)
        wb[0, :, 4:16] = 0xff          # every 6-bit scale and min at 63
        wb[1, :, 16:] = 0xff           # every code at 15
        x = (rng.standard_normal((ntok, k)) * 3).astype(np.float32)
        x[0, :256] = 127.0             # saturating activation codes
        xq = orc.quantize_q8_K(x)
        want = orc.matvec(orc.Q4_K, w, k, xq)
        for level in range(orc.simd_level() + 1):
            got, used = orc.matvec_q4K_simd(w, k, xq, level=level)
            assert used == level
            assert np.array_equal(got, want), (rows, k, level)
