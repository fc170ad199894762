"""Generate the committed golden fixtures that pin the CPU oracle.

Run in a container that has the gguf package (llama.cpp's gguf-py, 0.19.0
here) and the reference checkout; the output ``golden.npz`` is committed, so
the tests never need either at run time.

Contents
--------
* ``{q4K,q6K,q80}_raw`` / ``..._deq``: seeded random GGUF blocks (fp16 scale
  fields forced to finite, moderate values) and their dequantization by
  ``gguf.quants.dequantize`` — llama.cpp's own numpy restatement of
  dequantize_row_q4_K / q6_K / q8_0.
* ``{q5K,iq4xs,f16}_raw`` / ``..._deq``: the same for q5_K, IQ4_XS and f16
  (a second seeded generator, so the first fixtures keep their bytes).
* ``q80_x`` / ``q80_q``: fp32 rows and their q8_0 quantization by
  ``gguf.quants.quantize`` (which gguf-py documents as matching ggml's
  quantize_row_q8_0 bit for bit).
* ``kat_block`` / ``kat_values``: the reference's q4_K known-answer test — the
  32-byte block prefix written in debug/official_dequant.c:70-74 and the 16
  dequantized values the reference recorded for token 44883's embedding row
  in debug/mono_give_current.debug.tsv:2 (the first 8 are also what
  official_dequant prints).  Both are read from the reference files as text.
"""
import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# the reference checkout: M27B_REFERENCE_ROOT, else "reference" beside this repository
REF = os.environ.get("M27B_REFERENCE_ROOT") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))), "reference")


def fp16_bits(rng, n, lo, hi):
    v = rng.uniform(lo, hi, n).astype(np.float16)
    v *= np.where(rng.random(n) < 0.5, -1, 1).astype(np.float16)
    return v.view(np.uint16)


def random_blocks(rng, qtype, nblocks):
    from gguf import GGMLQuantizationType as T
    if qtype == T.Q4_K:
        b = rng.integers(0, 256, (nblocks, 144), dtype=np.uint8)
        b[:, 0:2] = np.abs(fp16_bits(rng, nblocks, 1e-4, 2e-2).view(np.float16)).view(np.uint16).view(np.uint8).reshape(-1, 2)
        b[:, 2:4] = np.abs(fp16_bits(rng, nblocks, 1e-4, 2e-2).view(np.float16)).view(np.uint16).view(np.uint8).reshape(-1, 2)
    elif qtype == T.Q6_K:
        b = rng.integers(0, 256, (nblocks, 210), dtype=np.uint8)
        b[:, 208:210] = fp16_bits(rng, nblocks, 1e-5, 1e-3).view(np.uint8).reshape(-1, 2)
    elif qtype == T.Q5_K:
        b = rng.integers(0, 256, (nblocks, 176), dtype=np.uint8)
        b[:, 0:2] = np.abs(fp16_bits(rng, nblocks, 1e-4, 2e-2).view(np.float16)).view(np.uint16).view(np.uint8).reshape(-1, 2)
        b[:, 2:4] = np.abs(fp16_bits(rng, nblocks, 1e-4, 2e-2).view(np.float16)).view(np.uint16).view(np.uint8).reshape(-1, 2)
    elif qtype == T.IQ4_XS:
        b = rng.integers(0, 256, (nblocks, 136), dtype=np.uint8)
        b[:, 0:2] = fp16_bits(rng, nblocks, 1e-5, 1e-3).view(np.uint8).reshape(-1, 2)
    elif qtype == T.F16:
        b = fp16_bits(rng, nblocks, 0.0, 4.0).view(np.uint8).reshape(nblocks, 2)
    else:
        b = rng.integers(0, 256, (nblocks, 34), dtype=np.uint8)
        b[:, 0:2] = fp16_bits(rng, nblocks, 1e-4, 1e-1).view(np.uint8).reshape(-1, 2)
    return b


def kat_from_reference():
    src = open(os.path.join(REF, "debug", "official_dequant.c")).read()
    body = re.search(r"uint8_t bytes\[\]\s*=\s*\{(.*?)\};", src, re.S).group(1)
    block = np.array([int(h, 16) for h in re.findall(r"0x([0-9a-fA-F]{2})", body)], dtype=np.uint8)
    assert block.size == 32
    with open(os.path.join(REF, "debug", "mono_give_current.debug.tsv")) as f:
        header = f.readline().rstrip("\n").split("\t")
        row = f.readline().rstrip("\n").split("\t")
    rec = dict(zip(header, row))
    assert rec["phase"] == "embed" and rec["label"] == "h"
    vals = np.array([float(v) for v in rec["values"].split(",")], dtype=np.float64)
    return block, vals


def main():
    import gguf
    from gguf import GGMLQuantizationType as T
    rng = np.random.default_rng(20251201)
    out = {}
    for name, qt, k in (("q4K", T.Q4_K, 512), ("q6K", T.Q6_K, 512), ("q80", T.Q8_0, 256)):
        be = 256 if qt != T.Q8_0 else 32
        rows = 6
        raw = random_blocks(rng, qt, rows * k // be).reshape(rows, -1)
        deq = gguf.quants.dequantize(raw, qt).reshape(rows, k).astype(np.float32)
        out[name + "_raw"] = raw
        out[name + "_deq"] = deq
        out[name + "_k"] = np.int64(k)
    rng2 = np.random.default_rng(20251202)
    for name, qt, k, be in (("q5K", T.Q5_K, 512, 256), ("iq4xs", T.IQ4_XS, 512, 256), ("f16", T.F16, 96, 1)):
        rows = 6
        raw = random_blocks(rng2, qt, rows * k // be).reshape(rows, -1)
        deq = gguf.quants.dequantize(raw, qt).reshape(rows, k).astype(np.float32)
        out[name + "_raw"] = raw
        out[name + "_deq"] = deq
        out[name + "_k"] = np.int64(k)
    x = (rng.standard_normal((4, 256)) * np.array([[1.0], [0.02], [100.0], [1e-30]])).astype(np.float32)
    x[3, :32] = 0.0  # an all-zero q8_0 block
    x[0, 40] = x[0, 32:64].max()  # duplicate the block maximum: an amax tie
    out["q80_x"] = x
    out["q80_q"] = gguf.quants.quantize(x, T.Q8_0).reshape(4, -1)
    blk, vals = kat_from_reference()
    out["kat_block"] = blk
    out["kat_values"] = vals
    out["gguf_version"] = np.array(gguf.__dict__.get("__version__", "0.19.0"))
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote", os.path.join(HERE, "golden.npz"), sorted(out))


if __name__ == "__main__":
    sys.exit(main())
