"""Seeded synthetic inputs with the shapes and distributions of the benchmark
configs (test helper).  The reference benchmarks no public dataset; weights are
N(0, sigma^2) quantized with the oracle's restatement of ggml's quantizers, or
seeded random valid blocks where Gaussian quantization of the full tensor is
too slow for a test (stated where used).
"""
import numpy as np

Q8_0, Q4_K, Q6_K, Q8_K = 8, 12, 14, 15


def gauss_weights(orc, qtype, rows, k, seed, sigma=0.02, chunk=2048):
    """rows x k fp32 N(0, sigma^2) from default_rng(seed), quantized to qtype.
    Chunked generation draws the same stream as one (rows, k) draw."""
    rng = np.random.default_rng(seed)
    out = np.empty((rows, orc.row_bytes(qtype, k)), dtype=np.uint8)
    for r0 in range(0, rows, chunk):
        n = min(chunk, rows - r0)
        x = (rng.standard_normal((n, k)) * sigma).astype(np.float32)
        out[r0:r0 + n] = orc.quantize_weights(qtype, x)
    return out


def _fp16_bits(v):
    return np.asarray(v, dtype=np.float16).view(np.uint16).view(np.uint8).reshape(-1, 2)


def random_valid_blocks(qtype, rows, k, seed, sigma=0.02):
    """Seeded random GGUF blocks whose fp16 scales give values of std ~sigma."""
    rng = np.random.default_rng(seed)
    if qtype == Q4_K:
        nb = rows * k // 256
        b = np.frombuffer(rng.bytes(nb * 144), dtype=np.uint8).reshape(nb, 144).copy()
        # |d*sc*q - dmin*m| with sc,m ~ U[0,63], q ~ U[0,15]
        b[:, 0:2] = _fp16_bits(rng.uniform(0.5, 1.5, nb) * sigma / 250.0)
        b[:, 2:4] = _fp16_bits(rng.uniform(0.5, 1.5, nb) * sigma / 120.0)
    elif qtype == Q6_K:
        nb = rows * k // 256
        b = np.frombuffer(rng.bytes(nb * 210), dtype=np.uint8).reshape(nb, 210).copy()
        b[:, 208:210] = _fp16_bits(rng.uniform(0.5, 1.5, nb) * sigma / 1300.0)
    else:
        nb = rows * k // 32
        b = np.frombuffer(rng.bytes(nb * 34), dtype=np.uint8).reshape(nb, 34).copy()
        b[:, 0:2] = _fp16_bits(rng.uniform(0.5, 1.5, nb) * sigma / 74.0)
    return b.reshape(rows, -1)


def gauss_act(n, k, seed, sigma=1.0):
    return (np.random.default_rng(seed).standard_normal((n, k)) * sigma).astype(np.float32)
