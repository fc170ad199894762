"""m27b_attn_decode_noalloc (split partials in the library's static device
scratch, no allocation) against m27b_attn_decode (caller-provided scratch).

Same kernels and same arithmetic, so the outputs agree to the test tolerance
(rtol 1e-6); two calls in a row with different shapes reuse the one scratch.
Runs alone in a fresh process or after the other tests (no shared state
besides the library's own per-device set-up)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-6, 1e-7


def _inputs(torch, seed, nq, nkv, hd, L):
    rng = np.random.default_rng(seed)
    ctx = L + 1
    t = lambda a: torch.from_numpy(a.astype(np.float32)).to("cuda")
    q = t(rng.standard_normal((nq, hd)))
    K = t(rng.standard_normal((ctx, nkv, hd)))
    V = t(rng.standard_normal((ctx, nkv, hd)))
    pos = torch.tensor([L - 1], dtype=torch.int32, device="cuda")
    return q, K, V, pos


def test_noalloc_matches_caller_scratch_two_calls(torch, m27b):
    # the single-GPU Qwen-27B shape needs 923,520 bytes of partials, within the static scratch
    assert m27b.attn_part_bytes(24, 256, 37) == 923520 <= m27b.attn_noalloc_scratch_bytes()
    shapes = [(24, 4, 256, 700, 37),
              (8, 2, 128, 65, 16)]
    for seed, (nq, nkv, hd, L, splits) in enumerate(shapes):
        q, K, V, pos = _inputs(torch, seed, nq, nkv, hd, L)
        scale = 1.0 / np.sqrt(hd)
        part = torch.empty(m27b.attn_part_bytes(nq, hd, splits), dtype=torch.uint8, device="cuda")
        want = torch.empty((nq, hd), dtype=torch.float32, device="cuda")
        got = torch.full((nq, hd), float("nan"), dtype=torch.float32, device="cuda")
        m27b.attn_decode(q, K, V, pos, nq, nkv, hd, splits, scale, part, want)
        m27b.attn_decode_noalloc(q, K, V, pos, nq, nkv, hd, splits, scale, got)
        torch.cuda.synchronize()
        assert torch.allclose(got, want, rtol=RTOL, atol=ATOL), (nq, hd, L)


def test_noalloc_rejects_oversized(torch, m27b):
    q, K, V, pos = _inputs(torch, 9, 64, 8, 256, 40)
    out = torch.empty((64, 256), dtype=torch.float32, device="cuda")
    assert m27b.attn_part_bytes(64, 256, 16) > m27b.attn_noalloc_scratch_bytes()
    with pytest.raises(m27b.M27BError, match="static scratch holds"):
        m27b.attn_decode_noalloc(q, K, V, pos, 64, 8, 256, 16, 0.0625, out)
