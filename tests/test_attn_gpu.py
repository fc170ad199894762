"""Decode attention (m27b_attn_decode) against a float64 numpy reference.

The kernel accumulates in fp32 with max-subtracted exponentials; compared at
rel-L2 <= 1e-5 per head."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def attn_ref(q, K, V, L, n_kv, scale):
    nq, hd = q.shape
    G = nq // n_kv
    out = np.empty((nq, hd))
    for h in range(nq):
        j = h // G
        s = (K[:L, j].astype(np.float64) @ q[h].astype(np.float64)) * scale
        w = np.exp(s - s.max())
        out[h] = w @ V[:L, j].astype(np.float64) / w.sum()
    return out


CASES = [  # n_q, n_kv, head_dim, L, splits
    (24, 4, 256, 1, 37), (24, 4, 256, 17, 37), (24, 4, 256, 700, 37), (24, 4, 256, 700, 1),
    (3, 1, 256, 513, 148), (12, 2, 256, 64, 74), (8, 2, 128, 300, 16), (8, 1, 64, 33, 8), (2, 2, 32, 5, 3),
    (6, 2, 96, 100, 10), (16, 2, 224, 257, 20),
]


@pytest.mark.parametrize("nq,nkv,hd,L,splits", CASES)
def test_attn_decode(torch, m27b, orc, nq, nkv, hd, L, splits):
    rng = np.random.default_rng(nq * 1000 + hd + L)
    ctx = L + 3
    q = rng.standard_normal((nq, hd)).astype(np.float32)
    K = rng.standard_normal((ctx, nkv, hd)).astype(np.float32)
    V = rng.standard_normal((ctx, nkv, hd)).astype(np.float32)
    dev = "cuda"
    t = lambda a: torch.from_numpy(a).to(dev)
    pos = torch.tensor([L - 1], dtype=torch.int32, device=dev)
    part = torch.empty(m27b.attn_part_bytes(nq, hd, splits), dtype=torch.uint8, device=dev)
    out = torch.empty((nq, hd), dtype=torch.float32, device=dev)
    scale = 1.0 / np.sqrt(hd)
    m27b.attn_decode(t(q), t(K), t(V), pos, nq, nkv, hd, splits, scale, part, out)
    got = out.cpu().numpy()
    want = attn_ref(q, K, V, L, nkv, scale)
    for h in range(nq):
        assert orc.rel_l2(got[h], want[h]) <= 1e-5, h


def test_attn_decode_validation(torch, m27b):
    z = torch.zeros(4096, dtype=torch.float32, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    for args, msg in [((24, 4, 250, 8), "head_dim"), ((24, 5, 256, 8), "multiple of n_kv"), ((18, 2, 256, 8), "at most 8"),
                      ((24, 4, 256, 0), "splits")]:
        with pytest.raises(m27b.M27BError, match=msg):
            m27b.attn_decode(z, z, z, pos, *args, 1.0, z, z)
