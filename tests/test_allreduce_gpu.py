"""The fused all-reduce's consumer on one GPU, through the C ABI
(m27b_allreduce_norm_quant, include/m27b_allreduce.h).

* Parity: the words of 1..8 source ranks carrying the awaited epoch are summed
  in rank order (bit-exact against numpy's fp32 sum in the same order) and
  RMSNorm + q8_K'd like m27b_act_quant_rmsnorm (same codes up to the last
  ulp of the norm: codes within 1, block scales within 1e-6).
* Error path: words whose epoch never arrives make every wait give up after
  the caller's short limit; the kernel returns, the launch reports status 3
  in the device status word, and the next call on the same device works.
  No GPU fault is involved: the wait is a bounded poll of ordinary memory.
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q8_K = 15


def _words(vals, ep):
    bits = vals.astype(np.float32).view(np.uint32).astype(np.uint64)
    return (bits | (np.uint64(ep) << np.uint64(32))).view(np.int64)


def _setup(torch, nsrc, k, seed, ep_words):
    rng = np.random.default_rng(seed)
    parts = (rng.standard_normal((nsrc, k)) * 0.5).astype(np.float32)
    words = torch.from_numpy(np.stack([_words(p, ep_words) for p in parts])).cuda()
    return parts, words


@pytest.mark.parametrize("nsrc,k", [(1, 256), (2, 5120), (3, 5120), (8, 17408)])
def test_consumer_sums_in_rank_order_and_quantizes(torch, m27b, nsrc, k):
    ep = 7 + nsrc
    parts, words = _setup(torch, nsrc, k, 40 + nsrc, ep)
    ss = torch.zeros(k // 256, dtype=torch.int64, device="cuda")
    epoch = torch.tensor([ep], dtype=torch.int32, device="cuda")
    norm_w = torch.from_numpy(np.random.default_rng(3).uniform(0.5, 1.5, k).astype(np.float32)).cuda()
    x_out = torch.empty(k, dtype=torch.float32, device="cuda")
    xq = torch.empty(m27b.act_bytes(Q8_K, k), dtype=torch.uint8, device="cuda")
    m27b.allreduce_norm_quant(words, nsrc, k, ss, epoch, k, x_out, xq, norm_w=norm_w, eps=1e-6, wait_ns=50_000_000)
    torch.cuda.synchronize()
    assert m27b.device_status() == 0
    want = parts[0].copy()
    for s in range(1, nsrc):
        want = (want + parts[s]).astype(np.float32)
    assert np.array_equal(x_out.cpu().numpy(), want)
    ref = m27b.act_quant(x_out.reshape(1, -1), Q8_K, norm_w=norm_w, eps=1e-6)
    got, exp = xq.cpu().numpy().reshape(-1, 292), ref.cpu().numpy().reshape(-1, 292)
    d_got, d_exp = got[:, :4].copy().view(np.float32), exp[:, :4].copy().view(np.float32)
    assert np.allclose(d_got, d_exp, rtol=1e-6, atol=0)
    q_got, q_exp = got[:, 4:260].view(np.int8).astype(int), exp[:, 4:260].view(np.int8).astype(int)
    assert np.abs(q_got - q_exp).max() <= 1
    assert (q_got == q_exp).mean() >= 0.999


def test_consumer_wait_runs_out_cleanly(torch, m27b):
    """Epoch 5 is awaited, the words carry epoch 4: every wait gives up after
    the 5 ms limit, status 3 is recorded, and the kernel returns."""
    k, nsrc = 5120, 2
    m27b.device_status(clear=True)
    _, words = _setup(torch, nsrc, k, 9, 4)
    ss = torch.zeros(k // 256, dtype=torch.int64, device="cuda")
    epoch = torch.tensor([5], dtype=torch.int32, device="cuda")
    x_out = torch.empty(k, dtype=torch.float32, device="cuda")
    xq = torch.empty(m27b.act_bytes(Q8_K, k), dtype=torch.uint8, device="cuda")
    t0 = time.perf_counter()
    m27b.allreduce_norm_quant(words, nsrc, k, ss, epoch, k, x_out, xq, wait_ns=5_000_000)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.5, "the short wait limit was not applied"
    assert m27b.device_status(clear=True) == 3
    assert m27b.device_status() == 0
    # the context stays usable: a following call with the right epoch succeeds
    epoch.fill_(4)
    ss.zero_()
    m27b.allreduce_norm_quant(words, nsrc, k, ss, epoch, k, x_out, xq, wait_ns=50_000_000)
    torch.cuda.synchronize()
    assert m27b.device_status() == 0


def test_consumer_rejects_bad_arguments(torch, m27b):
    k = 512
    w = torch.zeros((2, k), dtype=torch.int64, device="cuda")
    ss = torch.zeros(2, dtype=torch.int64, device="cuda")
    ep = torch.zeros(1, dtype=torch.int32, device="cuda")
    x = torch.empty(k, device="cuda")
    xq = torch.empty(m27b.act_bytes(Q8_K, k), dtype=torch.uint8, device="cuda")
    with pytest.raises(m27b.M27BError, match="nsrc"):
        m27b.allreduce_norm_quant(w, 9, k, ss, ep, k, x, xq)
    with pytest.raises(m27b.M27BError, match="multiple of 256"):
        m27b.allreduce_norm_quant(w, 2, k, ss, ep, 300, x, xq)
    with pytest.raises(m27b.M27BError, match="src_stride"):
        m27b.allreduce_norm_quant(w, 2, 256, ss, ep, k, x, xq)
