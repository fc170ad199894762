"""q4_K x 5..16 tokens on the tensor cores (tcgen05.mma kind::i8, TMEM
accumulators; csrc/qmv_q4k_mma.cu) against the oracle's ggml
vec_dot_q4_K_q8_K.

The integer sums are ggml's exactly (the two 8-bit scale planes recombine to
sum_s sc_s * dot_s); only the fp32 accumulation order differs, so the tight
tolerance of the dp4a kernels applies.  Shapes cover a partial last 128-row
tile, a tile smaller than 128 rows, more tiles than SMs (the persistent tile
loop), K of 1..24 super-blocks, every token count 5..16 (MMA N = 8 and 16,
padded token columns), the residual epilogue and rows read in place.  Every
run also checks the device status word: a pipeline hand-off that stalls shows
up there (a bounded wait that ran out) even when the sums come out right.  A
long chain of back-to-back launches at the decode engine's shapes exercises
the hand-offs under every warp timing the scheduler produces."""
import numpy as np
import pytest

import _data as D

pytestmark = pytest.mark.gpu

Q4_K, Q8_K = 12, 15
TIGHT = 2e-5


def _run(torch, orc, m27b, rows, k, n, seed, residual=False):
    w = D.gauss_weights(orc, Q4_K, rows, k, seed)
    x = D.gauss_act(n, k, seed + 1)
    xq_cpu = orc.quantize_q8_K(x)
    want = orc.matvec(Q4_K, w, k, xq_cpu)
    W = m27b.QWeight(w, Q4_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(x).cuda(), Q8_K)
    y = torch.full((n, rows), float("nan"), device="cuda")
    res = None
    if residual:
        r = D.gauss_act(n, rows, seed + 2)
        want = want + r
        res = torch.from_numpy(r).cuda()
    m27b.qmv(W, xq, n, y, residual=res)
    got = y.cpu().numpy()
    assert m27b.device_status() == 0  # no bounded wait of the pipeline ran out
    return orc.rel_l2(got, want)


@pytest.mark.parametrize("n", list(range(5, 17)))
def test_mma_tokens(torch, orc, m27b, n):
    assert _run(torch, orc, m27b, 300, 1280, n, 100 + n) <= TIGHT


@pytest.mark.parametrize("rows,k", [(1, 256), (77, 256), (128, 512), (256, 5120), (129, 6144), (19021, 256)])
@pytest.mark.parametrize("n", [5, 8, 16])
def test_mma_shapes(torch, orc, m27b, rows, k, n):
    assert _run(torch, orc, m27b, rows, k, n, rows + k + n) <= TIGHT


def test_mma_residual(torch, orc, m27b):
    assert _run(torch, orc, m27b, 500, 2048, 12, 7, residual=True) <= TIGHT


def test_mma_matches_single_token_kernel(torch, orc, m27b):
    # the tensor-core path (16 tokens) and the dp4a path (one token at a time)
    # compute the same integer sums: per-token results agree closely
    rows, k, n = 1000, 5120, 16
    w = D.gauss_weights(orc, Q4_K, rows, k, 9)
    x = D.gauss_act(n, k, 10)
    W = m27b.QWeight(w, Q4_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(x).cuda(), Q8_K)
    y16 = torch.empty((n, rows), device="cuda")
    m27b.qmv(W, xq, n, y16)
    nb = m27b.act_bytes(Q8_K, k)
    y1 = torch.empty((n, rows), device="cuda")
    for t in range(n):
        m27b.qmv(W, xq[t * nb:(t + 1) * nb], 1, y1[t:t + 1])
    assert orc.rel_l2(y16.cpu().numpy(), y1.cpu().numpy()) <= 1e-6


@pytest.mark.parametrize("n", [8, 16])
def test_mma_chain_of_launches(torch, orc, m27b, n):
    # 400 launches back to back (each overlapping its neighbours through
    # programmatic dependent launch) at o_proj's shape: same result every
    # time, no stalled hand-off
    rows, k = 5120, 6144
    w = D.gauss_weights(orc, Q4_K, rows, k, 21)
    x = D.gauss_act(n, k, 22)
    want = orc.matvec(Q4_K, w, k, orc.quantize_q8_K(x))
    W = m27b.QWeight(w, Q4_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(x).cuda(), Q8_K)
    ys = [torch.empty((n, rows), device="cuda") for _ in range(2)]
    m27b.qmv(W, xq, n, ys[0])
    first = ys[0].clone()
    for i in range(400):
        m27b.qmv(W, xq, n, ys[i & 1])
    torch.cuda.synchronize()
    assert m27b.device_status() == 0
    assert torch.equal(ys[0], first) and torch.equal(ys[1], first)
    assert orc.rel_l2(first.cpu().numpy(), want) <= TIGHT
