"""q4_K x 5..16 tokens on the tensor cores with each 128-row tile's K
dimension split across CTAs (m27b_qmv_mma_split, the verify pass's q4_K
projections) through the C ABI:
  * against the oracle (ggml vec_dot_q4_K_q8_K) on Gaussian-quantized
    weights: rel. L2 <= 1e-3 and <= 2e-5 (same
    integer sums; only the fp32 order of the ranges' partials differs);
  * at the verify pass's shapes (qkv 14336 x 5120, gate/up 17408 x 5120:
    2 ranges; o_proj 5120 x 6144: 6 ranges) against the one-unit-per-tile
    launch of m27b_qmv on random valid blocks: <= 2e-5, with and without
    the residual;
  * ragged shapes (a partial last tile, rows < 128, token counts 5..16 with
    padded MMA columns), deterministic results, the arrival counters back
    at zero, and the device status word clean (a stalled hand-off shows up
    there)."""
import numpy as np
import pytest

import _data as D

pytestmark = pytest.mark.gpu

Q4_K, Q8_K = 12, 15
TOL, TIGHT = 1e-3, 2e-5


@pytest.mark.parametrize("rows,k,n", [(1000, 4096, 7), (333, 6144, 8), (77, 5120, 5), (2048, 5120, 12),
                                      (17408, 5120, 8)])
def test_split_against_oracle(torch, orc, m27b, rows, k, n):
    w = D.gauss_weights(orc, Q4_K, rows, k, rows + n)
    x = D.gauss_act(n, k, 5 + n)
    want = orc.matvec(Q4_K, w, k, orc.quantize_q8_K(x))
    W = m27b.QWeight(w, Q4_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(x).cuda(), Q8_K)
    y = torch.full((n, rows), float("nan"), device="cuda")
    m27b.qmv_mma_split(W, xq, n, y)
    torch.cuda.synchronize()
    err = orc.rel_l2(y.cpu().numpy(), want)
    assert err <= TOL and err <= TIGHT, err
    assert m27b.device_status() == 0


@pytest.mark.parametrize("rows,k,n,residual", [(14336, 5120, 8, False), (17408, 5120, 8, False),
                                               (5120, 6144, 8, True), (17408, 5120, 16, False),
                                               (5120, 6144, 5, True)])
def test_split_verify_shapes_match_one_unit_launch(torch, m27b, rows, k, n, residual):
    W = m27b.QWeight(D.random_valid_blocks(Q4_K, rows, k, rows + n), Q4_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(D.gauss_act(n, k, 31)).cuda(), Q8_K)
    res = torch.from_numpy(D.gauss_act(n, rows, 32)).cuda() if residual else None
    want = torch.empty((n, rows), device="cuda")
    m27b.qmv(W, xq, n, want, residual=res)
    L = m27b.lib()
    part = torch.empty(L.m27b_qmv_mma_split_part_bytes(m27b.ctypes.byref(W.view), n), dtype=torch.uint8,
                       device="cuda")
    count = torch.zeros(L.m27b_qmv_mma_split_count_bytes(m27b.ctypes.byref(W.view)), dtype=torch.uint8,
                        device="cuda")
    ys = [torch.full((n, rows), float("nan"), device="cuda") for _ in range(3)]
    for y in ys:
        m27b.qmv_mma_split(W, xq, n, y, residual=res, part=part, count=count)
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])  # deterministic
    assert not count.any()                                             # counters back at zero
    base = want - res if residual else want
    d = (ys[0] - want).double()
    assert float(d.norm() / base.double().norm()) <= TIGHT
    assert m27b.device_status() == 0


def test_split_refuses_what_it_does_not_serve(torch, m27b):
    W = m27b.QWeight(D.random_valid_blocks(Q4_K, 256, 1024, 3), Q4_K, 1024, 256)
    xq = m27b.act_quant(torch.from_numpy(D.gauss_act(4, 1024, 4)).cuda(), Q8_K)
    with pytest.raises(m27b.M27BError, match="not served"):
        m27b.qmv_mma_split(W, xq, 4, torch.empty((4, 256), device="cuda"))
