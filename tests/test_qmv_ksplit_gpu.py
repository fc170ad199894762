"""q6_K x 5..16 tokens with the K dimension split across CTAs
(m27b_qmv_q6k_ksplit, the verify pass's ffn_down) through the C ABI:
  * against the oracle (ggml vec_dot_q6_K_q8_K) on Gaussian-quantized
    weights: rel. L2 <= 1e-3 and <= 2e-5 (same
    integer sums; only the fp32 order of the range partials differs);
  * at ffn_down's shape (5120 x 17408, 4 K ranges) against the one-pass
    kernel (m27b_qmv) on random valid blocks: <= 2e-5;
  * deterministic (two calls give the same bits) and the arrival counters are
    back at zero after every call; the residual epilogue; rows < 32 blocks
    are refused."""
import numpy as np
import pytest

import _data as D

pytestmark = pytest.mark.gpu

Q6_K, Q8_K = 14, 15
TOL, TIGHT = 1e-3, 2e-5


@pytest.mark.parametrize("rows,k,n", [(1000, 8192, 5), (333, 12288, 8), (777, 17408, 13)])
def test_ksplit_against_oracle(torch, orc, m27b, rows, k, n):
    w = D.gauss_weights(orc, Q6_K, rows, k, rows + n)
    x = D.gauss_act(n, k, 3 + n)
    want = orc.matvec(Q6_K, w, k, orc.quantize_q8_K(x))
    W = m27b.QWeight(w, Q6_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(x).cuda(), Q8_K)
    y = torch.full((n, rows), float("nan"), device="cuda")
    m27b.qmv_q6k_ksplit(W, xq, n, y)
    torch.cuda.synchronize()
    err = orc.rel_l2(y.cpu().numpy(), want)
    assert err <= TOL and err <= TIGHT, err
    assert m27b.device_status() == 0


@pytest.mark.parametrize("n", [5, 8, 16])
def test_ksplit_ffn_down_shape_matches_one_pass(torch, m27b, n):
    rows, k = 5120, 17408
    W = m27b.QWeight(D.random_valid_blocks(Q6_K, rows, k, 40 + n), Q6_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(D.gauss_act(n, k, 41)).cuda(), Q8_K)
    res = torch.from_numpy(D.gauss_act(n, rows, 42)).cuda()
    want = torch.empty((n, rows), device="cuda")
    m27b.qmv(W, xq, n, want, residual=res)
    part = torch.empty(m27b.lib().m27b_qmv_q6k_ksplit_part_bytes(m27b.ctypes.byref(W.view)), dtype=torch.uint8,
                       device="cuda")
    count = torch.zeros(m27b.lib().m27b_qmv_q6k_ksplit_count_bytes(m27b.ctypes.byref(W.view)), dtype=torch.uint8,
                        device="cuda")
    ys = [torch.full((n, rows), float("nan"), device="cuda") for _ in range(2)]
    for y in ys:
        m27b.qmv_q6k_ksplit(W, xq, n, y, residual=res, part=part, count=count)
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1])                 # deterministic
    assert not count.any()                           # counters back at zero
    d = (ys[0] - want).double()
    assert float(d.norm() / (want - res).double().norm()) <= TIGHT
    assert m27b.device_status() == 0


def test_ksplit_refuses_short_rows(torch, m27b):
    W = m27b.QWeight(D.random_valid_blocks(Q6_K, 64, 2048, 1), Q6_K, 2048, 64)
    xq = m27b.act_quant(torch.from_numpy(D.gauss_act(8, 2048, 2)).cuda(), Q8_K)
    with pytest.raises(m27b.M27BError, match="too short"):
        m27b.qmv_q6k_ksplit(W, xq, 8, torch.empty((8, 64), device="cuda"), part=torch.empty(16, dtype=torch.uint8,
                            device="cuda"), count=torch.zeros(16, dtype=torch.uint8, device="cuda"))
