"""q6_K x one token with the (row group, tile) items cut evenly over the
warps of the grid (m27b_qmv_q6k_stream, a decode step's ffn_down) through
the C ABI:
  * against the oracle (ggml vec_dot_q6_K_q8_K) on Gaussian-quantized
    weights: rel. L2 <= 1e-3 and <= 2e-5 (same
    integer sums; only the fp32 order of the runs' partials differs), over
    shapes whose groups span several runs, lie inside one run, end ragged
    (rows not a multiple of 8, rows not a multiple of 4 blocks), and leave
    most warps without an item;
  * at ffn_down's shape (5120 x 17408) against the one-pass kernel
    (m27b_qmv) on random valid blocks: <= 2e-5, with the residual epilogue;
  * deterministic (two calls give the same bits), the arrival counters back
    at zero after every call; rows too long to stage are refused."""
import numpy as np
import pytest

import _data as D

pytestmark = pytest.mark.gpu

Q6_K, Q8_K = 14, 15
TOL, TIGHT = 1e-3, 2e-5


@pytest.mark.parametrize("rows,k", [(5120, 17408), (1000, 8192), (333, 12288), (37, 2560), (8, 256), (4000, 1024),
                                    (21, 5120)])
def test_stream_against_oracle(torch, orc, m27b, rows, k):
    w = D.gauss_weights(orc, Q6_K, rows, k, rows + 7)
    x = D.gauss_act(1, k, 3 + rows)
    want = orc.matvec(Q6_K, w, k, orc.quantize_q8_K(x))
    W = m27b.QWeight(w, Q6_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(x).cuda(), Q8_K)
    y = torch.full((1, rows), float("nan"), device="cuda")
    m27b.qmv_q6k_stream(W, xq, y)
    torch.cuda.synchronize()
    err = orc.rel_l2(y.cpu().numpy(), want)
    assert err <= TOL and err <= TIGHT, err
    assert m27b.device_status() == 0


def test_stream_ffn_down_shape_matches_one_pass(torch, m27b):
    rows, k = 5120, 17408
    W = m27b.QWeight(D.random_valid_blocks(Q6_K, rows, k, 50), Q6_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(D.gauss_act(1, k, 51)).cuda(), Q8_K)
    res = torch.from_numpy(D.gauss_act(1, rows, 52)).cuda()
    want = torch.empty((1, rows), device="cuda")
    m27b.qmv(W, xq, 1, want, residual=res)
    L = m27b.lib()
    part = torch.empty(L.m27b_qmv_q6k_stream_part_bytes(m27b.ctypes.byref(W.view)), dtype=torch.uint8, device="cuda")
    count = torch.zeros(L.m27b_qmv_q6k_stream_count_bytes(m27b.ctypes.byref(W.view)), dtype=torch.uint8,
                        device="cuda")
    ys = [torch.full((1, rows), float("nan"), device="cuda") for _ in range(3)]
    for y in ys:
        m27b.qmv_q6k_stream(W, xq, y, residual=res, part=part, count=count)
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])  # deterministic
    assert not count.any()                                             # counters back at zero
    d = (ys[0] - want).double()
    assert float(d.norm() / (want - res).double().norm()) <= TIGHT
    assert m27b.device_status() == 0


def test_stream_refuses_rows_too_long(torch, m27b):
    k = 256 * 640
    W = m27b.QWeight(D.random_valid_blocks(Q6_K, 8, k, 1), Q6_K, k, 8)
    xq = m27b.act_quant(torch.from_numpy(D.gauss_act(1, k, 2)).cuda(), Q8_K)
    with pytest.raises(m27b.M27BError, match="too long"):
        m27b.qmv_q6k_stream(W, xq, torch.empty((1, 8), device="cuda"))
