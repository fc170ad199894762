"""q6_K x 1..8 tokens on the tensor cores (m27b_qmv_q6k_mma and
m27b_qmv_q6k_mma_argmax, the verify pass's ffn_down and lm_head) through the
C ABI:
  * against the oracle (ggml vec_dot_q6_K_q8_K) on Gaussian-quantized
    weights, with and without the K split: rel. L2 <= 1e-3 (north-star
    tolerance) and <= 2e-5 (same integer sums; only the fp32 order of the
    block and range partials differs);
  * at ffn_down's shape (5120 x 17408, K split) against the one-pass kernel
    (m27b_qmv) on random valid blocks, with the residual: <= 2e-5;
    deterministic, arrival counters back at zero;
  * ragged shapes: a partial last 128-row tile, rows < 128, 1..8 tokens;
  * the argmax epilogue: the logits within 2e-5 of the oracle's, each
    token's key the argmax of the kernel's own logits (ties to the smaller
    index, the row offset added), the same keys without logits;
  * refusals (token count, weight type, half-given scratch) and a clean
    device status word (a stalled hand-off shows up there)."""
import numpy as np
import pytest

import _data as D

pytestmark = pytest.mark.gpu

Q4_K, Q6_K, Q8_K = 12, 14, 15
TOL, TIGHT = 1e-3, 2e-5


@pytest.mark.parametrize("rows,k,n,split", [(1000, 8192, 5, True), (333, 4096, 8, False), (129, 2048, 1, True),
                                            (77, 5120, 3, False), (777, 17408, 7, True), (300, 17408, 8, False)])
def test_q6k_mma_against_oracle(torch, orc, m27b, rows, k, n, split):
    w = D.gauss_weights(orc, Q6_K, rows, k, rows + 3 * n)
    x = D.gauss_act(n, k, 7 + n)
    want = orc.matvec(Q6_K, w, k, orc.quantize_q8_K(x))
    W = m27b.QWeight(w, Q6_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(x).cuda(), Q8_K)
    y = torch.full((n, rows), float("nan"), device="cuda")
    m27b.qmv_q6k_mma(W, xq, n, y, split=split)
    torch.cuda.synchronize()
    err = orc.rel_l2(y.cpu().numpy(), want)
    assert err <= TOL and err <= TIGHT, err
    assert m27b.device_status() == 0


@pytest.mark.parametrize("n", [5, 8])
def test_q6k_mma_ffn_down_shape_matches_one_pass(torch, m27b, n):
    rows, k = 5120, 17408
    W = m27b.QWeight(D.random_valid_blocks(Q6_K, rows, k, 60 + n), Q6_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(D.gauss_act(n, k, 61)).cuda(), Q8_K)
    res = torch.from_numpy(D.gauss_act(n, rows, 62)).cuda()
    want = torch.empty((n, rows), device="cuda")
    m27b.qmv(W, xq, n, want, residual=res)
    L = m27b.lib()
    part = torch.empty(L.m27b_qmv_q6k_mma_part_bytes(m27b.ctypes.byref(W.view)), dtype=torch.uint8, device="cuda")
    count = torch.zeros(L.m27b_qmv_q6k_mma_count_bytes(m27b.ctypes.byref(W.view)), dtype=torch.uint8, device="cuda")
    ys = [torch.full((n, rows), float("nan"), device="cuda") for _ in range(3)]
    for y in ys:
        m27b.qmv_q6k_mma(W, xq, n, y, residual=res, part=part, count=count)
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])  # deterministic
    assert not count.any()                                             # counters back at zero
    d = (ys[0] - want).double()
    assert float(d.norm() / (want - res).double().norm()) <= TIGHT
    assert m27b.device_status() == 0


@pytest.mark.parametrize("rows,n,offset", [(4173, 8, 0), (1000, 5, 123456), (130, 2, 7)])
def test_q6k_mma_argmax(torch, orc, m27b, rows, n, offset):
    k = 5120
    w = D.gauss_weights(orc, Q6_K, rows, k, 90 + rows)
    x = D.gauss_act(n, k, 91)
    want = orc.matvec(Q6_K, w, k, orc.quantize_q8_K(x))
    W = m27b.QWeight(w, Q6_K, k, rows)
    xq = m27b.act_quant(torch.from_numpy(x).cuda(), Q8_K)
    logits = torch.full((n, rows), float("nan"), device="cuda")
    best = torch.zeros(n, dtype=torch.int64, device="cuda")
    m27b.qmv_q6k_mma_argmax(W, xq, n, best, logits=logits, row_offset=offset)
    best2 = torch.zeros(n, dtype=torch.int64, device="cuda")
    m27b.qmv_q6k_mma_argmax(W, xq, n, best2, row_offset=offset)
    torch.cuda.synchronize()
    lg = logits.cpu().numpy()
    assert orc.rel_l2(lg, want) <= TIGHT
    keys = [int(v) & 0xffffffffffffffff for v in best.cpu().numpy()]
    for t in range(n):
        assert m27b.argmax_key_index(keys[t]) == int(np.argmax(lg[t])) + offset
    assert torch.equal(best, best2)
    assert m27b.device_status() == 0


def test_q6k_mma_refusals(torch, m27b):
    W = m27b.QWeight(D.random_valid_blocks(Q6_K, 256, 2048, 5), Q6_K, 2048, 256)
    xq = m27b.act_quant(torch.from_numpy(D.gauss_act(9, 2048, 6)).cuda(), Q8_K)
    y = torch.empty((9, 256), device="cuda")
    with pytest.raises(m27b.M27BError, match="not served"):
        m27b.qmv_q6k_mma(W, xq, 9, y, split=False)
    with pytest.raises(m27b.M27BError, match="go together"):
        m27b.qmv_q6k_mma(W, xq, 4, y, part=torch.empty(64, dtype=torch.uint8, device="cuda"), split=False)
    W4 = m27b.QWeight(D.random_valid_blocks(Q4_K, 256, 2048, 7), Q4_K, 2048, 256)
    with pytest.raises(m27b.M27BError, match="repacked q6_K"):
        m27b.qmv_q6k_mma(W4, xq, 4, y, split=False)
