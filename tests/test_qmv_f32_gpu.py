"""Matvecs from fp32 activations (m27b_qmv_f32 / m27b_qmv_f32_rmsnorm): the
q4_K kernel (and, without RMSNorm, the q6_K kernel) quantizes its rows in
the prologue with the same q8_K routine as m27b_act_quant, so the one-launch
path must equal act_quant + qmv bit for bit; the RMSNorm variants are compared with the oracle (RMSNorm in fp32 +
ggml q8_K + vec_dot) at the matvec tolerance, and the two-launch path (other
weight types, more tokens) with the same entry's one-launch result."""
import numpy as np
import pytest

import _data as D

pytestmark = pytest.mark.gpu

Q8_0, Q4_K, Q6_K, Q8_K = 8, 12, 14, 15
TOL = 1e-3


def _w(orc, m27b, qtype, rows, k, seed):
    return D.gauss_weights(orc, qtype, rows, k, seed), m27b.QWeight(D.gauss_weights(orc, qtype, rows, k, seed), qtype,
                                                                     k, rows)


@pytest.mark.parametrize("rows,k,n", [(300, 5120, 1), (129, 1280, 2), (4096, 6144, 1), (77, 256, 4), (1000, 17408, 3)])
def test_qmv_f32_equals_separate_quant(torch, orc, m27b, rows, k, n):
    w, W = _w(orc, m27b, Q4_K, rows, k, rows + k)
    x = torch.from_numpy(D.gauss_act(n, k, 3 + n)).cuda()
    res = torch.from_numpy(D.gauss_act(n, rows, 4)).cuda()
    want = torch.empty((n, rows), device="cuda")
    m27b.qmv(W, m27b.act_quant(x, Q8_K), n, want, residual=res)
    got = torch.full((n, rows), float("nan"), device="cuda")
    m27b.qmv_f32(W, x, n, got, residual=res)
    assert torch.equal(got, want)


@pytest.mark.parametrize("rows,k,n", [(5120, 17408, 1), (333, 2048, 2), (77, 256, 4), (1000, 17408, 3)])
def test_qmv_f32_q6K_equals_separate_quant(torch, orc, m27b, rows, k, n):
    """ffn_down's shape (5120 x 17408) among them: the q6_K kernel's own
    quantizing prologue gives act_quant + qmv's result bit for bit."""
    w, W = _w(orc, m27b, Q6_K, rows, k, rows + k + 7)
    x = torch.from_numpy(D.gauss_act(n, k, 5 + n)).cuda()
    res = torch.from_numpy(D.gauss_act(n, rows, 6)).cuda()
    want = torch.empty((n, rows), device="cuda")
    m27b.qmv(W, m27b.act_quant(x, Q8_K), n, want, residual=res)
    got = torch.full((n, rows), float("nan"), device="cuda")
    m27b.qmv_f32(W, x, n, got, residual=res)
    assert torch.equal(got, want)
    assert orc.rel_l2(got.cpu().numpy() - res.cpu().numpy(),
                      orc.matvec(Q6_K, w, k, orc.quantize_q8_K(x.cpu().numpy()))) <= TOL


@pytest.mark.parametrize("n", [1, 3])
def test_qmv_f32_rmsnorm(torch, orc, m27b, n):
    rows, k = 700, 5120
    w, W = _w(orc, m27b, Q4_K, rows, k, 11)
    x = D.gauss_act(n, k, 12)
    nw = (1.0 + 0.1 * np.random.default_rng(13).standard_normal(k)).astype(np.float32)
    xn = (orc.rms_norm(x, 1e-6) * nw).astype(np.float32)
    want = orc.matvec(Q4_K, w, k, orc.quantize_q8_K(xn))
    got = torch.empty((n, rows), device="cuda")
    m27b.qmv_f32(W, torch.from_numpy(x).cuda(), n, got, norm_w=torch.from_numpy(nw).cuda(), eps=1e-6)
    assert orc.rel_l2(got.cpu().numpy(), want) <= TOL


def test_qmv_f32_rmsnorm_swiglu(torch, orc, m27b):
    rows, k, n = 600, 2048, 2
    g, G = _w(orc, m27b, Q4_K, rows, k, 21)
    u, U = _w(orc, m27b, Q4_K, rows, k, 22)
    x = D.gauss_act(n, k, 23)
    xq = orc.quantize_q8_K(orc.rms_norm(x, 1e-5))
    want = orc.silu_mul(orc.matvec(Q4_K, g, k, xq), orc.matvec(Q4_K, u, k, xq))
    got = torch.empty((n, rows), device="cuda")
    m27b.qmv_f32(G, torch.from_numpy(x).cuda(), n, got, eps=1e-5, up=U)
    assert orc.rel_l2(got.cpu().numpy(), want) <= TOL


@pytest.mark.parametrize("qtype,n", [(Q6_K, 5), (Q8_0, 2), (Q4_K, 8)])
def test_qmv_f32_two_launch_path(torch, orc, m27b, qtype, n):
    rows, k = 333, 2048
    w, W = _w(orc, m27b, qtype, rows, k, 31)
    x = D.gauss_act(n, k, 32)
    want = orc.matvec(qtype, w, k, orc.quantize_act(qtype, x))
    scratch = torch.empty(n * m27b.act_bytes(m27b.act_type_for(qtype), k), dtype=torch.uint8, device="cuda")
    got = torch.empty((n, rows), device="cuda")
    m27b.qmv_f32(W, torch.from_numpy(x).cuda(), n, got, xq_scratch=scratch)
    assert orc.rel_l2(got.cpu().numpy(), want) <= TOL
    with pytest.raises(m27b.M27BError, match="xq_scratch"):
        m27b.qmv_f32(W, torch.from_numpy(x).cuda(), n, got)


@pytest.mark.parametrize("n", [1, 4])
def test_act_quant_swiglu_equals_swiglu_epilogue(torch, orc, m27b, n):
    # gate and up as two matvecs, then silu(gate) * up quantized, gives the
    # same q8_K bytes as the fused SwiGLU epilogue followed by a quantizer
    rows, k = 2048, 5120
    (_, G), (_, U) = _w(orc, m27b, Q4_K, rows, k, 91), _w(orc, m27b, Q4_K, rows, k, 92)
    xq = m27b.act_quant(torch.from_numpy(D.gauss_act(n, k, 93)).cuda(), Q8_K)
    a = torch.empty((n, rows), device="cuda")
    m27b.qmv_swiglu(G, U, xq, n, a)
    fused = m27b.act_quant(a, Q8_K)
    g, u = torch.empty((n, rows), device="cuda"), torch.empty((n, rows), device="cuda")
    m27b.qmv(G, xq, n, g)
    m27b.qmv(U, xq, n, u)
    sep = m27b.act_quant_swiglu(g, u, Q8_K)
    want = orc.quantize_q8_K(orc.silu_mul(g.cpu().numpy(), u.cpu().numpy()))
    assert torch.equal(sep, fused)
    # against the oracle's silu * up (fp64 exp): at most a rare last-code flip
    got = sep.cpu().numpy().reshape(n, -1)
    assert (got != want).mean() < 1e-3
