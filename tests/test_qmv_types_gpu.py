"""q5_K, IQ4_XS, f16 and f32 matrices on the GPU against the oracle.

The reference dispatches these types to k_q5k_mv_q8 / k_iq4xs_mv_q8_dp4a
(q8 activations, src/mono27b_executor.cu:2066-2077) and to k_f16_mv /
k_f32_mv (fp32 activations, the fallback :2127-2137).  Here q5_K and IQ4_XS
run on the q4_K streaming design with ggml's q8_K activations (integer sums
equal to ggml's vec_dot_q5_K_q8_K / vec_dot_iq4_xs_q8_K, only the fp32
accumulation order differs: the tight bound), f16 / f32 on a vector-load
streaming kernel with ggml's f16 semantics (x rounded to fp16).  Covered:
ragged and full-size shapes, 1..6 tokens (the 4-token launch chunks), the
residual, SwiGLU and argmax epilogues, the quantize-in-prologue entry
(bit-identical to quantize + matvec), few-row and many-row grid shapes of
the f16 kernel, the shape errors, and a decode model whose layers mix the
new types with q4_K / q6_K.  Every run leaves the device status word clear."""
import numpy as np
import pytest

import _data as D
import _decode_ref as R

pytestmark = pytest.mark.gpu

F32, F16, Q4_K, Q5_K, Q6_K, Q8_K, IQ4_XS = 0, 1, 12, 13, 14, 15, 23
TIGHT = 2e-5
FLOAT_TOL = 1e-5


def _weights(orc, qt, rows, k, seed):
    return D.gauss_weights(orc, qt, rows, k, seed)


def _run_q8(torch, orc, m27b, qt, rows, k, n, seed, residual=False):
    w = _weights(orc, qt, rows, k, seed)
    x = D.gauss_act(n, k, seed + 1)
    want = orc.matvec(qt, w, k, orc.quantize_q8_K(x))
    W = m27b.QWeight(w, qt, k, rows)
    xq = m27b.act_quant(torch.from_numpy(x).cuda(), Q8_K)
    y = torch.full((n, rows), float("nan"), device="cuda")
    res = None
    if residual:
        r = D.gauss_act(n, rows, seed + 2)
        want = want + r
        res = torch.from_numpy(r).cuda()
    m27b.qmv(W, xq, n, y, residual=res)
    got = y.cpu().numpy()
    assert m27b.device_status() == 0
    return orc.rel_l2(got, want)


@pytest.mark.parametrize("qt", [Q5_K, IQ4_XS])
@pytest.mark.parametrize("rows,k", [(1, 512), (77, 512), (300, 1024), (129, 6144), (5120, 5120), (1000, 17408)])
def test_kquant_shapes(torch, orc, m27b, qt, rows, k):
    assert _run_q8(torch, orc, m27b, qt, rows, k, 1, rows + k + qt) <= TIGHT


@pytest.mark.parametrize("qt", [Q5_K, IQ4_XS])
@pytest.mark.parametrize("n", [2, 3, 4, 5, 6])
def test_kquant_tokens_and_residual(torch, orc, m27b, qt, n):
    assert _run_q8(torch, orc, m27b, qt, 700, 2048, n, 40 + n, residual=(n % 2 == 1)) <= TIGHT


def test_q5K_odd_block_count(torch, orc, m27b):
    # q5_K rows need no alignment beyond their 176-byte blocks (11 x 16 B)
    assert _run_q8(torch, orc, m27b, Q5_K, 333, 256 * 7, 2, 5) <= TIGHT


@pytest.mark.parametrize("qt", [Q5_K, IQ4_XS])
def test_kquant_swiglu_and_argmax(torch, orc, m27b, qt):
    rows, k, n = 600, 2048, 2
    wg, wu = _weights(orc, qt, rows, k, 61), _weights(orc, qt, rows, k, 62)
    x = D.gauss_act(n, k, 63)
    xq_c = orc.quantize_q8_K(x)
    want = orc.silu_mul(orc.matvec(qt, wg, k, xq_c), orc.matvec(qt, wu, k, xq_c))
    G, U = m27b.QWeight(wg, qt, k, rows), m27b.QWeight(wu, qt, k, rows)
    xq = m27b.act_quant(torch.from_numpy(x).cuda(), Q8_K)
    y = torch.empty((n, rows), device="cuda")
    m27b.qmv_swiglu(G, U, xq, n, y)
    assert orc.rel_l2(y.cpu().numpy(), want) <= TIGHT
    logits = torch.empty((n, rows), device="cuda")
    best = torch.empty(n, dtype=torch.int64, device="cuda")
    m27b.qmv_argmax(G, xq, n, best, logits=logits)
    want_lg = orc.matvec(qt, wg, k, xq_c)
    lg = logits.cpu().numpy()
    keys = best.cpu().numpy().view(np.uint64)
    assert orc.rel_l2(lg, want_lg) <= TIGHT
    for t in range(n):
        idx = m27b.argmax_key_index(keys[t])
        assert idx == int(np.argmax(lg[t]))  # consistent with its own logits, ties to the smallest
        assert want_lg[t, idx] >= want_lg[t].max() - 1e-5 * np.abs(want_lg[t]).max()
    assert m27b.device_status() == 0


@pytest.mark.parametrize("qt", [Q5_K, IQ4_XS])
@pytest.mark.parametrize("n", [1, 3])
def test_kquant_quantizing_prologue_is_bit_identical(torch, orc, m27b, qt, n):
    rows, k = 900, 5120
    W = m27b.QWeight(_weights(orc, qt, rows, k, 70 + n), qt, k, rows)
    x = torch.from_numpy(D.gauss_act(n, k, 80 + n)).cuda()
    y1 = torch.empty((n, rows), device="cuda")
    m27b.qmv_f32(W, x, n, y1)  # one launch: quantized in the kernel's prologue
    y2 = torch.empty((n, rows), device="cuda")
    m27b.qmv(W, m27b.act_quant(x, Q8_K), n, y2)
    assert torch.equal(y1, y2)
    assert m27b.device_status() == 0


@pytest.mark.parametrize("qt", [F16, F32])
@pytest.mark.parametrize("rows,k,n", [(48, 5120, 1), (5, 96, 3), (3000, 1024, 2), (40000, 256, 1), (700, 2048, 6)])
def test_float_weights(torch, orc, m27b, qt, rows, k, n):
    w = _weights(orc, qt, rows, k, rows + k)
    x = D.gauss_act(n, k, 90 + n)
    want = orc.matvec(qt, w, k, orc.quantize_act(qt, x))
    W = m27b.QWeight(w, qt, k, rows)
    xd = torch.from_numpy(x).cuda()
    y = torch.full((n, rows), float("nan"), device="cuda")
    r = D.gauss_act(n, rows, 3)
    m27b.qmv_f32(W, xd, n, y, residual=torch.from_numpy(r).cuda())
    assert orc.rel_l2(y.cpu().numpy(), want + r) <= FLOAT_TOL
    assert m27b.device_status() == 0


def test_shape_and_type_errors(torch, orc, m27b):
    W16 = m27b.QWeight(_weights(orc, F16, 8, 96, 1), F16, 96, 8)
    xq = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    y = torch.empty((1, 8), device="cuda")
    with pytest.raises(m27b.M27BError, match="fp32 activations"):
        m27b.qmv(W16, xq, 1, y)
    with pytest.raises(m27b.M27BError, match="plain matvec"):
        m27b.qmv_f32(W16, torch.zeros((1, 96), device="cuda"), 1, y, eps=1e-6)
    wi = _weights(orc, IQ4_XS, 8, 768, 2)  # 3 blocks per row: rows not 16-byte aligned
    Wi = m27b.QWeight(wi, IQ4_XS, 768, 8)
    with pytest.raises(m27b.M27BError, match="even number of blocks"):
        m27b.qmv(Wi, m27b.act_quant(torch.zeros((1, 768), device="cuda"), Q8_K), 1, y)
    w12 = torch.zeros(8 * 12, dtype=torch.uint16, device="cuda")  # 12 f16 values per row
    v = m27b.WeightView(w12.data_ptr(), F16, 12, 8)
    Wv = m27b.QWeight.__new__(m27b.QWeight)
    Wv.view, Wv.rows = v, 8
    with pytest.raises(m27b.M27BError, match="multiple of 8"):
        m27b.qmv_f32(Wv, torch.zeros((1, 16), device="cuda"), 1, y)


def test_decode_with_mixed_types(orc, m27b):
    # q/k/v q5_K, o_proj IQ4_XS, gate/up IQ4_XS, down q5_K, next to the
    # q4_K embedding and the q6_K head: the engine equals the decode reference
    c = dict(R.TINY, n_layers=2)
    types = dict(attn_q=Q5_K, attn_k=Q5_K, attn_v=Q5_K, attn_output=IQ4_XS, ffn_gate=IQ4_XS, ffn_up=IQ4_XS,
                 ffn_down=Q5_K)
    model = R.make_model(orc, c, seed=11, types=types)
    ref = R.RefDecoder(orc, model, c)
    d = dict(m27b.QWEN27)
    d.update(c)
    e = m27b.Engine(m27b.model_config(max_ctx=64, **d))
    try:
        for name, (qtype, row_elems, row_count, data) in model.items():
            e.load_tensor(name, qtype, row_elems, row_count, data)
        for pos, t in enumerate([3, 30, 300, 999, 4]):
            nxt, lg = e.decode_step(t, pos, logits=True)
            lg_ref, _ = ref.step(t, pos)
            assert orc.rel_l2(lg, lg_ref) <= 1e-3, pos
        assert m27b.device_status() == 0
    finally:
        e.close()
