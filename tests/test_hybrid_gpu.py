"""The hybrid model's Gated DeltaNet layers on the GPU against the decode
reference (tests/_decode_ref.py, which restates the reference's block
src/mono27b_executor.cu:2484-2548 in numpy).

A 4-layer model with attn_interval 2 alternates DeltaNet (layers 0, 2) and
attention (layers 1, 3) layers.  Covered: several decode steps (the conv and
delta-rule states carry over; the first step also builds the CUDA graph,
whose eager warm-up run must leave the states as they were), f16 and f32
conv weights, f16 and quantized beta/alpha projections, mixed projection
types, reset() restoring the zero state, device-side generation equal to the
host loop, and the verify pass refusing a hybrid model.

Tolerance: the kernels' fp32 sums run in another order than numpy's, so an
activation that lies within ~1e-5 of a q8_K rounding tie can take the other
code on one side; on this 512-wide model one such code moves the logits by
up to ~1e-2 for that step.  A wrong state update would persist: so the test
wants most steps at fp32-rounding level (median <= 1e-5), never two
consecutive steps above 1e-4, and every step <= 2e-2."""
import numpy as np
import pytest

import _decode_ref as R

pytestmark = pytest.mark.gpu

F16, Q4_K, Q5_K, IQ4_XS = 1, 12, 13, 23
HYB = dict(R.TINY, n_layers=4, attn_interval=2, ssm_d_inner=512, ssm_d_state=128, ssm_dt_rank=4, ssm_n_group=2,
           ssm_conv_kern=4)
STEP_TOL, MEDIAN_TOL, RUN_TOL = 2e-2, 1e-5, 1e-4


def _engine(m27b, c, model, max_ctx=64):
    d = dict(m27b.QWEN27)
    d.update(c)
    e = m27b.Engine(m27b.model_config(max_ctx=max_ctx, **d))
    for name, (qtype, row_elems, row_count, data) in model.items():
        e.load_tensor(name, qtype, row_elems, row_count, data)
    return e


@pytest.mark.parametrize("variant", ["default", "mixed_types"])
def test_hybrid_decode_matches_reference(orc, m27b, variant):
    types = {} if variant == "default" else dict(attn_gate=IQ4_XS, ssm_beta=Q4_K, ssm_alpha=Q4_K, ssm_out=Q5_K,
                                                 ssm_conv1d=F16)
    model = R.make_model(orc, HYB, seed=21, types=types)
    ref = R.RefDecoder(orc, model, HYB)
    e = _engine(m27b, HYB, model)
    try:
        errs = []
        for pos, t in enumerate([7, 70, 700, 77, 707, 17, 170, 901, 2, 333]):
            nxt, lg = e.decode_step(t, pos, logits=True)
            lg_ref, _ = ref.step(t, pos)
            errs.append(orc.rel_l2(lg, lg_ref))
            top = np.sort(lg_ref)[-2:]
            if errs[-1] <= RUN_TOL and top[1] - top[0] > 1e-3 * np.abs(lg_ref).max():
                assert nxt == orc.argmax(lg_ref), pos
        print("hybrid rel-L2 per step:", ["%.2e" % x for x in errs])
        assert max(errs) <= STEP_TOL, errs
        assert float(np.median(errs)) <= MEDIAN_TOL, errs
        assert not any(a > RUN_TOL and b > RUN_TOL for a, b in zip(errs, errs[1:])), errs
        assert m27b.device_status() == 0
    finally:
        e.close()


def test_hybrid_reset_generate_and_verify(orc, m27b):
    model = R.make_model(orc, HYB, seed=22)
    e = _engine(m27b, HYB, model)
    try:
        prompt = [5, 55, 555]
        first = [e.decode_step(t, p, logits=True)[1] for p, t in enumerate(prompt)]
        e.reset()
        again = [e.decode_step(t, p, logits=True)[1] for p, t in enumerate(prompt)]
        for a, b in zip(first, again):
            assert np.array_equal(a, b)  # the recurrent state restarts from zero
        # device-side greedy generation equals the host loop over decode_step
        # (each from the state after prompt[:-1]: a DeltaNet layer must see
        # every token exactly once, unlike an attention layer, which just
        # rewrites the cache entry of a repeated position)
        e.reset()
        for p, t in enumerate(prompt[:-1]):
            e.decode_step(t, p)
        gen = [int(t) for t in e.generate(prompt[-1], len(prompt) - 1, 8)]
        e.reset()
        for p, t in enumerate(prompt[:-1]):
            e.decode_step(t, p)
        tok, host = prompt[-1], []
        for i in range(8):
            tok = e.decode_step(tok, len(prompt) - 1 + i)
            host.append(tok)
        assert gen == host
        with pytest.raises(m27b.M27BError, match="hybrid"):
            e.verify([1, 2, 3], 10)
        assert m27b.device_status() == 0
    finally:
        e.close()
