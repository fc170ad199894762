"""Speculative verification and the speculative decoding loop on one GPU.

* m27b_engine_verify on n tokens equals n single decode steps fed the same
  tokens (the decode reference decides: the greedy tokens where the
  reference's top-2 margin is clear, logits at rel-L2 2e-3 — the batched
  kernels add the per-block partials in another order, and on this 512-wide
  model (2 q8_K blocks per row) one activation code that rounds the other way
  moves the logits by ~1e-3); 5+ tokens run the q4_K matrices on the tensor
  cores.
* A q8_0 draft model (every matrix q8_0, as the reference's draft) decodes
  like the reference decoder.
* The speculative loop is lossless: with any draft — an unrelated q8_0 model
  (almost nothing accepted) or the target's own weights (everything
  accepted) — it returns exactly the target's greedy tokens."""
import numpy as np
import pytest

import _decode_ref as R

pytestmark = pytest.mark.gpu

Q8_0 = 8
TOL = 1e-3


def _engine(m27b, c, model=None, max_ctx=96, weight_type=0):
    d = dict(m27b.QWEN27)
    d.update(c)
    e = m27b.Engine(m27b.model_config(max_ctx=max_ctx, weight_type=weight_type, **d))
    if model is not None:
        for name, (qtype, row_elems, row_count, data) in model.items():
            e.load_tensor(name, qtype, row_elems, row_count, data)
    return e


@pytest.mark.parametrize("n", [1, 4, 8, 13])
def test_verify_matches_reference(orc, m27b, n):
    c = dict(R.TINY, n_layers=2)
    model = R.make_model(orc, c, seed=3)
    ref = R.RefDecoder(orc, model, c, max_ctx=96)
    e = _engine(m27b, c, model)
    try:
        rng = np.random.default_rng(n)
        toks = [int(t) for t in rng.integers(0, c["vocab"], 6 + n)]
        for pos in range(6):  # a prefix through single steps
            e.decode_step(toks[pos], pos)
            ref.step(toks[pos], pos)
        nxt, lg = e.verify(toks[6:], 6, logits=True)
        errs = []
        for i in range(n):
            lg_ref, _ = ref.step(toks[6 + i], 6 + i)
            errs.append(orc.rel_l2(lg[i], lg_ref))
            top = np.sort(lg_ref)[-2:]
            if top[1] - top[0] > 1e-3 * np.abs(lg_ref).max():
                assert nxt[i] == orc.argmax(lg_ref), i
        print("verify rel-L2 per token:", ["%.2e" % x for x in errs])
        assert max(errs) <= 2e-3, errs
    finally:
        e.close()


def test_q8_0_draft_decodes_like_reference(orc, m27b):
    c = dict(n_layers=2, hidden=256, ffn=512, n_head=4, n_kv_head=2, head_dim=64, vocab=1000, n_rot=32,
             rope_theta=1e6, rms_eps=1e-6)
    model = R.make_model(orc, c, seed=4, qtype=Q8_0)
    ref = R.RefDecoder(orc, model, c)
    e = _engine(m27b, c, model)
    try:
        for pos, t in enumerate([5, 50, 500, 7]):
            nxt, lg = e.decode_step(t, pos, logits=True)
            lg_ref, _ = ref.step(t, pos)
            assert orc.rel_l2(lg, lg_ref) <= TOL, pos
    finally:
        e.close()


def _greedy(e, prompt, n):
    for pos, t in enumerate(prompt[:-1]):
        e.decode_step(t, pos)
    return [int(t) for t in e.generate(prompt[-1], len(prompt) - 1, n)]


@pytest.mark.parametrize("draft_kind", ["unrelated_q8_0", "self"])
def test_speculative_loop_is_lossless(orc, m27b, draft_kind):
    c = dict(R.TINY, n_layers=2)
    target_model = R.make_model(orc, c, seed=5)
    draft_model = R.make_model(orc, c, seed=6, qtype=Q8_0) if draft_kind != "self" else target_model
    prompt = [11, 22, 33, 44, 55]
    n_new = 30
    t1 = _engine(m27b, c, target_model)
    try:
        want = _greedy(t1, prompt, n_new)
    finally:
        t1.close()
    t2, d = _engine(m27b, c, target_model), _engine(m27b, c, draft_model)
    try:
        got, stats = m27b.speculative_generate(t2, d, prompt, n_new, k=7)
    finally:
        t2.close()
        d.close()
    assert got == want
    if draft_kind == "self":
        # the draft runs the single-token kernels, the verify pass the batched ones: near-ties may differ
        assert stats["accepted"] >= 0.9 * stats["proposed"]
