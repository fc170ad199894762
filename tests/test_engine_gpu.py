"""Decode engine on one GPU against the decode reference (oracle pieces + numpy).

Tolerance: the engine's fp32 glue (RMSNorm, RoPE with sincosf/powf, softmax
with expf, sums in another order) differs from the numpy reference in the last
bits; an activation that lands within an ulp of a q8_K rounding boundary can
then round the other way.  Logits and the hidden state are compared with
rel-L2 <= 1e-3 (the matvec tolerance), the greedy token exactly whenever the
reference's top-2 margin exceeds 1e-3 of the logit scale."""
import numpy as np
import pytest

import _decode_ref as R

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _engine(m27b, c, max_ctx=64):
    d = dict(m27b.QWEN27)
    d.update(c)
    return m27b.Engine(m27b.model_config(max_ctx=max_ctx, **d))


def _load(e, model):
    for name, (qtype, row_elems, row_count, data) in model.items():
        e.load_tensor(name, qtype, row_elems, row_count, data)


def _decode_compare(orc, m27b, c, seed, n_steps, prompt):
    model = R.make_model(orc, c, seed=seed)
    ref = R.RefDecoder(orc, model, c)
    e = _engine(m27b, c)
    try:
        _load(e, model)
        tok = prompt[0]
        for pos in range(n_steps):
            lg_ref, h_ref = ref.step(tok, pos)
            nxt, lg = e.decode_step(tok, pos, logits=True)
            assert orc.rel_l2(e.hidden(), h_ref) <= TOL, pos
            assert orc.rel_l2(lg, lg_ref) <= TOL, pos
            top = np.sort(lg_ref)[-2:]
            if top[1] - top[0] > 1e-3 * np.abs(lg_ref).max():
                assert nxt == orc.argmax(lg_ref), pos
            assert nxt == orc.argmax(lg), pos  # the engine's token is its own logits' first argmax
            tok = prompt[pos + 1] if pos + 1 < len(prompt) else orc.argmax(lg_ref)
    finally:
        e.close()


def test_engine_tiny_decode(orc, m27b):
    _decode_compare(orc, m27b, R.TINY, seed=0, n_steps=8, prompt=[5, 17, 900])


def test_engine_shared_kv_uneven(orc, m27b):
    # 4 query heads per kv head, head_dim 64, n_rot 32, ffn of 5 blocks
    c = dict(n_layers=3, hidden=768, ffn=1280, n_head=8, n_kv_head=2, head_dim=64, vocab=777, n_rot=32,
             rope_theta=1e6, rms_eps=1e-5)
    _decode_compare(orc, m27b, c, seed=1, n_steps=6, prompt=[1, 2, 3, 4])


def test_engine_unfused_head_dim(orc, m27b):
    # head_dim 96 does not divide 256: the engine uses its unfused attention kernels
    c = dict(n_layers=2, hidden=512, ffn=768, n_head=8, n_kv_head=2, head_dim=96, vocab=500, n_rot=32,
             rope_theta=1e6, rms_eps=1e-6)
    _decode_compare(orc, m27b, c, seed=6, n_steps=5, prompt=[3, 1, 4])


def test_engine_long_context(orc, m27b):
    # enough positions that every attention split holds several of them
    c = dict(R.TINY, n_layers=1)
    model = R.make_model(orc, c, seed=2)
    ref = R.RefDecoder(orc, model, c, max_ctx=300)
    e = _engine(m27b, c, max_ctx=300)
    try:
        _load(e, model)
        rng = np.random.default_rng(5)
        toks = rng.integers(0, c["vocab"], 300)
        for pos in range(300):
            lg_ref, _ = ref.step(int(toks[pos]), pos)
            _, lg = e.decode_step(int(toks[pos]), pos, logits=True)
            if pos in (0, 1, 63, 64, 150, 299):
                assert orc.rel_l2(lg, lg_ref) <= TOL, pos
    finally:
        e.close()


def test_engine_generate_matches_steps(orc, m27b):
    # on-device greedy generation = host-driven decode steps fed their own tokens
    c = dict(R.TINY, n_layers=3)
    model = R.make_model(orc, c, seed=4)
    e = _engine(m27b, c)
    try:
        _load(e, model)
        prompt = [9, 8, 7, 6]
        for pos, t in enumerate(prompt[:-1]):
            e.decode_step(t, pos)
        gen = e.generate(prompt[-1], len(prompt) - 1, 12)
        ref, tok = [], prompt[-1]
        for i in range(12):
            tok = e.decode_step(tok, len(prompt) - 1 + i)
            ref.append(tok)
        assert list(gen) == ref
    finally:
        e.close()


def test_engine_load_blob_equals_tensors(orc, m27b, tmp_path):
    # a model packed into a .m27b blob and loaded from it decodes bit for bit
    # like the same tensors loaded one by one
    c = dict(R.TINY, n_layers=2)
    model = R.make_model(orc, c, seed=8)
    path = tmp_path / "m.m27b"
    m27b.blob_pack(path, [dict(name=n, ggml_type=t, row_elems=re, row_count=rc, data=d)
                          for n, (t, re, rc, d) in model.items()], target_layers=c["n_layers"], vocab_size=c["vocab"])
    outs = []
    for via_blob in (False, True):
        e = _engine(m27b, c)
        try:
            if via_blob:
                e.load_blob(path)
            else:
                _load(e, model)
            steps = [e.decode_step(t, pos, logits=True) for pos, t in enumerate([4, 40, 400])]
            outs.append([(tok, lg.copy()) for tok, lg in steps])
        finally:
            e.close()
    for (t0, l0), (t1, l1) in zip(*outs):
        assert t0 == t1 and np.array_equal(l0, l1)


def test_engine_errors(m27b):
    e = _engine(m27b, R.TINY)
    try:
        with pytest.raises(m27b.M27BError, match="not loaded"):
            e.decode_step(0, 0)
        with pytest.raises(m27b.M27BError, match="outside the cache"):
            e.decode_step(0, 64)
        with pytest.raises(m27b.M27BError, match="outside the vocabulary"):
            e.decode_step(1000, 0)
        with pytest.raises(m27b.M27BError, match="unknown tensor"):
            e.load_tensor("blk.9.attn_q.weight", 12, 512, 1024, np.zeros(1024 * 288, np.uint8))
        with pytest.raises(m27b.M27BError, match="shape"):
            e.load_tensor("blk.0.attn_q.weight", 12, 512, 1000, np.zeros(1000 * 288, np.uint8))
    finally:
        e.close()


def test_engine_random_weights(m27b):
    # seeded synthetic weights: deterministic tokens, same across two engines
    c = dict(R.TINY, n_layers=4)
    runs = []
    for _ in range(2):
        e = _engine(m27b, c)
        try:
            e.random_weights(seed=11, sigma=0.02)
            assert e.weight_bytes_per_token() > 0
            tok, out = 3, []
            for pos in range(6):
                tok = e.decode_step(tok, pos)
                out.append(tok)
            runs.append(out)
        finally:
            e.close()
    assert runs[0] == runs[1]
    assert all(0 <= t < c["vocab"] for t in runs[0])
