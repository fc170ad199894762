"""Tensor-parallel decode on CPU: the engine's partition (m27b_engine_partition,
pure host code in libm27b) and the sharded decode math, run as gloo ranks.

The sharded decode uses the same partition the engine uses on the GPU: query
heads and their kv heads, FFN rows in whole 256-value blocks, o_proj / down
split along their input dimension with an all-reduce of the 5120-wide (here
512-wide) hidden state, vocabulary rows for the head.  Its hidden state must
match the single-rank reference to fp32 reduction order, and the global argmax
of the per-rank logits must match."""
import os
import socket

import numpy as np
import pytest

import _decode_ref as R


def _cfg(m27b, **kw):
    d = dict(m27b.QWEN27)
    d.update(kw)
    return m27b.model_config(**d)


def test_partition_qwen_shapes(m27b):
    H, KV, F, V = 24, 4, 17408, 248320
    for t in (1, 2, 4, 8):
        parts = [m27b.partition(_cfg(m27b, tp_rank=r, tp_size=t)) for r in range(t)]
        assert sum(p.n_q for p in parts) == H
        assert [p.q_lo for p in parts] == [sum(q.n_q for q in parts[:r]) for r in range(t)]
        for p in parts:
            # every local query head's kv head is local
            for h in range(p.q_lo, p.q_lo + p.n_q):
                assert p.kv_lo <= h // (H // KV) < p.kv_lo + p.n_kv
            assert p.n_f % 256 == 0 and p.f_lo % 256 == 0 and (p.n_q * 256) % 256 == 0
        assert sum(p.n_f for p in parts) == F and parts[-1].f_lo + parts[-1].n_f == F
        assert sum(p.n_v for p in parts) == V and parts[-1].v_lo + parts[-1].n_v == V
        # kv heads are replicated only when there are more ranks than kv heads
        assert sum(p.n_kv for p in parts) == max(KV, t)
    p8 = [m27b.partition(_cfg(m27b, tp_rank=r, tp_size=8)) for r in range(8)]
    # 68 blocks of down over 8 ranks: 8 or 9 blocks each (uneven split)
    assert sorted({p.n_f // 256 for p in p8}) == [8, 9]


HYB_OK = dict(attn_interval=4, ssm_d_inner=6144, ssm_d_state=128, ssm_dt_rank=48, ssm_n_group=16, ssm_conv_kern=4)


def _hyb(**kw):
    d = dict(HYB_OK)
    d.update(kw)
    return d


@pytest.mark.parametrize("bad", [dict(tp_size=5), dict(tp_rank=2, tp_size=2), dict(hidden=5000), dict(head_dim=288),
                                 dict(n_head=24, n_kv_head=5), dict(n_head=36, n_kv_head=4), dict(n_rot=3),
                                 dict(ffn=256, tp_size=2), dict(attn_interval=-1),
                                 _hyb(tp_size=2), _hyb(ssm_d_state=64), _hyb(ssm_dt_rank=47, ssm_d_inner=47 * 128),
                                 _hyb(ssm_d_inner=6000), _hyb(ssm_n_group=0), _hyb(ssm_conv_kern=1),
                                 _hyb(ssm_conv_kern=9)])
def test_partition_rejects(m27b, bad):
    kw = dict(tp_rank=0, tp_size=1)
    kw.update(bad)
    with pytest.raises(m27b.M27BError):
        m27b.partition(_cfg(m27b, **kw))


def test_partition_accepts_the_hybrid_layout(m27b):
    p = m27b.partition(_cfg(m27b, tp_rank=0, tp_size=1, **HYB_OK))
    assert p.n_q == 24 and p.n_f == 17408 and p.n_v == 248320


# Shape that exercises shared kv heads (4 q heads per kv head) and an uneven
# FFN split (5 blocks over 2 or 4 ranks).
TP_CFG = dict(n_layers=2, hidden=512, ffn=1280, n_head=8, n_kv_head=2, head_dim=128, vocab=1001, n_rot=64,
              rope_theta=1e7, rms_eps=1e-6)
TOKENS = [7, 500, 3]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_rank(rank, world, port, out_dir):
    import sys
    import torch
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (here, root, os.path.join(root, "mono-qwen27_b200")):
        sys.path.insert(0, p)
    import m27b
    from oracle import oracle as orc
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        d = dict(m27b.QWEN27)
        d.update(TP_CFG)
        p = m27b.partition(m27b.model_config(tp_rank=rank, tp_size=world, **d))
        part = {f: getattr(p, f) for f, _ in m27b.Partition._fields_}

        def allreduce(v):
            t = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32))
            dist.all_reduce(t)
            return t.numpy()

        model = R.make_model(orc, TP_CFG, seed=3)
        dec = R.RefDecoder(orc, model, TP_CFG, part=part, rank=rank, allreduce=allreduce)
        hid, best = [], []
        tok = TOKENS[0]
        for pos in range(len(TOKENS)):
            lg, h = dec.step(tok, pos)
            # global first argmax from the per-rank (max, index) pairs
            i = int(np.argmax(lg))
            pair = torch.tensor([float(lg[i]), float(p.v_lo + i)], dtype=torch.float64)
            allp = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
            dist.all_gather(allp, pair)
            m = max(a[0].item() for a in allp)
            g = min(int(a[1].item()) for a in allp if a[0].item() == m)
            hid.append(h)
            best.append(g)
            tok = TOKENS[pos + 1] if pos + 1 < len(TOKENS) else g
        if rank == 0:
            np.savez(os.path.join(out_dir, f"tp{world}.npz"), hidden=np.array(hid), best=np.array(best))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_sharded_decode_gloo(orc, world, tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_tp_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    got = np.load(tmp_path / f"tp{world}.npz")
    model = R.make_model(orc, TP_CFG, seed=3)
    ref = R.RefDecoder(orc, model, TP_CFG)
    tok = TOKENS[0]
    for pos in range(len(TOKENS)):
        lg, h = ref.step(tok, pos)
        # partial sums added in a different order: fp32 reduction-order tolerance
        assert orc.rel_l2(got["hidden"][pos], h) <= 1e-5, pos
        assert got["best"][pos] == orc.argmax(lg)
        tok = TOKENS[pos + 1] if pos + 1 < len(TOKENS) else int(got["best"][pos])


def test_delta_rule_reference_properties():
    """The decode reference's gated delta rule (the DeltaNet recurrence the
    GPU kernel is checked against) does what the rule defines: with beta = 1
    and no decay, writing value v at unit key k makes S k = v and leaves
    S unchanged on keys orthogonal to k; a decay e^g scales the old state."""
    import numpy as np
    import _decode_ref as R
    rng = np.random.default_rng(0)
    dk = dv = 8
    S = rng.standard_normal((dv, dk)).astype(np.float32)
    k = np.zeros(dk, np.float32)
    k[3] = 1.0
    other = np.zeros(dk, np.float32)
    other[5] = 1.0
    v = rng.standard_normal(dv).astype(np.float32)
    before_other = S @ other
    R.delta_rule(S, k, k, v, 1.0, 0.0)
    assert np.allclose(S @ k, v, atol=1e-6)
    assert np.allclose(S @ other, before_other, atol=1e-6)
    # beta = 0: only the decay acts
    S2 = rng.standard_normal((dv, dk)).astype(np.float32)
    want = np.float32(np.exp(-0.5)) * S2
    R.delta_rule(S2, k, k, v, 0.0, -0.5)
    assert np.allclose(S2, want, atol=1e-6)
