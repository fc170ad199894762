"""Tensor-parallel decode on 2 GPUs (one process per GPU) against the
single-rank decode reference, with the hidden-state all-reduces done by NCCL
or by the fused NVLink path (matvec rows pushed into every rank's window).
Skipped with fewer than 2 GPUs.

Every rank loads the full GGUF-named tensors and keeps its shard; the hidden
state after the last all-reduce is replicated on every rank and must match the
reference within the matvec tolerance, all ranks must return the same greedy
tokens, and the two all-reduce paths must agree (both add the same two
partials; their RMSNorm reductions run in different orders, so a q8_K code
can round the other way: 1e-4).  A verify pass over the generated
continuation (its all-reduces on NCCL, also on the engine that decodes with
the fused path) must return the greedy continuation on every rank, and the
fused decode step must carry on after it."""
import os
import time

import numpy as np
import pytest

import _decode_ref as R

pytestmark = pytest.mark.gpu

TP_CFG = dict(n_layers=2, hidden=512, ffn=1280, n_head=8, n_kv_head=2, head_dim=128, vocab=1001, n_rot=64,
              rope_theta=1e7, rms_eps=1e-6)
PROMPT = [7, 500, 3, 44]
N_GEN = 4


def _rank(rank, world, out_dir, comm):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (here, root, os.path.join(root, "mono-qwen27_b200")):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import m27b
    from oracle import oracle as orc
    torch.cuda.set_device(rank)
    d = dict(m27b.QWEN27)
    d.update(TP_CFG)
    e = m27b.Engine(m27b.model_config(max_ctx=32, tp_rank=rank, tp_size=world, **d))
    try:
        idf = os.path.join(out_dir, "nccl.id")
        if rank == 0:
            with open(idf + ".tmp", "wb") as f:
                f.write(m27b.nccl_unique_id())
            os.replace(idf + ".tmp", idf)
        deadline = time.time() + 120
        while not os.path.exists(idf):
            if time.time() > deadline:
                raise TimeoutError("no NCCL id from rank 0")
            time.sleep(0.05)
        with open(idf, "rb") as f:
            e.set_nccl(f.read())
        if comm == "p2p":
            e.enable_p2p()
        for name, (qtype, row_elems, row_count, data) in R.make_model(orc, TP_CFG, seed=3).items():
            e.load_tensor(name, qtype, row_elems, row_count, data)
        hid, toks = [], []
        for pos, t in enumerate(PROMPT):
            toks.append(e.decode_step(t, pos))
            hid.append(e.hidden())
        gen = e.generate(toks[-1], len(PROMPT), N_GEN)
        # a verify pass over the generated continuation (its all-reduces on
        # NCCL in both modes): the greedy token after each drafted token
        vt = [int(toks[-1])] + [int(x) for x in gen[:N_GEN - 1]]
        vnext = e.verify(vt, len(PROMPT))
        after = e.decode_step(int(gen[-1]), len(PROMPT) + N_GEN)  # the fused step still works afterwards
        np.savez(os.path.join(out_dir, f"{comm}_rank{rank}.npz"), hidden=np.array(hid), toks=np.array(toks), gen=gen,
                 vnext=np.array(vnext), after=np.array([after]))
    finally:
        e.close()


def _run(tmp_path, comm):
    import torch.multiprocessing as mp
    d = tmp_path / comm
    d.mkdir()
    mp.spawn(_rank, args=(2, str(d), comm), nprocs=2, join=True)
    return [np.load(d / f"{comm}_rank{i}.npz") for i in range(2)]


def test_tp2_decode(orc, tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = {comm: _run(tmp_path, comm) for comm in ("nccl", "p2p")}
    ref = R.RefDecoder(orc, R.make_model(orc, TP_CFG, seed=3), TP_CFG)
    ref_out = [ref.step(t, pos) for pos, t in enumerate(PROMPT)]
    for comm, r in res.items():
        assert (r[0]["toks"] == r[1]["toks"]).all() and (r[0]["gen"] == r[1]["gen"]).all(), comm
        np.testing.assert_array_equal(r[0]["hidden"], r[1]["hidden"])
        for pos, (lg, h) in enumerate(ref_out):
            assert orc.rel_l2(r[0]["hidden"][pos], h) <= 1e-3, (comm, pos)
            top = np.sort(lg)[-2:]
            if top[1] - top[0] > 1e-3 * np.abs(lg).max():
                assert r[0]["toks"][pos] == orc.argmax(lg), (comm, pos)
    a, b = res["nccl"][0], res["p2p"][0]
    for pos in range(len(PROMPT)):
        assert orc.rel_l2(b["hidden"][pos], a["hidden"][pos]) <= 1e-4, pos
    assert (a["toks"] == b["toks"]).all() and (a["gen"] == b["gen"]).all()
    for comm, r in res.items():
        # verify agrees with the greedy continuation and across ranks, on both paths
        assert (r[0]["vnext"] == r[1]["vnext"]).all() and (r[0]["after"] == r[1]["after"]).all(), comm
        assert (r[0]["vnext"] == r[0]["gen"]).all(), (comm, r[0]["vnext"], r[0]["gen"])
    assert (a["after"] == b["after"]).all()
