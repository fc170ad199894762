"""Tensor-parallel decode on 2 GPUs (one process per GPU, NCCL between them)
against the single-rank decode reference.  Skipped with fewer than 2 GPUs.

Every rank loads the full GGUF-named tensors and keeps its shard; the hidden
state after the last all-reduce is replicated on every rank and must match the
reference within the matvec tolerance, and all ranks must return the same
greedy tokens."""
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


def _rank(rank, world, out_dir):
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
        for name, (qtype, row_elems, row_count, data) in R.make_model(orc, TP_CFG, seed=3).items():
            e.load_tensor(name, qtype, row_elems, row_count, data)
        hid, toks = [], []
        for pos, t in enumerate(PROMPT):
            toks.append(e.decode_step(t, pos))
            hid.append(e.hidden())
        gen = e.generate(toks[-1], len(PROMPT), N_GEN)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), hidden=np.array(hid), toks=np.array(toks), gen=gen)
    finally:
        e.close()


def test_tp2_decode(orc, tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_rank, args=(2, str(tmp_path)), nprocs=2, join=True)
    r = [np.load(tmp_path / f"rank{i}.npz") for i in range(2)]
    assert (r[0]["toks"] == r[1]["toks"]).all() and (r[0]["gen"] == r[1]["gen"]).all()
    np.testing.assert_array_equal(r[0]["hidden"], r[1]["hidden"])
    ref = R.RefDecoder(orc, R.make_model(orc, TP_CFG, seed=3), TP_CFG)
    for pos, t in enumerate(PROMPT):
        lg, h = ref.step(t, pos)
        assert orc.rel_l2(r[0]["hidden"][pos], h) <= 1e-3, pos
        top = np.sort(lg)[-2:]
        if top[1] - top[0] > 1e-3 * np.abs(lg).max():
            assert r[0]["toks"][pos] == orc.argmax(lg), pos
