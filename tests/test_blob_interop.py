"""`.m27b` interoperability with the reference's own reader and writer
(src/mono27b_blob.cpp, compiled in place from the reference checkout into
oracle/_ref/ref_blob_tool by oracle/build.py; CPU only, skipped without it).

* A blob written by m27b_blob_pack passes the reference's
  mono27b_validate_blob_file (header tags and layer counts, section bounds,
  tokenizer section, a target-matvec and an output-head entry) and
  mono27b_read_weights_section lists the same entries, field for field.
* A blob written by the reference's mono27b_write_stub_blob opens with
  m27b_blob_open: same entries, same payload bytes."""
import os
import subprocess

import numpy as np
import pytest

import _decode_ref as R


def _tool():
    from oracle import build as ob
    t = ob.build_reference_blob_tool()
    if not t or not os.path.exists(t):
        pytest.skip("reference .m27b tool not built (no reference checkout)")
    return t


def _run(*args):
    r = subprocess.run(list(args), capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    return r.stdout.splitlines()


def _entry_line(e):
    return (f"{e.name.decode()} {e.ggml_type} {e.source_model} {e.role} {e.row_elems} {e.row_count} "
            f"{e.data_offset} {e.data_bytes}")


def test_reference_validates_our_blob(orc, m27b, tmp_path):
    tool = _tool()
    model = R.make_model(orc, R.TINY, seed=0)
    tensors = [dict(name=n, ggml_type=t, row_elems=re, row_count=rc, data=d) for n, (t, re, rc, d) in model.items()]
    draft = R.make_model(orc, dict(R.TINY, n_layers=1), seed=1, qtype=8)
    tensors += [dict(name="blk.0.ffn_up.weight", ggml_type=8, row_elems=R.TINY["hidden"], row_count=R.TINY["ffn"],
                     data=draft["blk.0.ffn_up.weight"][3], source=2)]
    path = tmp_path / "ours.m27b"
    # the reference validates its fixed model constants: 64 target layers, 5 draft layers
    m27b.blob_pack(path, tensors, target_layers=64, draft_layers=5, vocab_size=R.TINY["vocab"])
    out = _run(tool, "validate", str(path))
    assert out[0] == f"valid {len(tensors)}", out[:2]
    b = m27b.Blob(path)
    try:
        assert out[1:] == [_entry_line(b.entry(i)[0]) for i in range(len(b))]
    finally:
        b.close()
    # layer counts other than the reference's constants are refused there
    bad = tmp_path / "bad.m27b"
    m27b.blob_pack(bad, tensors, target_layers=2, draft_layers=5, vocab_size=R.TINY["vocab"])
    assert _run(tool, "validate", str(bad))[0].startswith("invalid: invalid blob layer counts")


def test_we_read_the_reference_blob(m27b, tmp_path):
    tool = _tool()
    path = tmp_path / "ref.m27b"
    out = _run(tool, "write", str(path))
    assert out[0].startswith("written ")
    b = m27b.Blob(path)
    try:
        assert len(b) == int(out[0].split()[1])
        assert b.header.max_ctx_hint == 4096
        base = 0
        for i in range(len(b)):
            e, data = b.entry(i)
            assert _entry_line(e) == out[1 + i]
            want = ((np.arange(base, base + e.data_bytes) * 7 + 3) & 0xff).astype(np.uint8)
            assert np.array_equal(data, want), e.name
            base += e.data_bytes
    finally:
        b.close()
