"""`.m27b` blob packer / reader (include/m27b_blob.h) and the GGUF packer CLI
(mono-qwen27_b200/m27b_pack.py), on the CPU.

The layout follows the reference's include/mono27b_format.h: a 136-byte
header, 24-byte section descriptors, a 32-byte tokenizer section, a 16-byte
weights section and 104-byte entries whose data offsets are relative to the
weights section."""
import ctypes
import os

import numpy as np
import pytest

import _decode_ref as R


def test_struct_sizes(m27b):
    assert ctypes.sizeof(m27b.BlobHeader) == 136
    assert ctypes.sizeof(m27b.WeightEntry) == 104


def _pack_tiny(orc, m27b, path, drop=()):
    model = R.make_model(orc, R.TINY, seed=0)
    tensors = [dict(name=n, ggml_type=t, row_elems=re, row_count=rc, data=d)
               for n, (t, re, rc, d) in model.items() if n not in drop]
    m27b.blob_pack(path, tensors, target_layers=R.TINY["n_layers"], vocab_size=R.TINY["vocab"])
    return model


def test_pack_open_roundtrip(orc, m27b, tmp_path):
    path = tmp_path / "tiny.m27b"
    model = _pack_tiny(orc, m27b, path)
    b = m27b.Blob(path)
    h = b.header
    assert h.magic == 0x4237324D and h.schema_version == 4 and h.section_count == 2
    assert h.file_bytes == os.path.getsize(path) and h.target_layers == R.TINY["n_layers"]
    assert bytes(h.target_arch).rstrip(b"\0") == b"qwen35"
    assert len(b) == len(model)
    raw = path.read_bytes()
    sec = np.frombuffer(raw[h.section_table_offset:h.section_table_offset + 48], dtype=np.uint64).reshape(2, 3)
    w_off = int(sec[1, 1])  # weights section offset (second descriptor: kind/reserved, offset, bytes)
    for i in range(len(b)):
        e, data = b.entry(i)
        name = e.name.decode()
        t, re, rc, d = model[name]
        assert (e.ggml_type, e.row_elems, e.row_count) == (t, re, rc)
        want = np.ascontiguousarray(d).view(np.uint8).reshape(-1)
        assert np.array_equal(data, want)
        # data offsets are relative to the weights section
        assert np.array_equal(np.frombuffer(raw[w_off + e.data_offset:w_off + e.data_offset + e.data_bytes], np.uint8),
                              want)
        expect_role = 3 if name == "output.weight" else (1 if t != 0 and rc > 1 else 0)
        assert e.role == expect_role and e.source_model == 1
    b.close()


def test_open_rejects(orc, m27b, tmp_path):
    good = tmp_path / "good.m27b"
    _pack_tiny(orc, m27b, good)
    raw = bytearray(good.read_bytes())
    cases = {
        "bad magic": raw[:0] + b"XXXX" + raw[4:],
        "file size": raw[:-1],
        "schema": raw[:4] + (5).to_bytes(4, "little") + raw[8:],
    }
    for msg, data in cases.items():
        p = tmp_path / f"bad_{msg.replace(' ', '_')}.m27b"
        p.write_bytes(bytes(data))
        with pytest.raises(m27b.M27BError, match=msg.split()[0]):
            m27b.Blob(p)
    nohead = tmp_path / "nohead.m27b"
    _pack_tiny(orc, m27b, nohead, drop=("output.weight",))
    with pytest.raises(m27b.M27BError, match="output head"):
        m27b.Blob(nohead)
    with pytest.raises(m27b.M27BError, match="missing blob"):
        m27b.Blob(tmp_path / "absent.m27b")


def test_gguf_packer_cli(orc, m27b, tmp_path):
    gguf = pytest.importorskip("gguf")
    import m27b_pack
    model = R.make_model(orc, dict(R.TINY, n_layers=1), seed=5)
    src = tmp_path / "tiny.gguf"
    w = gguf.GGUFWriter(str(src), "qwen35")
    for name, (t, re, rc, d) in model.items():
        if t == 0:
            w.add_tensor(name, np.asarray(d, dtype=np.float32).reshape(rc, re) if rc > 1 else np.asarray(d, np.float32))
        else:
            w.add_tensor(name, np.ascontiguousarray(d).reshape(rc, -1), raw_dtype=gguf.GGMLQuantizationType(t))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    out = tmp_path / "tiny.m27b"
    assert m27b_pack.main(["--target", str(src), "--out", str(out)]) == 0
    b = m27b.Blob(out)
    assert b.header.target_layers == 1
    got = {e.name.decode(): (e, d) for e, d in b.entries()}
    assert set(got) == set(model)
    for name, (t, re, rc, d) in model.items():
        e, data = got[name]
        assert (e.ggml_type, e.row_elems, e.row_count) == (t, re, rc), name
        assert np.array_equal(data, np.ascontiguousarray(d).view(np.uint8).reshape(-1)), name
