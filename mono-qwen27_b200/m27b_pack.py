#!/usr/bin/env python
"""Pack GGUF tensors into a mono27b `.m27b` blob (the reference's mono27b_pack,
absent from its source tree): the target model's tensors (source 1) and,
optionally, a draft model's (source 2), each as a raw GGUF block payload
with its name, type and shape; output.weight is the output head, quantized
2-D tensors are matvecs, the rest (norms) role 0.

    python mono-qwen27_b200/m27b_pack.py --target model.gguf [--draft draft.gguf] --out model.m27b

Reads GGUF files with the `gguf` Python package; the writing is the C ABI's
m27b_blob_pack (libm27b).
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import m27b  # noqa: E402


def gguf_tensors(path, source):
    """Tensors of a GGUF file as packer dicts, plus (layers, arch, vocab)."""
    import numpy as np
    from gguf import GGUFReader
    r = GGUFReader(path)
    out = []
    layers = set()
    for t in r.tensors:
        dims = [int(d) for d in t.shape]
        row_elems = dims[0]
        row_count = int(np.prod(dims[1:])) if len(dims) > 1 else 1
        out.append(dict(name=t.name, ggml_type=int(t.tensor_type), row_elems=row_elems, row_count=row_count,
                        data=np.ascontiguousarray(t.data).view(np.uint8).reshape(-1), source=source))
        if t.name.startswith("blk."):
            layers.add(int(t.name.split(".")[1]))
    arch = "qwen35"
    f = r.fields.get("general.architecture")
    if f is not None:
        arch = bytes(f.parts[f.data[0]]).decode()
    vocab = next((t["row_count"] for t in out if t["name"] in ("output.weight", "token_embd.weight")), 1)
    return out, len(layers), arch, vocab


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--target", required=True, help="target model GGUF")
    ap.add_argument("--draft", help="draft model GGUF")
    ap.add_argument("--out", required=True)
    ap.add_argument("--max-ctx", type=int, default=8192)
    a = ap.parse_args(argv)
    tensors, t_layers, t_arch, vocab = gguf_tensors(a.target, m27b.SOURCE_TARGET)
    d_layers, d_arch = 0, "dflash-draft"
    if a.draft:
        dt, d_layers, d_arch, _ = gguf_tensors(a.draft, m27b.SOURCE_DRAFT)
        tensors += dt
    m27b.blob_pack(a.out, tensors, max_ctx_hint=a.max_ctx, target_layers=t_layers, draft_layers=d_layers,
                   target_arch=t_arch[:15], draft_arch=d_arch[:15], vocab_size=vocab)
    print(f"{a.out}: {len(tensors)} tensors, {os.path.getsize(a.out)} bytes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
