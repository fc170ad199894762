"""The reference executor's C API as libm27b exports it (CPU only).

tests/abi/api_probe.cpp is compiled against the reference's own headers
(include/mono27b_config.h, include/mono27b_gguf.h, read in place from the
reference checkout) and against this project's include/mono27b_api.h: every
struct of the interface must have the same size and field offsets in both.
The reference-header build links libm27b.so and calls the entry points whose
argument checks answer before any CUDA call (the reference's error
convention: false plus a message).  Skipped where the reference checkout is
absent (its headers are not copied into this repository)."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PROBE = os.path.join(ROOT, "tests", "abi", "api_probe.cpp")
LIBDIR = os.path.join(ROOT, "mono-qwen27_b200", "lib")
CUDA_INC = "/usr/local/cuda/include"


def _ref_include():
    from oracle import build as ob
    inc = os.path.join(ob.REFERENCE_ROOT, "include")
    return inc if os.path.exists(os.path.join(inc, "mono27b_config.h")) else None


def _build(tmp_path, name, extra):
    exe = str(tmp_path / name)
    cmd = ["g++", "-std=c++17", "-O0", "-Wno-invalid-offsetof", "-I", os.path.join(ROOT, "include"), "-I", CUDA_INC,
           PROBE, "-o", exe] + extra
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def _run(exe, *args):
    r = subprocess.run([exe, *args], capture_output=True, text=True, timeout=120,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "")))
    assert r.returncode == 0, r.stderr
    return r.stdout


def test_struct_layouts_match_the_reference_headers(tmp_path, m27b):
    inc = _ref_include()
    if not inc:
        pytest.skip("reference checkout not present")
    ours = _run(_build(tmp_path, "probe_ours", []))
    ref = _run(_build(tmp_path, "probe_ref", ["-DM27B_PROBE_REFERENCE_HEADERS", "-I", inc, "-L", LIBDIR, "-lm27b",
                                              "-Wl,-rpath," + LIBDIR]))
    assert ours.count("\n") > 40
    assert ours == ref


def test_reference_header_program_links_and_calls(tmp_path, m27b):
    """A program written against the reference's headers (the executor API
    and, through M27B_EXTERNAL_WEIGHTVIEW, the matvec seam) links against
    libm27b and gets the reference's error convention back."""
    inc = _ref_include()
    if not inc:
        pytest.skip("reference checkout not present")
    exe = _build(tmp_path, "probe_ref", ["-DM27B_PROBE_REFERENCE_HEADERS", "-I", inc, "-L", LIBDIR, "-lm27b",
                                         "-Wl,-rpath," + LIBDIR])
    out = _run(exe, "--call")
    assert re.search(r"^load_weights 0 mono27b_engine_load_weights: token_embd.weight not found$", out, re.M), out
    assert "free_logits 1" in out and "free_state ok" in out and "argmax 0" in out
    assert re.search(r"^m27b_qmv 0 m27b_qmv: null activation pointer$", out, re.M), out
