"""Build recipe for the CPU oracle (test infrastructure only).

* ``liboracle.so`` — the C restatement of ggml's k-quant semantics
  (``ggml_semantics.c``), compiled with ``-ffp-contract=off`` so that every
  dequantized value is an unfused ``fl(fl(d*sc)*q) - fl(dmin*m)``.
* ``_ref/official_dequant`` — the reference's own q4_K dequant known-answer
  program, compiled from ``debug/official_dequant.c`` where it lies in the
  reference checkout (only when that checkout is present; the built binary is
  git-ignored but travels with the tree).  Nothing is copied out of the
  reference: gcc reads the file in place.
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_KAT = os.path.join(REF_DIR, "official_dequant")
REF_GPU = os.path.join(REF_DIR, "libref_gpu.so")
REF_BLOB = os.path.join(REF_DIR, "ref_blob_tool")
# The reference checkout: M27B_REFERENCE_ROOT, else a directory named
# "reference" beside this repository's own directory (absent on a GPU box,
# where the programs built from it travel prebuilt).
REFERENCE_ROOT = os.environ.get("M27B_REFERENCE_ROOT") or os.path.join(
    os.path.dirname(os.path.dirname(HERE)), "reference")


def _stale(out, srcs):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs)


def build_oracle(force=False):
    src = os.path.join(HERE, "ggml_semantics.c")
    if force or _stale(LIB, [src, __file__]):
        cmd = ["gcc", "-O2", "-march=x86-64-v2", "-fopenmp", "-ffp-contract=off", "-fPIC",
               "-shared", "-std=c11", "-Wall", "-Wextra", "-o", LIB, src, "-lm"]
        subprocess.run(cmd, check=True)
    return LIB


def build_reference_kat(force=False):
    """Compile the reference's q4_K dequant KAT program, if the reference is mounted."""
    src = os.path.join(REFERENCE_ROOT, "debug", "official_dequant.c")
    if not os.path.exists(src):
        return REF_KAT if os.path.exists(REF_KAT) else None
    os.makedirs(REF_DIR, exist_ok=True)
    if force or _stale(REF_KAT, [src]):
        subprocess.run(["gcc", "-O0", "-ffp-contract=off", "-fno-strict-aliasing", "-o", REF_KAT, src, "-lm"],
                       check=True)
    return REF_KAT


def build_reference_gpu(force=False):
    """Compile the reference executor's CUDA file in place, through
    ref_gpu_harness.cu, into oracle/_ref/libref_gpu.so (sm_100a, the
    reference's own CUDA flags) — the "reference kernels on B200" comparison
    arm.  Only when the reference checkout is present; returns the library
    path if it exists."""
    src = os.path.join(REFERENCE_ROOT, "src", "mono27b_executor.cu")
    harness = os.path.join(HERE, "ref_gpu_harness.cu")
    if not os.path.exists(src):
        return REF_GPU if os.path.exists(REF_GPU) else None
    os.makedirs(REF_DIR, exist_ok=True)
    if force or _stale(REF_GPU, [src, harness]):
        nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
        subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "--use_fast_math",
                        "--default-stream=per-thread", "-shared", "-Xcompiler", "-fPIC", "-Xcompiler",
                        "-fvisibility=hidden", "-w",
                        "-I", os.path.join(REFERENCE_ROOT, "include"), "-I", os.path.join(REFERENCE_ROOT, "src"),
                        harness, "-o", REF_GPU], check=True)
    return REF_GPU


def build_reference_blob_tool(force=False):
    """Compile the reference's .m27b reader/writer (src/mono27b_blob.cpp, in
    place) with ref_blob_tool.cpp into oracle/_ref/ref_blob_tool, when the
    reference checkout is present."""
    src = os.path.join(REFERENCE_ROOT, "src", "mono27b_blob.cpp")
    tool = os.path.join(HERE, "ref_blob_tool.cpp")
    if not os.path.exists(src):
        return REF_BLOB if os.path.exists(REF_BLOB) else None
    os.makedirs(REF_DIR, exist_ok=True)
    if force or _stale(REF_BLOB, [src, tool]):
        subprocess.run(["g++", "-std=c++17", "-O1", "-w", "-I", os.path.join(REFERENCE_ROOT, "include"), tool, src,
                        "-o", REF_BLOB], check=True)
    return REF_BLOB


if __name__ == "__main__":
    print(build_oracle(force=True))
    print(build_reference_kat(force=True))
    print(build_reference_gpu(force=True))
    print(build_reference_blob_tool(force=True))
