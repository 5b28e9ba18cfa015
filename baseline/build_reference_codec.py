"""Compile the reference TACO codec (TempName-5090 src/taco/codec.cu), unmodified,
for sm_100a into baseline/_ref/libref_taco_codec.so.  Used only by
tests/test_reference_parity_gpu.py to check byte/bit parity of this framework's
codec kernels against the reference's own kernels on the same GPU.

The reference has no installable package, so its codec source is staged
verbatim (never edited) under baseline/_ref/src/taco/ -- the git-ignored
location of the reference arm, which travels with the repository to GPU boxes
-- and built from there.  The source is taken from baseline/_ref if present,
else from the reference checkout (--reference / TN5B_REFERENCE).

    python baseline/build_reference_codec.py [--reference DIR]
"""
import argparse
import hashlib
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
STAGED = os.path.join(REF_DIR, "src", "taco", "codec.cu")
LIB = os.path.join(REF_DIR, "libref_taco_codec.so")


def find_source(reference=None):
    """Path of the reference codec source, staging it from the checkout if needed."""
    if os.path.exists(STAGED):
        return STAGED
    reference = reference or os.environ.get("TN5B_REFERENCE", "/root/reference")
    src = os.path.join(reference, "src", "taco", "codec.cu")
    if not os.path.exists(src):
        return None
    os.makedirs(os.path.dirname(STAGED), exist_ok=True)
    shutil.copyfile(src, STAGED)  # verbatim: the reference's own file, for the oracle build only
    return STAGED


def build(reference=None) -> str:
    src = find_source(reference)
    if src is None:
        raise FileNotFoundError("reference codec source not found (baseline/_ref or the reference checkout)")
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--fmad=false", "-std=c++17",
           "-Xcompiler", "-fPIC", "-shared", "-cudart=shared", "-o", LIB, src]
    subprocess.run(cmd, check=True)
    with open(src, "rb") as f:
        digest = hashlib.sha256(f.read()).hexdigest()
    with open(LIB + ".source-sha256", "w") as f:
        f.write(digest + "\n")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    print(build(ap.parse_args().reference))
