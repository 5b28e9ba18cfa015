"""Compile the reference TACO codec (TempName-5090 src/taco/codec.cu), unmodified,
for sm_100a into baseline/_ref/libref_taco_codec.so (git-ignored).  Used only by
tests/test_reference_parity_gpu.py to check byte/bit parity of this framework's
codec kernels against the reference's own kernels on the same GPU.

    python baseline/build_reference_codec.py [--reference /path/to/reference]
"""
import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build(reference: str) -> str:
    src = os.path.join(reference, "src", "taco", "codec.cu")
    out_dir = os.path.join(HERE, "_ref")
    os.makedirs(out_dir, exist_ok=True)
    out = os.path.join(out_dir, "libref_taco_codec.so")
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--fmad=false", "-std=c++17",
           "-Xcompiler", "-fPIC", "-shared", "-cudart=shared", "-o", out, src]
    subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TN5B_REFERENCE", "/root/reference"))
    print(build(ap.parse_args().reference))
