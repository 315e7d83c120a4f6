"""Build the reference's own CUDA kernels from source for the B200: TEST INFRASTRUCTURE ONLY.

Compiles kernels/kokoro.cu of the reference crate, unmodified, with the reference's flags
(build.rs:36: -fmad=true -O3) but for sm_100a instead of compute_89 PTX, into
oracle/_ref/kokoro_ref.cubin. tests/golden/make_ref_golden.py loads that cubin on a GPU box and
records the reference kernels' outputs on seeded inputs (golden vectors for the oracle). Nothing
of the product links or loads it.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
CUBIN = os.path.join(OUT_DIR, "kokoro_ref.cubin")
REF_SRC = os.environ.get("KOKORO_REFERENCE", "/root/reference") + "/kernels/kokoro.cu"


def build() -> str:
    if not os.path.exists(REF_SRC):
        raise FileNotFoundError(f"reference kernel source not found: {REF_SRC}")
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = ["/usr/local/cuda/bin/nvcc", "-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-fmad=true",
           "-O3", REF_SRC, "-o", CUBIN]
    subprocess.run(cmd, check=True)
    return CUBIN


if __name__ == "__main__":
    print(build(), file=sys.stdout)
