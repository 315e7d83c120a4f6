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
def reference_dir():
    """The reference checkout: $KOKORO_REFERENCE, else a ``reference`` directory beside this
    repository; None when neither exists (a GPU box carries only the prebuilt oracle/_ref)."""
    d = os.environ.get("KOKORO_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return d if os.path.isdir(d) else None


def ref_src():
    d = reference_dir()
    return None if d is None else os.path.join(d, "kernels", "kokoro.cu")


def build() -> str:
    src = ref_src()
    if src is None or not os.path.exists(src):
        raise FileNotFoundError("reference kernel source not found (set KOKORO_REFERENCE)")
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = [os.environ.get("NVCC", "nvcc"), "-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-fmad=true",
           "-O3", src, "-o", CUBIN]
    subprocess.run(cmd, check=True)
    return CUBIN


if __name__ == "__main__":
    print(build(), file=sys.stdout)
