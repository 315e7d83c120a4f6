"""Build libkokoro_b200.so in-tree with nvcc for sm_100a (no torch dependency in the library)."""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libkokoro_b200.so")
SOURCES = ["kk_engine.cu", "kk_conv_simt.cu", "kk_kernels.cu", "kk_lstm.cu", "kk_tc.cu", "kk_attn_tc.cu", "kk_selftest.cu", "kk_weights.cpp", "kk_wav.cpp", "kk_pth.cpp"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
COMPILE = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [
        os.path.join(HERE, "..", "include", "kokoro_b200.h"), __file__]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every CUDA/C++ source of the engine into one shared library; returns its path."""
    if not force and not _stale():
        return LIB
    objs = []
    tmpdir = os.path.join(HERE, "_build")
    os.makedirs(tmpdir, exist_ok=True)
    procs = []
    for src in SOURCES:
        obj = os.path.join(tmpdir, src + ".o")
        cmd = [NVCC, *COMPILE, "-c", os.path.join(CSRC, src), "-o", obj]
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = []
    for src, p in procs:
        out = p.communicate()[0].decode()
        if p.returncode != 0:
            failed.append(f"--- {src}\n{out}")
        elif verbose and out.strip():
            print(f"--- {src}\n{out}")
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    link = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC", *objs,
            "-o", LIB + ".tmp", "-lcuda"]
    r = subprocess.run(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n" + r.stdout.decode())
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
