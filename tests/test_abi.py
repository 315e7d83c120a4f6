"""The C ABI library: builds, loads without a GPU, exports every declared symbol, fails loudly."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    h = open(os.path.join(ROOT, "include", "kokoro_b200.h")).read()
    return sorted(set(re.findall(r"KK_API\s+[\w\s\*]+?\b(kk_\w+)\s*\(", h)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ("kk_create", "kk_destroy", "kk_forward_batch", "kk_decode_batch", "kk_fetch_audio",
              "kk_last_error"):
        assert s in syms


def test_library_exports_every_declared_symbol(kk):
    lib = kk.load_library()
    for s in declared_symbols():
        assert hasattr(lib, s), s


def test_create_without_gpu_fails_with_status(kk, tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = kk.load_library()
    h = ctypes.c_void_p()
    st = lib.kk_create(str(tmp_path / "missing.safetensors").encode(), 0, 0, ctypes.byref(h))
    assert st != 0 and not h.value
    assert lib.kk_last_error(None)
    lib.kk_destroy(None)  # no-op


def test_gpu_kokoro_raises_kokoro_error(kk, tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(kk.KokoroError):
        kk.GpuKokoro(str(tmp_path / "missing.safetensors"), 0, "bf16")
