"""PyTorch zip checkpoints over the C ABI (include/kokoro_b200.h, ``kk_pth_*``), mirroring the
reference's ``src/torchpt.rs``:

* ``load_kmodel_checkpoint``: kokoro-v1_0.pth, a dict of state dicts, as ``{"submodule.param":
  array}`` (a leading ``module.`` dropped), ``src/torchpt.rs:302-319``;
* ``load_voice_pack``: voices/<name>.pt, one ``[rows, 1, 256]`` tensor, ``src/torchpt.rs:322-335``.

Only STORED zip entries, a small pickle opcode set (interpreted, never executed) and the globals
``collections.OrderedDict``, ``torch._utils._rebuild_tensor_v2`` and ``torch.FloatStorage`` are
accepted; anything else raises ``PthError`` naming it.
"""
from __future__ import annotations

import ctypes
from collections import OrderedDict

import numpy as np

from .engine import load_library

KK_PTH_CHECKPOINT, KK_PTH_VOICE = 0, 1


class PthError(RuntimeError):
    pass


def _read(path: str, kind: int) -> "OrderedDict[str, np.ndarray]":
    lib = load_library()
    h = ctypes.c_void_p()
    if lib.kk_pth_open(str(path).encode(), kind, ctypes.byref(h)) != 0:
        raise PthError(lib.kk_pth_error().decode())
    try:
        out = OrderedDict()
        dims = (ctypes.c_int64 * 8)()
        for i in range(lib.kk_pth_count(h)):
            nd = lib.kk_pth_shape(h, i, dims, 8)
            shape = tuple(dims[d] for d in range(nd))
            n = int(np.prod(shape)) if shape else 1
            ptr = lib.kk_pth_data(h, i)
            a = np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctypes.c_float)), shape=(n,)) if n else np.empty(0)
            out[lib.kk_pth_name(h, i).decode()] = a.astype(np.float32, copy=True).reshape(shape)
        return out
    finally:
        lib.kk_pth_close(h)


def load_kmodel_checkpoint(path: str) -> "OrderedDict[str, np.ndarray]":
    return _read(path, KK_PTH_CHECKPOINT)


def load_voice_pack(path: str) -> np.ndarray:
    return _read(path, KK_PTH_VOICE)["voice"]
