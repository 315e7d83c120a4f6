"""WAV output, mirroring the reference's `src/wav.rs` over the C ABI (include/kokoro_b200.h):

* ``Format`` (``Pcm16`` / ``Float32``), ``HEADER_LEN``, ``MAX_DATA_BYTES``: ``src/wav.rs:10-24``
* ``check_riff_size`` / ``header``: ``src/wav.rs:33-61`` (the 4 GiB limit is enforced, never wrapped)
* ``encode``: ``src/wav.rs:63-87`` (PCM_16 = sample * 0x7FFF rounded half to even, clamped, clipped
  samples counted)
* ``write_atomic``: ``src/wav.rs:89-107``; ``read_canonical``: ``src/wav.rs:109-130``
* ``assemble``: ``src/wav.rs:132-187`` (in-order concatenation with a sha256 check of every part,
  temporary file + rename)

Errors raise ``WavError`` (the reference's ``anyhow`` errors), with the same messages.
"""
from __future__ import annotations

import ctypes
import enum
import os
from dataclasses import dataclass
from typing import List, Sequence, Tuple

import numpy as np

from .engine import load_library

HEADER_LEN = 44
MAX_DATA_BYTES = 0xFFFFFFFF - 36


class Format(enum.IntEnum):
    Pcm16 = 0
    Float32 = 1


class WavError(RuntimeError):
    pass


@dataclass
class Encoded:
    bytes: bytes
    clipped: int


@dataclass
class Assembled:
    sha256: str
    data_bytes: int
    samples: int


def _lib():
    return load_library()


def _err(lib) -> WavError:
    return WavError(lib.kk_wav_error().decode())


def check_riff_size(data_bytes: int) -> None:
    header(Format.Pcm16, 24000, data_bytes)


def header(fmt: Format, sample_rate: int, data_bytes: int) -> bytes:
    lib = _lib()
    out = (ctypes.c_uint8 * HEADER_LEN)()
    if data_bytes < 0 or lib.kk_wav_header(int(fmt), sample_rate, data_bytes, out) != 0:
        raise _err(lib)
    return bytes(out)


def encode(audio: np.ndarray, sample_rate: int, fmt: Format) -> Encoded:
    lib = _lib()
    a = np.ascontiguousarray(audio, np.float32)
    n = ctypes.c_int64()
    lib.kk_wav_encode(a.ctypes.data, a.size, sample_rate, int(fmt), None, 0, ctypes.byref(n), None)
    buf = np.empty(n.value, np.uint8)
    clipped = ctypes.c_int64()
    if lib.kk_wav_encode(a.ctypes.data, a.size, sample_rate, int(fmt), buf.ctypes.data, buf.size, ctypes.byref(n),
                         ctypes.byref(clipped)) != 0:
        raise _err(lib)
    return Encoded(buf.tobytes(), clipped.value)


def encode_pcm16_samples(pcm: np.ndarray, sample_rate: int) -> bytes:
    """A PCM_16 WAV from samples already converted (kk_fetch_audio_pcm16's device conversion)."""
    pcm = np.ascontiguousarray(pcm, np.int16)
    return header(Format.Pcm16, sample_rate, pcm.size * 2) + pcm.astype("<i2").tobytes()


def sha256_hex(data: bytes) -> str:
    lib = _lib()
    out = ctypes.create_string_buffer(65)
    buf = np.frombuffer(data, np.uint8) if len(data) else np.zeros(1, np.uint8)
    if lib.kk_sha256_hex(buf.ctypes.data, len(data), out) != 0:
        raise _err(lib)
    return out.value.decode()


def write_atomic(path: str, data: bytes, sync: bool = True) -> None:
    tmp = os.path.splitext(path)[0] + ".partial"
    with open(tmp, "wb") as f:
        f.write(data)
        if sync:
            f.flush()
            os.fsync(f.fileno())
    os.replace(tmp, path)


def read_canonical(path: str, fmt: Format, sample_rate: int) -> int:
    lib = _lib()
    d = ctypes.c_uint64()
    if lib.kk_wav_read_canonical(path.encode(), int(fmt), sample_rate, ctypes.byref(d)) != 0:
        raise _err(lib)
    return d.value


def assemble(parts: Sequence[Tuple[str, str]], fmt: Format, sample_rate: int, dest: str, sync: bool = True) -> Assembled:
    lib = _lib()
    n = len(parts)
    paths = (ctypes.c_char_p * max(n, 1))(*[p.encode() for p, _ in parts])
    shas = (ctypes.c_char_p * max(n, 1))(*[h.encode() for _, h in parts])
    out = ctypes.create_string_buffer(65)
    db, ns = ctypes.c_uint64(), ctypes.c_uint64()
    if lib.kk_wav_assemble(n, paths, shas, int(fmt), sample_rate, dest.encode(), 1 if sync else 0, out,
                           ctypes.byref(db), ctypes.byref(ns)) != 0:
        raise _err(lib)
    return Assembled(out.value.decode(), db.value, ns.value)


def write_lines(audios: List[np.ndarray], directory: str, sample_rate: int = 24000,
                fmt: Format = Format.Pcm16) -> List[Tuple[str, str]]:
    """Each line's audio as its own WAV part (atomic write), returning (path, sha256) for
    ``assemble`` in line order."""
    parts = []
    for i, a in enumerate(audios):
        e = encode(a, sample_rate, fmt)
        p = os.path.join(directory, f"line{i:06d}.wav")
        write_atomic(p, e.bytes, sync=False)
        parts.append((p, sha256_hex(e.bytes)))
    return parts
