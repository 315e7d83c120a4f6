"""Host-side mirror of the reference crate's engine API over the C ABI (include/kokoro_b200.h).

Names, argument meaning and error behaviour follow the reference:

* ``BatchItem`` / ``ItemNoise``: ``src/gpu_batch.rs:14-24``
* ``GpuKokoro.forward_batch``: ``src/gpu_batch.rs:179`` (here ``Engine.forward_batch``)
* ``BatchPolicy`` / ``plan_batches``: ``src/engine.rs:148-183``
* ``Engine.synth_batch`` (validation, length-bucketed batches, split-in-half on failure, results
  in input order): ``src/engine.rs:185-241``
* ``mix_seed``: ``src/engine.rs:141-146``; ``Voice.ref_s``: ``src/engine.rs:46-60``

The library is loaded with ctypes; there is no CPU fallback: if the shared library is missing or
cannot be loaded, ``load_library`` raises.
"""
from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkokoro_b200.so")

KK_OK, KK_ERR_INVALID_ARG, KK_ERR_OOM, KK_ERR_CUDA, KK_ERR_TIMEOUT, KK_ERR_IO = range(6)
KK_PRECISION_FP32, KK_PRECISION_BF16 = 0, 1
KK_OPT_KEEP_AUDIO_ON_DEVICE, KK_OPT_SYNC_EACH_STAGE, KK_OPT_PROFILE, KK_OPT_OUTPUT_PCM16 = 1, 2, 3, 4
KK_OPT_GAP_CANARY, KK_OPT_NEGCTL_NOMASK, KK_OPT_ATTENTION_F32 = 5, 6, 7
STATUS_NAMES = {0: "OK", 1: "INVALID_ARG", 2: "OOM", 3: "CUDA", 4: "TIMEOUT", 5: "IO"}

MAX_PHONEMES = 510  # src/engine.rs:12
STYLE_DIM = 128
SAMPLES_PER_FRAME = 600
SAMPLE_RATE = 24000

# Every symbol include/kokoro_b200.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_SIGS = {
    "kk_create": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_P)]),
    "kk_destroy": (None, [_P]),
    "kk_last_error": (ctypes.c_char_p, [_P]),
    "kk_identity": (ctypes.c_char_p, [_P]),
    "kk_forward_batch": (ctypes.c_int, [_P, ctypes.c_int, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "kk_forward_batch_noise": (ctypes.c_int, [_P, ctypes.c_int, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "kk_wait_selftest": (ctypes.c_int, [_P, ctypes.c_int64]),
    "kk_fetch_audio": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_int64]),
    "kk_fetch_audio_all": (ctypes.c_int, [_P, _P, _P]),
    "kk_decode_batch": (ctypes.c_int, [_P, ctypes.c_int, _P, _P, _P, _P, _P, _P, _P, _P]),
    "kk_decode_batch_noalloc": (ctypes.c_int, [_P, ctypes.c_int, _P, _P, _P, _P, _P, _P, _P, _P]),
    "kk_set_option": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int64]),
    "kk_device_bytes": (ctypes.c_int64, [_P]),
    "kk_launch_count": (ctypes.c_int64, [_P]),
    "kk_last_times": (ctypes.c_int, [_P, _P]),
    "kk_profile_entry": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_char_p, ctypes.c_int, _P, _P, _P]),
    "kk_profile_launch": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_char_p, ctypes.c_int, _P, _P, _P]),
    "kk_profile_reset": (None, [_P]),
    "kk_conv_selftest": (ctypes.c_int, [ctypes.c_int, _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_int, _P]),
    "kk_conv_selftest_error": (ctypes.c_char_p, []),
    "kk_attention_selftest": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, _P, _P, _P]),
    "kk_attention_selftest_bf16": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, _P, _P, _P]),
    "kk_lstm_selftest": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P, _P, _P]),
    "kk_fetch_audio_pcm16": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_int64, _P]),
    "kk_wav_header": (ctypes.c_int, [ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, _P]),
    "kk_wav_encode": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_uint32, ctypes.c_int, _P, ctypes.c_int64, _P, _P]),
    "kk_wav_read_canonical": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.c_uint32, _P]),
    "kk_wav_assemble": (ctypes.c_int, [ctypes.c_int, _P, _P, ctypes.c_int, ctypes.c_uint32, ctypes.c_char_p,
                                       ctypes.c_int, ctypes.c_char_p, _P, _P]),
    "kk_sha256_hex": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_char_p]),
    "kk_wav_error": (ctypes.c_char_p, []),
    "kk_memory_stats": (ctypes.c_int, [_P, _P]),
    "kk_pth_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(_P)]),
    "kk_pth_count": (ctypes.c_int, [_P]),
    "kk_pth_name": (ctypes.c_char_p, [_P, ctypes.c_int]),
    "kk_pth_shape": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_int]),
    "kk_pth_data": (ctypes.c_void_p, [_P, ctypes.c_int]),
    "kk_pth_close": (None, [_P]),
    "kk_pth_error": (ctypes.c_char_p, []),
    "kk_device_memory": (ctypes.c_int, [ctypes.c_int, _P, _P]),
}


class ConvCase(ctypes.Structure):
    """kk_conv_case of include/kokoro_b200.h."""
    _fields_ = [("cin", ctypes.c_int), ("cout", ctypes.c_int), ("K", ctypes.c_int), ("dil", ctypes.c_int),
                ("pad", ctypes.c_int), ("rows_in", ctypes.c_int), ("ldx", ctypes.c_int), ("up2", ctypes.c_int),
                ("in_mode", ctypes.c_int), ("slope", ctypes.c_float), ("rows_out", ctypes.c_int),
                ("ldy", ctypes.c_int), ("out_mode", ctypes.c_int), ("oscale", ctypes.c_float),
                ("ldsc", ctypes.c_int), ("n_items", ctypes.c_int), ("item_in", _P), ("item_out", _P),
                ("pre", ctypes.c_int)]


def conv_selftest(ordinal: int, *, x, w, item_in, item_out, rows_out, pad, dil=1, up2=0, in_mode=0,
                  slope=0.2, out_mode=0, oscale=1.0, bias=None, coef=None, alpha=None, sc=None, y=None,
                  n_items=None, want_stats=False, timing_iters=0, pre=0):
    """One convolution through the tcgen05 kernel (kk_conv_selftest). x [rows][ldx] f32, w torch
    layout [cout][cin][K]; returns y [rows_out][ldy] (and [n_items][cout][2] statistics); with
    timing_iters > 0 returns (result, device ms per launch)."""
    lib = load_library()
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    cout, cin, K = w.shape
    item_in = np.ascontiguousarray(item_in, np.int32)
    item_out = np.ascontiguousarray(item_out, np.int32)
    n_items = int(n_items if n_items is not None else max(item_in.max(), item_out.max()) + 1)
    y = np.ascontiguousarray(np.zeros((rows_out, cout), np.float32) if y is None else y, np.float32)
    c = ConvCase(cin, cout, K, dil, pad, len(item_in), x.shape[1], up2, in_mode, slope, rows_out, y.shape[1],
                 out_mode, oscale, 0 if sc is None else sc.shape[1], n_items,
                 item_in.ctypes.data, item_out.ctypes.data, pre)
    keep = []

    def ptr(a):
        if a is None:
            return None
        a = np.ascontiguousarray(a, np.float32)
        keep.append(a)
        return a.ctypes.data
    stat = np.zeros((n_items, cout, 2), np.float64) if want_stats else None
    ms = ctypes.c_double(0.0)
    st = lib.kk_conv_selftest(ordinal, ctypes.byref(c), x.ctypes.data, w.ctypes.data, ptr(bias), ptr(coef),
                              ptr(alpha), ptr(sc), y.ctypes.data, None if stat is None else stat.ctypes.data,
                              timing_iters, ctypes.byref(ms))
    if st != KK_OK:
        raise KokoroError(st, lib.kk_conv_selftest_error().decode())
    res = (y, stat) if want_stats else y
    return (res, ms.value) if timing_iters > 0 else res


def attention_selftest(ordinal: int, tok_len, qkv, bf16_rows: bool = False):
    """The BF16 mode's tensor-core attention (kk_attention_selftest): qkv [sum T][2304] f32 of items
    of tok_len rows each; returns ctx [sum T][768]. bf16_rows: qkv is a uint16 array of bf16 bit
    patterns (kk_attention_selftest_bf16, the QKV projection's output form)."""
    lib = load_library()
    tl = np.ascontiguousarray(tok_len, np.int32)
    qkv = np.ascontiguousarray(qkv, np.uint16 if bf16_rows else np.float32)
    ctx = np.zeros((qkv.shape[0], 768), np.float32)
    fn = lib.kk_attention_selftest_bf16 if bf16_rows else lib.kk_attention_selftest
    st = fn(ordinal, len(tl), tl.ctypes.data, qkv.ctypes.data, ctx.ctypes.data)
    if st != KK_OK:
        raise KokoroError(st, lib.kk_conv_selftest_error().decode())
    return ctx


def lstm_selftest(ordinal: int, tc: int, lens, gx, whh, bhh):
    """One BiLSTM recurrence (kk_lstm_selftest): gx [sum len][2048], whh [2][1024][256],
    bhh [2][1024]; returns h [sum len][512]."""
    lib = load_library()
    ln = np.ascontiguousarray(lens, np.int32)
    gx = np.ascontiguousarray(gx, np.float32)
    whh = np.ascontiguousarray(whh, np.float32)
    bhh = np.ascontiguousarray(bhh, np.float32)
    out = np.zeros((gx.shape[0], 512), np.float32)
    st = lib.kk_lstm_selftest(ordinal, tc, len(ln), ln.ctypes.data, gx.ctypes.data, whh.ctypes.data, bhh.ctypes.data,
                              out.ctypes.data)
    if st != KK_OK:
        raise KokoroError(st, lib.kk_conv_selftest_error().decode())
    return out


_lib = None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the engine library (building it first when its sources are newer)."""
    global _lib
    if _lib is not None:
        return _lib
    if os.path.exists(os.path.join(HERE, "csrc")) and os.environ.get("KK_NO_BUILD") != "1":
        from . import build as _build  # noqa: WPS433

        _build.build()
    if not os.path.exists(path):
        raise RuntimeError(f"kokoro-b200 library not found at {path}: run build() first")
    lib = ctypes.CDLL(path)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class KokoroError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


@dataclass
class ItemNoise:
    """Per-item excitation noise (src/gpu_batch.rs:12-17): a counter stream keyed by ``seed``
    (ItemNoise::Counter, the product path) or, when ``sine`` is set, replayed draws
    [600 * N * 9] with their initial phases ``rand_ini`` [9] (ItemNoise::Fixed, parity tests). The
    draw count must match the durations the forward uses, predicted or forced; rand_ini cannot
    change the output (the reference adds it at a sample its phase downsample never reads)."""

    seed: int = 0
    sine: Optional[np.ndarray] = None
    rand_ini: Optional[np.ndarray] = None


@dataclass
class BatchItem:
    ids: np.ndarray
    ref_s: np.ndarray
    speed: float = 1.0
    noise: ItemNoise = field(default_factory=ItemNoise)


@dataclass
class Output:
    audio: np.ndarray           # f32 samples, or int16 PCM_16 samples with pcm16=True
    pred_dur: np.ndarray
    clipped: int = 0            # PCM_16 samples clipped on the device (pcm16=True)


class GpuKokoro:
    """One engine bound to one CUDA device (``Gpu::new`` + ``GpuKokoro::with_gpu``)."""

    def __init__(self, weights_path: str, cuda_ordinal: int = 0, precision: str = "fp32"):
        self.lib = load_library()
        prec = {"fp32": KK_PRECISION_FP32, "bf16": KK_PRECISION_BF16}[precision]
        h = ctypes.c_void_p()
        st = self.lib.kk_create(weights_path.encode(), cuda_ordinal, prec, ctypes.byref(h))
        if st != KK_OK:
            raise KokoroError(st, self.lib.kk_last_error(None).decode())
        self.h = h
        self.precision = precision
        self.ordinal = cuda_ordinal

    def close(self):
        if getattr(self, "h", None):
            self.lib.kk_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def _check(self, st: int):
        if st != KK_OK:
            raise KokoroError(st, self.lib.kk_last_error(self.h).decode())

    @property
    def identity(self) -> str:
        return self.lib.kk_identity(self.h).decode()

    def set_option(self, option: int, value: int):
        self._check(self.lib.kk_set_option(self.h, option, value))

    def launch_count(self) -> int:
        return int(self.lib.kk_launch_count(self.h))

    def device_bytes(self) -> int:
        return int(self.lib.kk_device_bytes(self.h))

    def memory_stats(self) -> dict:
        """Device memory of the engine and of its last call (kk_memory_stats)."""
        out = (ctypes.c_int64 * 5)()
        self._check(self.lib.kk_memory_stats(self.h, out))
        return {"weight_bytes": out[0], "arena_bytes": out[1], "peak_bytes": out[2], "tokens": out[3],
                "frames": out[4]}

    def device_memory(self) -> tuple:
        """(free, total) bytes of this engine's device."""
        return device_memory(self.ordinal)

    def last_times(self) -> dict:
        """Device-side timings of the last call (CUDA events on the engine stream)."""
        out = (ctypes.c_double * 4)()
        self._check(self.lib.kk_last_times(self.h, out))
        return {"total_ms": out[0], "compute_ms": out[1], "h2d_bytes": int(out[2]), "d2h_bytes": int(out[3])}

    def profile(self) -> dict:
        """{kernel class: (launches, device ms, algorithmic FLOPs)} accumulated under KK_OPT_PROFILE."""
        n = self.lib.kk_profile_entry(self.h, -1, None, 0, None, None, None)
        res = {}
        for i in range(max(n, 0)):
            name = ctypes.create_string_buffer(64)
            la, ms, fl = ctypes.c_int64(), ctypes.c_double(), ctypes.c_double()
            self.lib.kk_profile_entry(self.h, i, name, 64, ctypes.byref(la), ctypes.byref(ms), ctypes.byref(fl))
            res[name.value.decode()] = (int(la.value), float(ms.value), float(fl.value))
        return res

    def profile_launches(self) -> List[tuple]:
        """[(class, device ms, algorithmic FLOPs, algorithmic bytes)] per launch profiled since the
        last reset."""
        n = self.lib.kk_profile_launch(self.h, -1, None, 0, None, None, None)
        res = []
        name = ctypes.create_string_buffer(64)
        ms, fl, by = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
        for i in range(max(n, 0)):
            self.lib.kk_profile_launch(self.h, i, name, 64, ctypes.byref(ms), ctypes.byref(fl), ctypes.byref(by))
            res.append((name.value.decode(), float(ms.value), float(fl.value), float(by.value)))
        return res

    def profile_reset(self):
        self.lib.kk_profile_reset(self.h)

    def wait_selftest(self, limit_ns: int = 5000):
        """Drive the bounded in-kernel wait to expiry on a barrier nothing arrives on
        (kk_wait_selftest); raises KokoroError with status KK_ERR_TIMEOUT, as a forward whose wait
        expired would."""
        self._check(self.lib.kk_wait_selftest(self.h, int(limit_ns)))

    def forward_batch(self, items: Sequence[BatchItem], forced_dur: Optional[Sequence[np.ndarray]] = None,
                      fetch: bool = True, pcm16: bool = False) -> List[Output]:
        """Batched ragged forward; results in input order (src/gpu_batch.rs:179-421). pcm16=True
        converts the audio to PCM_16 on the device (the WAV rule of src/wav.rs:76-84) and returns
        int16 samples with per-item clip counts."""
        self._check(self.lib.kk_set_option(self.h, KK_OPT_OUTPUT_PCM16, 1 if pcm16 else 0))
        n = len(items)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(it.ids, np.int64) for it in items]) if n else
                                   np.zeros(0, np.int64))
        lens = np.ascontiguousarray([len(it.ids) for it in items], dtype=np.int32)
        ref_s = np.ascontiguousarray(np.stack([np.asarray(it.ref_s, np.float32) for it in items]) if n else
                                     np.zeros((0, 256), np.float32))
        speed = np.ascontiguousarray([it.speed for it in items], dtype=np.float32)
        seeds = np.ascontiguousarray([it.noise.seed & ((1 << 64) - 1) for it in items], dtype=np.uint64)
        fd = None
        if forced_dur is not None:
            fd = np.ascontiguousarray(np.concatenate([np.asarray(d, np.int64) for d in forced_dur]))
        dur = np.zeros(ids.shape[0], np.int64)
        ns = np.zeros(n, np.int64)
        if any(it.noise.sine is not None for it in items):
            # per-item ItemNoise (kk_forward_batch_noise): replayed draws where given, counter elsewhere
            sines = [None if it.noise.sine is None else np.ascontiguousarray(it.noise.sine, np.float32)
                     for it in items]
            ptrs = (ctypes.c_void_p * n)(*[None if a is None else a.ctypes.data for a in sines])
            nlen = np.ascontiguousarray([0 if a is None else a.size for a in sines], dtype=np.int64)
            ri = np.ascontiguousarray(np.stack([np.zeros(9, np.float32) if it.noise.rand_ini is None else
                                                np.asarray(it.noise.rand_ini, np.float32).reshape(9)
                                                for it in items]))
            self._check(self.lib.kk_forward_batch_noise(self.h, n, _ptr(ids), _ptr(lens), _ptr(ref_s), _ptr(speed),
                                                        _ptr(seeds), ctypes.cast(ptrs, ctypes.c_void_p), _ptr(nlen),
                                                        _ptr(ri), _ptr(fd), _ptr(dur), _ptr(ns)))
        else:
            self._check(self.lib.kk_forward_batch(self.h, n, _ptr(ids), _ptr(lens), _ptr(ref_s), _ptr(speed),
                                                  _ptr(seeds), None, _ptr(fd), _ptr(dur), _ptr(ns)))
        outs = []
        o = 0
        for i in range(n):
            clipped = ctypes.c_int64(0)
            if pcm16:
                a = np.empty(int(ns[i]), np.int16)
                if fetch:
                    self._check(self.lib.kk_fetch_audio_pcm16(self.h, i, _ptr(a), a.shape[0], ctypes.byref(clipped)))
            else:
                a = np.empty(int(ns[i]), np.float32)
            outs.append(Output(a, dur[o:o + lens[i]].copy(), int(clipped.value)))
            o += lens[i]
        if fetch and not pcm16 and n:
            # every item's audio in one call (the library copies items on several threads)
            dst = (ctypes.c_void_p * n)(*[o_.audio.ctypes.data for o_ in outs])
            cap = np.ascontiguousarray(ns, dtype=np.int64)
            self._check(self.lib.kk_fetch_audio_all(self.h, ctypes.cast(dst, ctypes.c_void_p), _ptr(cap)))
        return outs

    def decode_batch(self, asr: Sequence[np.ndarray], f0: Sequence[np.ndarray], n_curve: Sequence[np.ndarray],
                     s_dec: np.ndarray, seeds: Optional[Sequence[int]] = None,
                     noise: Optional[Sequence[np.ndarray]] = None, fetch: bool = True) -> List[np.ndarray]:
        """Decoder + generator only: asr [N_b, 512] time-major, f0 / n [2 N_b], s_dec [B, 128]."""
        B = len(asr)
        nf = np.ascontiguousarray([a.shape[0] for a in asr], dtype=np.int32)
        asr_c = np.ascontiguousarray(np.concatenate([np.asarray(a, np.float32) for a in asr]))
        f0_c = np.ascontiguousarray(np.concatenate([np.asarray(a, np.float32) for a in f0]))
        n_c = np.ascontiguousarray(np.concatenate([np.asarray(a, np.float32) for a in n_curve]))
        sd = np.ascontiguousarray(np.asarray(s_dec, np.float32).reshape(B, 128))
        sds = None if seeds is None else np.ascontiguousarray(np.asarray(seeds, np.uint64))
        nz = None if noise is None else np.ascontiguousarray(np.concatenate([np.asarray(x, np.float32) for x in noise]))
        out = np.empty(int(nf.sum()) * SAMPLES_PER_FRAME, np.float32) if fetch else None
        self._check(self.lib.kk_decode_batch(self.h, B, _ptr(nf), _ptr(asr_c), _ptr(f0_c), _ptr(n_c), _ptr(sd),
                                             _ptr(sds), _ptr(nz), _ptr(out)))
        if not fetch:
            return []
        res, o = [], 0
        for k in nf:
            res.append(out[o:o + k * SAMPLES_PER_FRAME])
            o += k * SAMPLES_PER_FRAME
        return res


    def decode_batch_noalloc(self, asr: Sequence[np.ndarray], f0: Sequence[np.ndarray],
                             n_curve: Sequence[np.ndarray], s_dec: np.ndarray,
                             seeds: Optional[Sequence[int]] = None,
                             noise: Optional[Sequence[np.ndarray]] = None) -> List[np.ndarray]:
        """decode_batch without any device / pinned-host allocation, for callers that cannot
        allocate (a streaming audio thread must not wait on cudaMalloc; a GPU shared under a fixed
        memory budget must not let the engine's arena grow). Scratch is a 64 MiB static device
        array shared by every call on the device; at most 8 items and 120 N-frames per call
        (2 gap frames per item included). Calls that overlap on one device race on the array."""
        B = len(asr)
        nf = np.ascontiguousarray([a.shape[0] for a in asr], dtype=np.int32)
        asr_c = np.ascontiguousarray(np.concatenate([np.asarray(a, np.float32) for a in asr]))
        f0_c = np.ascontiguousarray(np.concatenate([np.asarray(a, np.float32) for a in f0]))
        n_c = np.ascontiguousarray(np.concatenate([np.asarray(a, np.float32) for a in n_curve]))
        sd = np.ascontiguousarray(np.asarray(s_dec, np.float32).reshape(B, 128))
        sds = None if seeds is None else np.ascontiguousarray(np.asarray(seeds, np.uint64))
        nz = None if noise is None else np.ascontiguousarray(np.concatenate([np.asarray(x, np.float32) for x in noise]))
        out = np.empty(int(nf.sum()) * SAMPLES_PER_FRAME, np.float32)
        self._check(self.lib.kk_decode_batch_noalloc(self.h, B, _ptr(nf), _ptr(asr_c), _ptr(f0_c), _ptr(n_c),
                                                     _ptr(sd), _ptr(sds), _ptr(nz), _ptr(out)))
        res, o = [], 0
        for k in nf:
            res.append(out[o:o + k * SAMPLES_PER_FRAME])
            o += k * SAMPLES_PER_FRAME
        return res


# ------------------------------------------------------------------------------ scheduling layer

def mix_seed(seed: int, index: int) -> int:
    """splitmix64 per-item seed derivation (src/engine.rs:141-146)."""
    m = (1 << 64) - 1
    z = (seed ^ ((index * 0x9E3779B97F4A7C15) & m)) & m
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    return z ^ (z >> 31)


def device_memory(cuda_ordinal: int) -> tuple:
    """(free, total) bytes of a CUDA device (kk_device_memory)."""
    lib = load_library()
    f, t = ctypes.c_int64(), ctypes.c_int64()
    st = lib.kk_device_memory(cuda_ordinal, ctypes.byref(f), ctypes.byref(t))
    if st != KK_OK:
        raise KokoroError(st, "cudaMemGetInfo failed")
    return int(f.value), int(t.value)


# Working set of one forward per output frame (peak arena bytes / frames) and predicted frames per
# phoneme token at speed 1, measured on a B200 over config 4's 251-line batch (BF16 mode); used
# until the engine has run a forward of its own.
# (measured: 30.8 GB peak for 69,319 frames = 444 KB per frame; 2.03 frames per token)
DEFAULT_BYTES_PER_FRAME = 450_000
DEFAULT_FRAMES_PER_PHONEME = 2.5


@dataclass
class BatchPolicy:
    """Batching budget (src/engine.rs:148-161): total phoneme characters and items per batch."""

    max_phonemes: int = 4000
    max_items: int = 64

    @classmethod
    def from_free_vram(cls, gpu: "GpuKokoro", speed: float = 1.0, max_items: int = 1024, headroom: float = 0.85,
                       bytes_per_frame: Optional[float] = None,
                       frames_per_phoneme: Optional[float] = None) -> "BatchPolicy":
        """A phoneme budget derived from the device's free memory, the scheduler rule of
        docs/design/BATCHING.md:44-47 (the reference's code keeps a fixed budget).

        Memory available to a batch = (free device memory + the engine's arena, which the next call
        reuses) x ``headroom``. Frames that fit = that / bytes per frame (the engine's own last
        forward when it has run one, else ``DEFAULT_BYTES_PER_FRAME``); phonemes = frames /
        (frames per phoneme / speed), frames per phoneme again from the last forward (never below
        the default, so a short calibration batch cannot inflate the budget). A batch that still
        does not fit fails with KK_ERR_OOM and ``synth_batch`` splits it in half."""
        st = gpu.memory_stats()
        free, _total = gpu.device_memory()
        avail = (free + st["arena_bytes"]) * headroom
        bpf = bytes_per_frame
        if bpf is None:
            bpf = st["peak_bytes"] / st["frames"] if st["frames"] > 0 and st["tokens"] > 0 else DEFAULT_BYTES_PER_FRAME
            bpf = max(bpf, DEFAULT_BYTES_PER_FRAME * 0.5)
        fpp = frames_per_phoneme
        if fpp is None:
            fpp = DEFAULT_FRAMES_PER_PHONEME
            if st["tokens"] > 0:
                fpp = max(fpp, st["frames"] / st["tokens"] * speed)
        frames = avail / bpf
        return cls(max_phonemes=max(MAX_PHONEMES + 2, int(frames / (fpp / speed))), max_items=max_items)


def plan_batches(lens: Sequence[int], p: BatchPolicy) -> List[List[int]]:
    """Sort by length (stable on index), greedily fill each batch up to the policy budget
    (src/engine.rs:165-183)."""
    order = sorted(range(len(lens)), key=lambda i: (lens[i], i))
    out, cur, s = [], [], 0
    for i in order:
        if cur and (len(cur) >= p.max_items or s + lens[i] > p.max_phonemes):
            out.append(cur)
            cur, s = [], 0
        s += lens[i]
        cur.append(i)
    if cur:
        out.append(cur)
    return out


@dataclass
class Voice:
    """Voice pack [rows, 256]; ref_s = pack[n_phoneme_chars - 1] (src/engine.rs:46-60)."""

    pack: np.ndarray
    sha256: str = ""  # of the .pt file(s) it came from, comma-joined (provenance)

    def ref_s(self, n_chars: int) -> np.ndarray:
        if n_chars < 1:
            raise ValueError("empty phoneme string")
        if n_chars - 1 >= self.pack.shape[0]:
            raise ValueError(f"phoneme length {n_chars} exceeds voice pack rows {self.pack.shape[0]}")
        return self.pack[n_chars - 1]


@dataclass
class Synth:
    audio: np.ndarray
    pred_dur: np.ndarray
    dropped: list


class Engine:
    """Resident synthesis engine (src/engine.rs:62-241).

    The text frontend is out of scope: a request is a phoneme string (mapped to token ids with the
    model's vocabulary, config.json, as the reference's ``phonemes_to_ids``) or a sequence of
    phoneme token ids (without the boundary pads, which ``synth_batch`` adds)."""

    def __init__(self, weights_path: str, cuda_ordinal: int = 0, precision: str = "fp32",
                 model_dir: Optional[str] = None):
        """weights_path: a safetensors file or the PyTorch checkpoint (.pth) itself; model_dir
        holds config.json and voices/<name>.pt (src/engine.rs:80-112)."""
        from . import wav
        self.gpu = GpuKokoro(weights_path, cuda_ordinal, precision)
        self.model_dir = model_dir if model_dir is not None else os.path.dirname(os.path.abspath(weights_path))
        self.voices = {}
        with open(weights_path, "rb") as f:
            self.model_sha256 = wav.sha256_hex(f.read())
        self.vocab, self.config_sha256 = {}, ""
        cfg = os.path.join(self.model_dir, "config.json")
        if os.path.exists(cfg):
            with open(cfg, "rb") as f:
                raw = f.read()
            self.config_sha256 = wav.sha256_hex(raw)
            self.vocab = {k: int(v) for k, v in json.loads(raw.decode("utf-8")).get("vocab", {}).items()}

    def phonemes_to_ids(self, ps: str) -> tuple:
        """[0] + vocab ids of the characters + [0]; characters outside the vocabulary are dropped
        and returned (src/model.rs:146-157)."""
        ids, dropped = [0], []
        for c in ps:
            if c in self.vocab:
                ids.append(self.vocab[c])
            else:
                dropped.append(c)
        ids.append(0)
        return np.asarray(ids, np.int64), dropped

    def identity(self) -> str:
        return self.gpu.identity

    def add_voice(self, name: str, pack: np.ndarray):
        self.voices[name] = Voice(np.asarray(pack, np.float32).reshape(-1, 256))

    def _load_voice_part(self, part: str) -> Voice:
        if part in self.voices:
            return self.voices[part]
        from . import pth, wav
        path = part if part.endswith(".pt") else os.path.join(self.model_dir, "voices", part + ".pt")
        pack = pth.load_voice_pack(path)
        with open(path, "rb") as f:
            digest = wav.sha256_hex(f.read())
        return Voice(pack.reshape(pack.shape[0], 256), digest)

    def voice(self, spec: str) -> Voice:
        """Voice by name (an added pack, or voices/<name>.pt under model_dir), explicit .pt path, or
        comma-separated element-wise mean of several (src/engine.rs:115-137)."""
        if spec not in self.voices:
            vs = [self._load_voice_part(p) for p in spec.split(",")]
            if any(v.pack.shape != vs[0].pack.shape for v in vs):
                raise ValueError("voice packs have different shapes")
            pack = vs[0].pack if len(vs) == 1 else np.mean(np.stack([v.pack for v in vs]), axis=0).astype(np.float32)
            self.voices[spec] = Voice(pack, ",".join(v.sha256 for v in vs))
        return self.voices[spec]

    def synth_batch(self, reqs: Sequence[tuple], voice: str, speed: float = 1.0,
                    policy: BatchPolicy = BatchPolicy()) -> list:
        """reqs: [(phoneme string or token ids without pads, seed)]. Returns per request a Synth
        or an Exception, in input order; a failing batch is split in half down to single items.
        The length rules count phoneme characters (dropped ones included), as the reference does."""
        results: list = [None] * len(reqs)
        prepared = []
        for i, (toks, _seed) in enumerate(reqs):
            n = len(toks)
            try:
                if n == 0:
                    raise ValueError("empty phoneme string")
                if n > MAX_PHONEMES:
                    raise ValueError(f"oversize: {n} phoneme chars > {MAX_PHONEMES}")
                if isinstance(toks, str):
                    ids, dropped = self.phonemes_to_ids(toks)
                else:
                    ids, dropped = np.concatenate([[0], np.asarray(toks, np.int64), [0]]), []
                prepared.append((i, ids, self.voice(voice).ref_s(n), dropped))
            except Exception as e:  # per-chunk validation error (src/engine.rs:194-211)
                results[i] = e
        lens = [len(p[1]) for p in prepared]
        stack = list(reversed(plan_batches(lens, policy)))
        while stack:
            batch = stack.pop()
            items = [BatchItem(prepared[k][1], prepared[k][2], speed, ItemNoise(seed=reqs[prepared[k][0]][1]))
                     for k in batch]
            try:
                outs = self.gpu.forward_batch(items)
                for k, o in zip(batch, outs):
                    results[prepared[k][0]] = Synth(o.audio, o.pred_dur, prepared[k][3])
            except KokoroError as e:
                if len(batch) > 1:
                    mid = len(batch) // 2
                    stack.append(batch[mid:])
                    stack.append(batch[:mid])
                else:
                    results[prepared[batch[0]][0]] = e
        return [r if r is not None else RuntimeError("internal: missing batch result") for r in results]
