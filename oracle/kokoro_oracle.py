"""CPU oracle for the batched Kokoro-82M forward -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA engine and the timed CPU baseline. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it; the product path
(the C-ABI library) never does.

It restates, per utterance and in fp32 (f64 where the reference accumulates in f64), the forward
that ``GpuKokoro::forward_batch`` (``src/gpu_batch.rs:179-421``) computes for each item of a
batch.  Batching does not change per-item results in the reference (``docs/design/BATCHING.md``),
so the oracle runs one item at a time.  Order of authority followed:

* stage order and glue: ``src/gpu_batch.rs:179-481``;
* per-element arithmetic: ``kernels/kokoro.cu`` -- SineGen ``:188-254``, STFT ``:470-490``,
  iSTFT ``:264-280,492-508``, noise ``:282-302``, AdaIN stats ``:776-810`` and apply
  ``:317-334``, Snake ``:700-714``, LSTM gates ``:400-450``, LayerNorm ``:44-82``,
  gelu_new ``:84-90``, softmax ``:93-122``;
* shapes, constants and names: ``src/model.rs``, ``src/nn.rs``, ``src/vocoder.rs``,
  ``src/albert.rs``.

The upstream Python model (kokoro 0.9.4) is not vendored in the reference, so parity of this
oracle is pinned by the reference's structural known answers (state-dict census, frame/sample
arithmetic, the splitmix64 constants) and by golden vectors produced from the reference's own
CUDA kernels compiled from source (``tests/golden``); see the tests for which.
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

_HERE = os.path.dirname(os.path.abspath(__file__))

STYLE_DIM, HIDDEN, MAX_DUR = 128, 512, 50
HEADS, HEAD_DIM, ALBERT_LAYERS = 12, 64, 12
N_FFT, HOP, HARMONICS, UPSAMPLE = 20, 5, 9, 300
SAMPLES_PER_FRAME = 600
PI_F = np.float32(3.14159274101257324)  # kernels/kokoro.cu:9
F32 = np.float32


# ----------------------------------------------------------------------------- numeric helpers

def fma32(a, b, c):
    """f32 fused multiply-add: the f32 product is exact in f64; one rounding of the f64 sum to
    f32 (double rounding is possible only at exact f32 ties, not observed in practice)."""
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(F32)


def weight_norm(v: np.ndarray, g: np.ndarray) -> np.ndarray:
    """torch._weight_norm(v, g, dim=0) as src/ops.rs:9-23: f64 row norm cast to f32,
    scale = g / norm (f32), w = v * scale (f32)."""
    rows = g.reshape(-1).shape[0]
    vr = v.reshape(rows, -1).astype(F32)
    norm = np.sqrt((vr.astype(np.float64) ** 2).sum(axis=1)).astype(F32)
    scale = (g.reshape(-1).astype(F32) / norm).astype(F32)
    return (vr * scale[:, None]).astype(F32).reshape(v.shape)


def ln_rows(x: np.ndarray, g=None, b=None, eps=1e-5) -> np.ndarray:
    """Row LayerNorm with f64 reductions (src/ops.rs:26-50, kernels/kokoro.cu:44-82)."""
    x = np.asarray(x, F32)
    d = x.shape[-1]
    mean = (x.astype(np.float64).sum(-1, keepdims=True) / d).astype(F32)
    c = (x - mean).astype(np.float64)
    var = ((c * c).sum(-1, keepdims=True) / d).astype(F32)
    inv = (F32(1.0) / np.sqrt(var + F32(eps))).astype(F32)
    o = ((x - mean) * inv).astype(F32)
    if g is not None:
        o = (o * g).astype(F32)
    if b is not None:
        o = (o + b).astype(F32)
    return o


def gelu_new(x: torch.Tensor) -> torch.Tensor:
    """kernels/kokoro.cu:84-90 (tanh approximation, c = (float)sqrt(2/pi))."""
    c = 0.797884560802865355
    return 0.5 * x * (1.0 + torch.tanh(c * (x + 0.044715 * x * x * x)))


def sigmoid32(x: np.ndarray) -> np.ndarray:
    """1 / (1 + exp(-x)) in f32 (src/ops.rs:48-50)."""
    x = np.asarray(x, F32)
    return (F32(1.0) / (F32(1.0) + np.exp(-x))).astype(F32)


def durations_from_logits(logits: np.ndarray, speed: float):
    """src/model.rs:90-99: round-half-even(sum_j sigmoid(l_ij) / speed), clamped to >= 1.
    The f32 sum is sequential in j (Rust iterator sum).  Returns (durations, pre-round values)."""
    s = np.cumsum(sigmoid32(logits), axis=1, dtype=F32)[:, -1]
    q = (s / F32(speed)).astype(F32)
    d = np.maximum(np.rint(q).astype(np.int64), 1)
    return d, q


# ----------------------------------------------------------------------------- noise

M64 = (1 << 64) - 1


def splitmix_at(seed: int, ctr: np.ndarray) -> np.ndarray:
    """splitmix64 output number ``ctr`` of the stream at ``seed`` (src/vocoder.rs:22-27)."""
    with np.errstate(over="ignore"):
        c = np.asarray(ctr, dtype=np.uint64)
        x = np.uint64(seed & M64) + (c + np.uint64(1)) * np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return x ^ (x >> np.uint64(31))


def counter_noise(seed: int, n: int) -> np.ndarray:
    """Counter-based Gaussian stream (kernels/kokoro.cu:282-302): pair i uses
    splitmix_at(seed, 1024 + i), Box-Muller with log / sqrt / cos / sin correctly rounded to f32
    (evaluated in f64), exactly as the engine generates it in place."""
    npair = (n + 1) // 2
    x = splitmix_at(seed, np.arange(npair, dtype=np.uint64) + np.uint64(1024))
    u1 = ((x >> np.uint64(40)) + np.uint64(1)).astype(F32) * F32(1.0 / 16777216.0)
    u2 = ((x >> np.uint64(16)) & np.uint64(0xFFFFFF)).astype(F32) * F32(1.0 / 16777216.0)
    r = np.sqrt(-2.0 * np.log(u1.astype(np.float64))).astype(F32)
    th = (F32(6.2831855) * u2).astype(F32)
    out = np.empty(2 * npair, F32)
    out[0::2] = r * np.cos(th.astype(np.float64)).astype(F32)
    out[1::2] = r * np.sin(th.astype(np.float64)).astype(F32)
    return out[:n]


def mix_seed(seed: int, index: int) -> int:
    """Per-item seed derivation (src/engine.rs:141-146)."""
    z = (seed ^ ((index * 0x9E3779B97F4A7C15) & M64)) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


# ----------------------------------------------------------------------------- source / STFT

def _twiddles():
    k = np.arange(11)[:, None]
    n = np.arange(20)[None, :]
    a = 2.0 * np.pi * ((k * n) % 20) / 20.0
    return np.cos(a), np.sin(a)


TW_COS, TW_SIN = _twiddles()
HANN = (0.5 - 0.5 * np.cos(2.0 * np.pi * np.arange(20) / 20.0)).astype(F32)  # src/gpu.rs:101


def _rad(f0c: np.ndarray, t: np.ndarray) -> np.ndarray:
    """rad_h(t) = remainder(f0[nearest source of t] * (h + 1) / 24000, 1) (kernels/kokoro.cu:188-204)."""
    L = f0c.shape[0]
    near = F32(1.0 / UPSAMPLE)
    hs = np.arange(HARMONICS, dtype=F32)[:, None] + F32(1.0)
    src = np.minimum(np.floor(t.astype(F32) * near).astype(np.int64), L - 1)
    a = ((f0c[src][None, :] * hs) / F32(24000.0)).astype(F32)
    m = np.fmod(a, F32(1.0))
    return np.where((m != 0) & (m < 0), m + F32(1.0), m).astype(F32)


def sine_phase_pre(f0c: np.ndarray) -> np.ndarray:
    """phase_pre [9, D]: linear downsample (x 1/300) of rad, f64 cumulative sum, * 2 pi * 300
    (sine_phase_pre, kernels/kokoro.cu:206-226; FMA placement of the reference). rand_ini is
    added by the reference only at sample 0, which this downsample never reads (real >= 149.5),
    so it cannot change the result."""
    f0c = np.asarray(f0c, F32)
    L = f0c.shape[0]
    S = L * UPSAMPLE
    D = int(math.floor(S * (1.0 / UPSAMPLE)))
    down = F32(1.0 / (1.0 / UPSAMPLE))
    d = np.arange(D)
    real = fma32(down, d.astype(F32) + F32(0.5), F32(-0.5))
    real = np.maximum(real, F32(0.0))
    i0 = np.minimum(np.floor(real).astype(np.int64), S - 1)
    l1 = np.clip(real - i0.astype(F32), F32(0.0), F32(1.0)).astype(F32)
    i1 = np.where(i0 < S - 1, i0 + 1, i0)
    l0 = (F32(1.0) - l1).astype(F32)
    v = fma32(_rad(f0c, i0), l0[None, :], (_rad(f0c, i1) * l1[None, :]).astype(F32))
    acc = np.cumsum(v.astype(np.float64), axis=1)
    return ((acc.astype(F32) * F32(2.0)) * PI_F * F32(300.0)).astype(F32)


def har_from_phase(f0c: np.ndarray, pp: np.ndarray, noise: np.ndarray, lw: np.ndarray, lb: float) -> np.ndarray:
    """har[t] = tanh(sum_h lw_h (0.1 sin(phase(t, h)) uv + amp noise[t, h]) + lb), phase linearly
    upsampled (x 300) from phase_pre (sine_har_source, kernels/kokoro.cu:228-254)."""
    f0c = np.asarray(f0c, F32)
    L = f0c.shape[0]
    S = L * UPSAMPLE
    D = pp.shape[1]
    near = F32(1.0 / UPSAMPLE)
    up = F32(1.0 / UPSAMPLE)
    t = np.arange(S)
    src = np.minimum(np.floor(t.astype(F32) * near).astype(np.int64), L - 1)
    f0 = f0c[src]
    uv = (f0 > F32(10.0)).astype(F32)
    amp = (uv * F32(0.003) + ((F32(1.0) - uv) * F32(0.1)) / F32(3.0)).astype(F32)
    real = fma32(up, t.astype(F32) + F32(0.5), F32(-0.5))
    real = np.maximum(real, F32(0.0))
    i0 = np.minimum(np.floor(real).astype(np.int64), D - 1)
    l1 = np.clip(real - i0.astype(F32), F32(0.0), F32(1.0)).astype(F32)
    i1 = np.where(i0 < D - 1, i0 + 1, i0)
    l0 = (F32(1.0) - l1).astype(F32)
    nz = np.asarray(noise, F32).reshape(S, HARMONICS)
    acc = np.zeros(S, F32)
    for h in range(HARMONICS):
        ph = fma32(pp[h, i0], l0, (pp[h, i1] * l1).astype(F32))
        sine = (np.sin(ph.astype(np.float64)).astype(F32) * F32(0.1)).astype(F32)
        vv = ((sine * uv).astype(F32) + (amp * nz[:, h]).astype(F32)).astype(F32)
        acc = (acc + (F32(lw[h]) * vv).astype(F32)).astype(F32)
    return np.tanh((acc + F32(lb)).astype(np.float64)).astype(F32)


def sinegen_har(f0c: np.ndarray, noise: np.ndarray, lw: np.ndarray, lb: float) -> np.ndarray:
    """Harmonic source of one item (kernels/kokoro.cu:188-254, src/gpu_batch.rs:319-350).

    f0c: F0 curve [L] (2N domain); noise: [S * 9] f32 draws (index t*9 + h); returns har [S]."""
    f0c = np.asarray(f0c, F32)
    return har_from_phase(f0c, sine_phase_pre(f0c), noise, lw, lb)


def stft20(x: np.ndarray) -> np.ndarray:
    """Reflect-padded centred STFT, n_fft 20, hop 5, periodic Hann, f64 DFT -> [mag(11); phase(11)]
    (kernels/kokoro.cu:470-490); x [S] -> [22, 1 + S // 5]. Sequential f64 accumulation and
    magnitude / phase rounded once from f64, matching the engine bit for bit."""
    x = np.asarray(x, F32)
    S = x.shape[0]
    Fn = 1 + S // HOP
    p = np.arange(Fn)[:, None] * HOP + np.arange(20)[None, :] - 10
    src = np.where(p < 0, -p, np.where(p >= S, 2 * S - 2 - p, p))
    buf = (x[src] * HANN[None, :]).astype(F32).astype(np.float64)
    re = np.zeros((Fn, 11))
    im = np.zeros((Fn, 11))
    for n in range(20):  # sequential f64 accumulation, no fused multiply-add
        re = re + buf[:, n:n + 1] * TW_COS[None, :, n]
        im = im - buf[:, n:n + 1] * TW_SIN[None, :, n]
    im[:, 0] = 0.0
    im[:, 10] = 0.0
    rf, imf = re.astype(F32), im.astype(F32)
    mag = np.hypot(rf.astype(np.float64), imf.astype(np.float64)).astype(F32)
    ph = np.arctan2(imf.astype(np.float64), rf.astype(np.float64)).astype(F32)
    return np.concatenate([mag.T, ph.T], axis=0)  # [22, F]


def istft20(post: np.ndarray) -> np.ndarray:
    """exp/sin magnitude-phase, 20-point inverse real DFT (f64), Hann window, overlap-add divided
    by the window envelope, trim 10 (kernels/kokoro.cu:264-280, 492-508).  post [22, F] -> [5(F-1)]."""
    post = np.asarray(post, F32)
    Fn = post.shape[1]
    m = np.exp(post[:11]).astype(F32)
    p = np.sin(post[11:]).astype(F32)
    re = (m * np.cos(p)).astype(F32).astype(np.float64)  # [11, F]
    im = (m * np.sin(p)).astype(F32).astype(np.float64)
    sgn = np.where(np.arange(20) % 2 == 0, 1.0, -1.0)
    v = re[0][:, None] + re[10][:, None] * sgn[None, :]
    for k in range(1, 10):
        v = v + 2.0 * (re[k][:, None] * TW_COS[k][None, :] - im[k][:, None] * TW_SIN[k][None, :])
    fr = (v / 20.0) * HANN.astype(np.float64)[None, :]  # [F, 20]
    n_out = HOP * (Fn - 1)
    total = n_out + 20
    acc = np.zeros(total + HOP * 4)
    env = np.zeros_like(acc)
    w2 = HANN.astype(np.float64) ** 2
    for f in range(Fn):
        acc[HOP * f : HOP * f + 20] += fr[f]
        env[HOP * f : HOP * f + 20] += w2
    j = np.arange(n_out) + 10
    return (acc[j] / env[j]).astype(F32)


# ----------------------------------------------------------------------------- layer arithmetic

def chan_stats(x: np.ndarray, eps: float = 1e-5):
    """Per-channel mean / rstd over time of x [C, T]: biased variance, eps 1e-5, accumulated in
    f64 (chan_stats_seg, kernels/kokoro.cu:776-810)."""
    xn = np.asarray(x, F32).astype(np.float64)
    mean = xn.mean(axis=1)
    var = ((xn - mean[:, None]) ** 2).mean(axis=1)
    return mean.astype(F32), (F32(1.0) / np.sqrt(var.astype(F32) + F32(eps))).astype(F32)


def adain_apply(x, mean, rstd, nw, nb, gamma, beta, slope=None):
    """(1 + gamma) * ((x - mean) * rstd * nw + nb) + beta, then optional leaky ReLU
    (adain_apply_seg, kernels/kokoro.cu:317-334). x [C, T]; per-channel vectors."""
    x = np.asarray(x, F32)
    v = ((x - mean[:, None]) * rstd[:, None]).astype(F32)
    v = ((F32(1.0) + gamma[:, None]) * (v * nw[:, None] + nb[:, None]) + beta[:, None]).astype(F32)
    if slope is not None:
        v = np.where(v < 0, v * F32(slope), v).astype(F32)
    return v


def lstm_dir(gx: torch.Tensor, whh: torch.Tensor, bhh: torch.Tensor, reverse: bool) -> torch.Tensor:
    """One LSTM direction: gates = gx[t] + (W_hh h + b_hh), order i, f, g, o
    (lstm_seq_batched, kernels/kokoro.cu:400-450). gx [T, 4H] already includes W_ih x + b_ih."""
    T = gx.shape[0]
    H = whh.shape[1]
    h = torch.zeros(H)
    c = torch.zeros(H)
    out = torch.zeros(T, H)
    for t in (range(T - 1, -1, -1) if reverse else range(T)):
        g = gx[t] + (whh @ h + bhh)
        i, f_, gg, o = g[:H], g[H:2 * H], g[2 * H:3 * H], g[3 * H:]
        c = torch.sigmoid(f_) * c + torch.sigmoid(i) * torch.tanh(gg)
        h = torch.sigmoid(o) * torch.tanh(c)
        out[t] = h
    return out


# ----------------------------------------------------------------------------- WAV output

WAV_PCM16, WAV_FLOAT32 = 0, 1
WAV_MAX_DATA_BYTES = 0xFFFFFFFF - 36  # src/wav.rs:23-24


def wav_header(fmt: int, sample_rate: int, data_bytes: int) -> bytes:
    """Canonical 44-byte RIFF/WAVE header (src/wav.rs:44-61); ValueError above the RIFF limit."""
    if data_bytes > WAV_MAX_DATA_BYTES:
        raise ValueError("the audio exceeds the 4 GiB limit of a WAV file")
    bits, tag = (32, 3) if fmt == WAV_FLOAT32 else (16, 1)
    le = lambda v, n: int(v).to_bytes(n, "little")  # noqa: E731
    return (b"RIFF" + le(36 + data_bytes, 4) + b"WAVEfmt " + le(16, 4) + le(tag, 2) + le(1, 2) + le(sample_rate, 4) +
            le(sample_rate * bits // 8, 4) + le(bits // 8, 2) + le(bits, 2) + b"data" + le(data_bytes, 4))


def wav_encode(audio: np.ndarray, sample_rate: int, fmt: int):
    """(bytes, clipped) as src/wav.rs:63-87: PCM_16 = f32 (s * 32767) rounded half to even; values
    outside [-32768, 32767] are counted and clamped; NaN counts and becomes 0 (Rust's saturating
    cast)."""
    a = np.asarray(audio, np.float32)
    if fmt == WAV_FLOAT32:
        return wav_header(fmt, sample_rate, a.size * 4) + a.astype("<f4").tobytes(), 0
    v = np.rint(a * np.float32(32767.0))  # numpy rint: round half to even
    bad = ~((v >= -32768.0) & (v <= 32767.0))
    q = np.where(np.isnan(v), 0.0, np.clip(v, -32768.0, 32767.0)).astype(np.int16)
    return wav_header(fmt, sample_rate, a.size * 2) + q.astype("<i2").tobytes(), int(bad.sum())


# ----------------------------------------------------------------------------- model

class KokoroOracle:
    """fp32 CPU restatement of the Kokoro-82M forward on a raw state dict (numpy arrays)."""

    def __init__(self, sd: "dict[str, np.ndarray]", threads: int | None = None):
        if threads:
            torch.set_num_threads(threads)
        self.sd = sd
        self.trace = None  # dict: stage name -> time-major array, when set (diagnostics)

    def _rec(self, name, x, channel_major=True):
        if self.trace is not None:
            a = x.numpy() if isinstance(x, torch.Tensor) else np.asarray(x)
            self.trace[name] = (a.T if channel_major and a.ndim == 2 else a).copy()

    # -- weights
    def t(self, name):
        return torch.from_numpy(np.ascontiguousarray(self.sd[name], dtype=F32))

    def conv_w(self, prefix):
        """src/weights.rs:62-70: plain .weight if present, else weight_norm(weight_v, weight_g)."""
        if prefix + ".weight" in self.sd:
            return self.t(prefix + ".weight")
        return torch.from_numpy(weight_norm(self.sd[prefix + ".weight_v"], self.sd[prefix + ".weight_g"]))

    def bias(self, prefix):
        k = prefix + ".bias"
        return self.t(k) if k in self.sd else None

    def norm_affine(self, prefix, c):
        """src/weights.rs:76-84: AdaIN InstanceNorm affine defaults to 1 / 0 when absent."""
        w = self.sd.get(prefix + ".norm.weight")
        b = self.sd.get(prefix + ".norm.bias")
        return (np.ones(c, F32) if w is None else w.astype(F32), np.zeros(c, F32) if b is None else b.astype(F32))

    def linear(self, x, prefix):
        y = x @ self.t(prefix + ".weight").T
        b = self.bias(prefix)
        return y + b if b is not None else y

    def conv(self, x, prefix, stride=1, pad=0, dil=1):
        """Conv1d on [C, T] (zero padding = per-item padding in the ragged layout)."""
        return F.conv1d(x[None], self.conv_w(prefix), self.bias(prefix), stride=stride, padding=pad, dilation=dil)[0]

    # -- ALBERT (src/albert.rs:67-81, src/gpu_batch.rs:423-455)
    def albert(self, ids):
        T = len(ids)
        we = self.sd["bert.embeddings.word_embeddings.weight"][ids]
        pe = self.sd["bert.embeddings.position_embeddings.weight"][:T]
        tt = self.sd["bert.embeddings.token_type_embeddings.weight"][0]
        x = ((we + tt[None, :]).astype(F32) + pe).astype(F32)
        x = ln_rows(x, self.sd["bert.embeddings.LayerNorm.weight"], self.sd["bert.embeddings.LayerNorm.bias"], 1e-12)
        h = self.linear(torch.from_numpy(x), "bert.encoder.embedding_hidden_mapping_in")
        L = "bert.encoder.albert_layer_groups.0.albert_layers.0"
        for _ in range(ALBERT_LAYERS):
            q = self.linear(h, f"{L}.attention.query").view(T, HEADS, HEAD_DIM).transpose(0, 1)
            k = self.linear(h, f"{L}.attention.key").view(T, HEADS, HEAD_DIM).transpose(0, 1)
            v = self.linear(h, f"{L}.attention.value").view(T, HEADS, HEAD_DIM).transpose(0, 1)
            p = torch.softmax((q @ k.transpose(1, 2)) * (HEAD_DIM ** -0.5), dim=-1)
            ctx = (p @ v).transpose(0, 1).reshape(T, HEADS * HEAD_DIM)
            a = self.linear(ctx, f"{L}.attention.dense") + h
            a = torch.from_numpy(ln_rows(a.numpy(), self.sd[f"{L}.attention.LayerNorm.weight"], self.sd[f"{L}.attention.LayerNorm.bias"], 1e-12))
            f = gelu_new(self.linear(a, f"{L}.ffn"))
            o = self.linear(f, f"{L}.ffn_output") + a
            h = torch.from_numpy(ln_rows(o.numpy(), self.sd[f"{L}.full_layer_layer_norm.weight"], self.sd[f"{L}.full_layer_layer_norm.bias"], 1e-12))
        return h

    # -- LSTM (kernels/kokoro.cu:400-450; torch gate order i, f, g, o)
    def bilstm(self, x, prefix):
        outs = []
        for sfx, rev in (("", False), ("_reverse", True)):
            gx = x @ self.t(f"{prefix}.weight_ih_l0{sfx}").T + self.t(f"{prefix}.bias_ih_l0{sfx}")
            outs.append(lstm_dir(gx, self.t(f"{prefix}.weight_hh_l0{sfx}"), self.t(f"{prefix}.bias_hh_l0{sfx}"), rev))
        return torch.cat(outs, dim=1)

    # -- AdaIN family (kernels/kokoro.cu:776-810, 317-334)
    def adain(self, x, prefix, s, c):
        """AdaIN1d on x [C, T] with style s [128]: per-channel biased stats (eps 1e-5), affine,
        then (1 + gamma) * . + beta."""
        gb = self.linear(s, prefix + ".fc")
        xn = x.numpy().astype(np.float64)
        mean = xn.mean(axis=1).astype(F32)
        var = ((xn - xn.mean(axis=1, keepdims=True)) ** 2).mean(axis=1).astype(F32)
        rstd = (F32(1.0) / np.sqrt(var + F32(1e-5))).astype(F32)
        nw, nb = self.norm_affine(prefix, c)
        v = (x - torch.from_numpy(mean)[:, None]) * torch.from_numpy(rstd)[:, None]
        v = v * torch.from_numpy(nw)[:, None] + torch.from_numpy(nb)[:, None]
        return (1.0 + gb[:c])[:, None] * v + gb[c:][:, None]

    def resblk(self, x, prefix, s, din, dout, upsample):
        """AdainResBlk1d (src/gpu_batch.rs:103-135)."""
        r = F.leaky_relu(self.adain(x, prefix + ".norm1", s, din), 0.2)
        if upsample:
            w = self.conv_w(prefix + ".pool")
            r = F.conv_transpose1d(r[None], w, self.bias(prefix + ".pool"), stride=2, padding=1, output_padding=1, groups=din)[0]
        r = self.conv(r, prefix + ".conv1", pad=1)
        r = F.leaky_relu(self.adain(r, prefix + ".norm2", s, dout), 0.2)
        r = self.conv(r, prefix + ".conv2", pad=1)
        sc = x.repeat_interleave(2, dim=1) if upsample else x
        if din != dout:
            sc = self.conv(sc, prefix + ".conv1x1")
        return (r + sc) * float(F32(1.0) / np.sqrt(F32(2.0)))

    def snake_block(self, x, prefix, s, c, k):
        """AdaINResBlock1 with Snake x + sin(a x)^2 / a (src/gpu_batch.rs:137-154)."""
        for i, d in enumerate((1, 3, 5)):
            a1 = self.t(f"{prefix}.alpha1.{i}")[0]
            a2 = self.t(f"{prefix}.alpha2.{i}")[0]
            xt = self.adain(x, f"{prefix}.adain1.{i}", s, c)
            xt = xt + (1.0 / a1) * torch.sin(a1 * xt) ** 2
            xt = self.conv(xt, f"{prefix}.convs1.{i}", pad=(k * d - d) // 2, dil=d)
            xt = self.adain(xt, f"{prefix}.adain2.{i}", s, c)
            xt = xt + (1.0 / a2) * torch.sin(a2 * xt) ** 2
            xt = self.conv(xt, f"{prefix}.convs2.{i}", pad=(k - 1) // 2)
            x = xt + x
        return x

    # -- text side
    def text_encoder(self, ids):
        """src/gpu_batch.rs:457-481."""
        x = self.t("text_encoder.embedding.weight")[ids].T.contiguous()  # [512, T]
        for i in range(3):
            y = self.conv(x, f"text_encoder.cnn.{i}.0", pad=2)
            y = ln_rows(y.T.numpy(), self.sd[f"text_encoder.cnn.{i}.1.gamma"], self.sd[f"text_encoder.cnn.{i}.1.beta"], 1e-5)
            x = F.leaky_relu(torch.from_numpy(y), 0.2).T.contiguous()
        return self.bilstm(x.T.contiguous(), "text_encoder.lstm")  # [T, 512]

    def duration_side(self, ids, s_pro, speed):
        """ALBERT -> bert_encoder -> duration encoder -> predictor LSTM -> duration logits
        (src/gpu_batch.rs:216-248).  Returns (d [T, 640], logits [T, 50])."""
        bert = self.albert(ids)
        d_en = self.linear(bert, "bert_encoder")
        T = d_en.shape[0]
        sp = s_pro[None, :].expand(T, STYLE_DIM)
        x = torch.cat([d_en, sp], dim=1)
        for i in range(3):
            h = self.bilstm(x, f"predictor.text_encoder.lstms.{2 * i}")
            gb = self.linear(s_pro, f"predictor.text_encoder.lstms.{2 * i + 1}.fc").numpy()
            o = ln_rows(h.numpy(), None, None, 1e-5)
            h = torch.from_numpy(((F32(1.0) + gb[:HIDDEN]) * o + gb[HIDDEN:]).astype(F32))
            x = torch.cat([h, sp], dim=1)
        self._rec("bert", bert, False)
        self._rec("x640", x, False)
        xl = self.bilstm(x, "predictor.lstm")
        logits = self.linear(xl, "predictor.duration_proj.linear_layer")
        self._rec("logits", logits, False)
        return x, logits

    def f0n(self, en, s_pro):
        """Shared LSTM + F0/N AdainResBlk1d stacks + 1x1 projections (src/gpu_batch.rs:281-292)."""
        sh = self.bilstm(en, "predictor.shared").T.contiguous()  # [512, N]
        self._rec("sh", sh)
        outs = []
        for name in ("F0", "N"):
            h = self.resblk(sh, f"predictor.{name}.0", s_pro, 512, 512, False)
            h = self.resblk(h, f"predictor.{name}.1", s_pro, 512, 256, True)
            h = self.resblk(h, f"predictor.{name}.2", s_pro, 256, 256, False)
            outs.append(self.conv(h, f"predictor.{name}_proj")[0])
        return outs[0], outs[1]

    # -- decoder + generator
    def decode(self, asr, f0, n, s_dec, noise):
        """Decoder + iSTFTNet generator for one item (src/gpu_batch.rs:299-420).

        asr [512, N], f0 / n [2N], s_dec [128], noise: [600 N * 9] sine-noise draws."""
        g = "decoder.generator"
        f0 = torch.as_tensor(np.asarray(f0, F32))
        n = torch.as_tensor(np.asarray(n, F32))
        N = asr.shape[1]
        f0n = self.conv(f0[None], "decoder.F0_conv", stride=2, pad=1)
        nn_ = self.conv(n[None], "decoder.N_conv", stride=2, pad=1)
        self._rec("xcat0", torch.cat([asr, f0n, nn_], 0))
        x = self.resblk(torch.cat([asr, f0n, nn_], 0), "decoder.encode", s_dec, 514, 1024, False)
        self._rec("enc", x)
        asr_res = self.conv(asr, "decoder.asr_res.0")
        for i in range(4):
            x = torch.cat([x, asr_res, f0n, nn_], 0)
            x = self.resblk(x, f"decoder.decode.{i}", s_dec, 1090, 1024 if i < 3 else 512, i == 3)
        self._rec("xd", x)
        # harmonic source + STFT
        har = sinegen_har(f0.numpy(), noise, self.sd[f"{g}.m_source.l_linear.weight"][0], float(self.sd[f"{g}.m_source.l_linear.bias"][0]))
        spec = torch.from_numpy(stft20(har))  # [22, 120N + 1]
        self._rec("har", har, False)
        self._rec("spec", spec)
        for i in range(2):
            x = F.leaky_relu(x, 0.1)
            if i == 0:
                xs = self.conv(spec, f"{g}.noise_convs.0", stride=6, pad=3)
                self._rec("xs0", xs)
                xs = self.snake_block(xs, f"{g}.noise_res.0", s_dec, 256, 7)
                self._rec("xsr0", xs)
                x = F.conv_transpose1d(x[None], self.conv_w(f"{g}.ups.0"), self.bias(f"{g}.ups.0"), stride=10, padding=5)[0]
            else:
                xs = self.conv(spec, f"{g}.noise_convs.1")
                xs = self.snake_block(xs, f"{g}.noise_res.1", s_dec, 128, 11)
                self._rec("xsr1", xs)
                x = F.conv_transpose1d(x[None], self.conv_w(f"{g}.ups.1"), self.bias(f"{g}.ups.1"), stride=6, padding=3)[0]
                x = torch.cat([x[:, 1:2], x], dim=1)  # ReflectionPad1d((1, 0))
            x = x + xs
            self._rec("y0" if i == 0 else "y1", x)
            ch = 256 if i == 0 else 128
            acc = None
            for j, k in enumerate((3, 7, 11)):
                r = self.snake_block(x, f"{g}.resblocks.{i * 3 + j}", s_dec, ch, k)
                if j == 0 and i == 0:
                    self._rec("r0_0", r)
                acc = r if acc is None else acc + r
            x = acc / 3.0
            self._rec("x1" if i == 0 else "x2", x)
        x = F.leaky_relu(x, 0.01)
        post = self.conv(x, f"{g}.conv_post", pad=3)
        audio = istft20(post.numpy())
        self._rec("post", post)
        self._rec("audio", audio, False)
        assert audio.shape[0] == SAMPLES_PER_FRAME * N
        return audio

    @torch.no_grad()
    def forward(self, ids, ref_s, speed=1.0, seed=0, noise=None, forced_dur=None, want=()):
        """One utterance: ids [T] (pads included), ref_s [256].  Returns dict with ``audio``,
        ``dur`` and any intermediates named in ``want`` (logits, dur_q, f0, n)."""
        ids = np.asarray(ids, np.int64)
        ref_s = np.asarray(ref_s, F32)
        s_dec = torch.from_numpy(ref_s[:STYLE_DIM].copy())
        s_pro = torch.from_numpy(ref_s[STYLE_DIM:].copy())
        d, logits = self.duration_side(ids, s_pro, speed)
        dur, q = durations_from_logits(logits.numpy(), speed)
        if forced_dur is not None:
            dur = np.asarray(forced_dur, np.int64)
        src = np.repeat(np.arange(len(ids)), dur)
        N = src.shape[0]
        en = d[src]
        f0, n = self.f0n(en, s_pro)
        self._rec("f0", f0, False)
        self._rec("nc", n, False)
        t_en = self.text_encoder(ids)
        asr = t_en[src].T.contiguous()
        self._rec("t_en", t_en, False)
        if noise is None:
            noise = counter_noise(seed, SAMPLES_PER_FRAME * N * HARMONICS)
        audio = self.decode(asr, f0, n, s_dec, noise)
        out = {"audio": audio, "dur": dur}
        if "logits" in want:
            out["logits"] = logits.numpy()
        if "dur_q" in want:
            out["dur_q"] = q
        if "f0" in want:
            out["f0"], out["n"] = f0.numpy(), n.numpy()
        if "asr" in want:  # text encoder output per token [T, 512] and aligned per frame [512, N]
            out["t_en"], out["asr"] = t_en.numpy(), asr.numpy()
        return out

    @torch.no_grad()
    def durations(self, ids, ref_s, speed=1.0):
        """Predicted durations only (src/gpu_batch.rs:216-248, src/model.rs:90-99): (dur, unrounded)."""
        ids = np.asarray(ids, np.int64)
        ref_s = np.asarray(ref_s, F32)
        _d, logits = self.duration_side(ids, torch.from_numpy(ref_s[STYLE_DIM:].copy()), speed)
        return durations_from_logits(logits.numpy(), speed)
