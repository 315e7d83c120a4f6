"""Kokoro-82M state-dict manifest, seeded random-init generator and a minimal safetensors codec.

The manifest lists every tensor the model loaders of the reference crate read, with their exact
names and shapes, in the checkpoint's raw form (weight-normed convolutions as ``weight_v`` +
``weight_g``):

* ALBERT (PL-BERT): ``src/albert.rs:36-64``
* ``bert_encoder``: ``src/model.rs:136``
* text encoder: ``src/model.rs:29-44``
* predictor: ``src/model.rs:60-86``
* decoder + iSTFTNet generator: ``src/vocoder.rs:54-111``
* layer suffix patterns (Linear, Conv1d, ConvTranspose1d, AdaIN1d, AdainResBlk1d, AdaINResBlock1,
  BiLSTM): ``src/nn.rs:15-189``

The AdaIN ``InstanceNorm1d`` affine parameters (``*.norm.weight`` / ``*.norm.bias``) are absent
from the real checkpoint and default to 1 / 0 (``src/weights.rs:76-84``); the generator leaves
them out so that the loaders' defaulting path is exercised.

Random init follows torch's default initialisers (kaiming-uniform bounds 1/sqrt(fan_in),
weight_norm ``g = ||v||``), perturbed so that no parameter class is trivially constant, plus two
calibrations that keep synthetic inputs in a realistic operating range:

* ``predictor.duration_proj.linear_layer``: bias ``logit(2.2/50)`` and weight std 0.02, giving
  about 2.2 frames per token (the reference's real-model ratio is 2.37 frames per phoneme char);
* ``predictor.F0_proj``: bias 120 Hz and gain 110, so that the harmonic source sees both voiced
  (F0 > 10 Hz) and unvoiced frames.
"""
from __future__ import annotations

import json
import math
import os
import struct
from collections import OrderedDict

import numpy as np

STYLE_DIM = 128
HIDDEN = 512
MAX_DUR = 50
N_TOKEN = 178
ALBERT_EMB, ALBERT_HID, ALBERT_FFN, MAX_POS = 128, 768, 2048, 512
ALBERT_LAYER = "bert.encoder.albert_layer_groups.0.albert_layers.0"

# Tensor kinds drive the initialiser: "lin_w", "bias", "conv_v", "conv_g", "convT_v",
# "plain_conv_w", "emb", "albert_emb", "ln_w", "ln_b", "lstm", "alpha", and the calibrated heads.


def _linear(m, prefix, din, dout, bias=True):
    m[f"{prefix}.weight"] = ((dout, din), "lin_w", din)
    if bias:
        m[f"{prefix}.bias"] = ((dout,), "bias", din)


def _conv_wn(m, prefix, cin, cout, k, bias=True):
    """weight_norm(Conv1d): weight_v [cout, cin, k], weight_g [cout, 1, 1] (src/nn.rs:36-57)."""
    m[f"{prefix}.weight_g"] = ((cout, 1, 1), "conv_g", cin * k)
    m[f"{prefix}.weight_v"] = ((cout, cin, k), "conv_v", cin * k)
    if bias:
        m[f"{prefix}.bias"] = ((cout,), "bias", cin * k)


def _conv_plain(m, prefix, cin, cout, k, bias=True):
    m[f"{prefix}.weight"] = ((cout, cin, k), "plain_conv_w", cin * k)
    if bias:
        m[f"{prefix}.bias"] = ((cout,), "bias", cin * k)


def _lstm(m, prefix, din, h):
    """nn.LSTM(din, h, bidirectional) single layer (src/nn.rs:170-189)."""
    for sfx in ("", "_reverse"):
        m[f"{prefix}.weight_ih_l0{sfx}"] = ((4 * h, din), "lstm", h)
        m[f"{prefix}.weight_hh_l0{sfx}"] = ((4 * h, h), "lstm", h)
        m[f"{prefix}.bias_ih_l0{sfx}"] = ((4 * h,), "lstm", h)
        m[f"{prefix}.bias_hh_l0{sfx}"] = ((4 * h,), "lstm", h)


def _adain(m, prefix, c):
    """AdaIN1d: fc Linear(style, 2c); norm affine absent from the checkpoint (src/nn.rs:87-100)."""
    _linear(m, f"{prefix}.fc", STYLE_DIM, 2 * c)


def _adain_resblk1d(m, prefix, din, dout, upsample):
    """StyleTTS2 AdainResBlk1d (src/nn.rs:103-141)."""
    _conv_wn(m, f"{prefix}.conv1", din, dout, 3)
    _conv_wn(m, f"{prefix}.conv2", dout, dout, 3)
    _adain(m, f"{prefix}.norm1", din)
    _adain(m, f"{prefix}.norm2", dout)
    if din != dout:
        _conv_wn(m, f"{prefix}.conv1x1", din, dout, 1, bias=False)
    if upsample:
        # depthwise ConvTranspose1d(din, din, 3, stride 2, groups din): weight [din, 1, 3]
        m[f"{prefix}.pool.weight_g"] = ((din, 1, 1), "conv_g", 3)
        m[f"{prefix}.pool.weight_v"] = ((din, 1, 3), "conv_v", 3)
        m[f"{prefix}.pool.bias"] = ((din,), "bias", 3)


def _adain_resblock1(m, prefix, c, k):
    """iSTFTNet AdaINResBlock1 with Snake, dilations (1, 3, 5) (src/nn.rs:143-166)."""
    for i in range(3):
        _conv_wn(m, f"{prefix}.convs1.{i}", c, c, k)
    for i in range(3):
        _conv_wn(m, f"{prefix}.convs2.{i}", c, c, k)
    for i in range(3):
        _adain(m, f"{prefix}.adain1.{i}", c)
    for i in range(3):
        _adain(m, f"{prefix}.adain2.{i}", c)
    for i in range(3):
        m[f"{prefix}.alpha1.{i}"] = ((1, c, 1), "alpha", 1)
    for i in range(3):
        m[f"{prefix}.alpha2.{i}"] = ((1, c, 1), "alpha", 1)


def manifest() -> "OrderedDict[str, tuple]":
    """Ordered {name: (shape, kind, fan_in)} for the raw Kokoro-82M state dict."""
    m: "OrderedDict[str, tuple]" = OrderedDict()
    # ---- ALBERT (src/albert.rs:36-64)
    m["bert.embeddings.word_embeddings.weight"] = ((N_TOKEN, ALBERT_EMB), "albert_emb", 1)
    m["bert.embeddings.position_embeddings.weight"] = ((MAX_POS, ALBERT_EMB), "albert_emb", 1)
    m["bert.embeddings.token_type_embeddings.weight"] = ((2, ALBERT_EMB), "albert_emb", 1)
    m["bert.embeddings.LayerNorm.weight"] = ((ALBERT_EMB,), "ln_w", 1)
    m["bert.embeddings.LayerNorm.bias"] = ((ALBERT_EMB,), "ln_b", 1)
    _linear(m, "bert.encoder.embedding_hidden_mapping_in", ALBERT_EMB, ALBERT_HID)
    L = ALBERT_LAYER
    m[f"{L}.full_layer_layer_norm.weight"] = ((ALBERT_HID,), "ln_w", 1)
    m[f"{L}.full_layer_layer_norm.bias"] = ((ALBERT_HID,), "ln_b", 1)
    for n in ("query", "key", "value", "dense"):
        _linear(m, f"{L}.attention.{n}", ALBERT_HID, ALBERT_HID)
    m[f"{L}.attention.LayerNorm.weight"] = ((ALBERT_HID,), "ln_w", 1)
    m[f"{L}.attention.LayerNorm.bias"] = ((ALBERT_HID,), "ln_b", 1)
    _linear(m, f"{L}.ffn", ALBERT_HID, ALBERT_FFN)
    _linear(m, f"{L}.ffn_output", ALBERT_FFN, ALBERT_HID)
    # AlbertModel's pooler: in the checkpoint, unused by the forward
    _linear(m, "bert.pooler", ALBERT_HID, ALBERT_HID)
    # ---- bert_encoder (src/model.rs:136)
    _linear(m, "bert_encoder", ALBERT_HID, HIDDEN)
    # ---- predictor (src/model.rs:60-86)
    cin = HIDDEN + STYLE_DIM
    for i in range(3):
        _lstm(m, f"predictor.text_encoder.lstms.{2 * i}", cin, HIDDEN // 2)
        _linear(m, f"predictor.text_encoder.lstms.{2 * i + 1}.fc", STYLE_DIM, 2 * HIDDEN)
    _lstm(m, "predictor.lstm", cin, HIDDEN // 2)
    m["predictor.duration_proj.linear_layer.weight"] = ((MAX_DUR, HIDDEN), "dur_w", HIDDEN)
    m["predictor.duration_proj.linear_layer.bias"] = ((MAX_DUR,), "dur_b", HIDDEN)
    _lstm(m, "predictor.shared", cin, HIDDEN // 2)
    for name in ("F0", "N"):
        _adain_resblk1d(m, f"predictor.{name}.0", HIDDEN, HIDDEN, False)
        _adain_resblk1d(m, f"predictor.{name}.1", HIDDEN, HIDDEN // 2, True)
        _adain_resblk1d(m, f"predictor.{name}.2", HIDDEN // 2, HIDDEN // 2, False)
    m["predictor.F0_proj.weight"] = ((1, HIDDEN // 2, 1), "f0_w", HIDDEN // 2)
    m["predictor.F0_proj.bias"] = ((1,), "f0_b", HIDDEN // 2)
    _conv_plain(m, "predictor.N_proj", HIDDEN // 2, 1, 1)
    # ---- text encoder (src/model.rs:29-44)
    m["text_encoder.embedding.weight"] = ((N_TOKEN, HIDDEN), "emb", 1)
    for i in range(3):
        _conv_wn(m, f"text_encoder.cnn.{i}.0", HIDDEN, HIDDEN, 5)
        m[f"text_encoder.cnn.{i}.1.gamma"] = ((HIDDEN,), "ln_w", 1)
        m[f"text_encoder.cnn.{i}.1.beta"] = ((HIDDEN,), "ln_b", 1)
    _lstm(m, "text_encoder.lstm", HIDDEN, HIDDEN // 2)
    # ---- decoder (src/vocoder.rs:98-111)
    _adain_resblk1d(m, "decoder.encode", 514, 1024, False)
    for i in range(3):
        _adain_resblk1d(m, f"decoder.decode.{i}", 1090, 1024, False)
    _adain_resblk1d(m, "decoder.decode.3", 1090, 512, True)
    _conv_wn(m, "decoder.F0_conv", 1, 1, 3)
    _conv_wn(m, "decoder.N_conv", 1, 1, 3)
    _conv_wn(m, "decoder.asr_res.0", 512, 64, 1)
    # ---- generator (src/vocoder.rs:54-80)
    g = "decoder.generator"
    m[f"{g}.m_source.l_linear.weight"] = ((1, 9), "lin_w", 9)
    m[f"{g}.m_source.l_linear.bias"] = ((1,), "bias", 9)
    _conv_plain(m, f"{g}.noise_convs.0", 22, 256, 12)
    _conv_plain(m, f"{g}.noise_convs.1", 22, 128, 1)
    _adain_resblock1(m, f"{g}.noise_res.0", 256, 7)
    _adain_resblock1(m, f"{g}.noise_res.1", 128, 11)
    # weight_norm(ConvTranspose1d): weight_v [cin, cout, k], weight_g [cin, 1, 1]
    for i, (ci, co, k) in enumerate(((512, 256, 20), (256, 128, 12))):
        m[f"{g}.ups.{i}.weight_g"] = ((ci, 1, 1), "conv_g", co * k)
        m[f"{g}.ups.{i}.weight_v"] = ((ci, co, k), "convT_v", co * k)
        m[f"{g}.ups.{i}.bias"] = ((co,), "bias", co * k)
    for i in range(2):
        ch = 512 >> (i + 1)
        for j, k in enumerate((3, 7, 11)):
            _adain_resblock1(m, f"{g}.resblocks.{i * 3 + j}", ch, k)
    _conv_wn(m, f"{g}.conv_post", 128, 22, 7)
    return m


def census(m=None):
    """(number of tensors, number of weight-normed modules, total element count)."""
    m = m or manifest()
    n_wn = sum(1 for k in m if k.endswith(".weight_g"))
    numel = sum(int(np.prod(s)) for s, _, _ in m.values())
    return len(m), n_wn, numel


def random_init(seed: int = 0) -> "OrderedDict[str, np.ndarray]":
    """Deterministic random init of every manifest tensor (f32), drawn in manifest order."""
    rng = np.random.default_rng(seed)
    m = manifest()
    out: "OrderedDict[str, np.ndarray]" = OrderedDict()
    pending_g = {}
    for name, (shape, kind, fan) in m.items():
        n = int(np.prod(shape))
        if kind in ("lin_w", "plain_conv_w", "conv_v", "convT_v", "bias"):
            b = 1.0 / math.sqrt(fan)
            a = rng.uniform(-b, b, n)
        elif kind == "conv_g":
            a = None  # filled once weight_v is drawn (weight_g precedes weight_v in the manifest)
            pending_g[name[: -len("weight_g")]] = shape
            a = rng.uniform(0.8, 1.2, n)  # multiplicative perturbation of ||v||, applied below
        elif kind == "lstm":
            b = 1.0 / math.sqrt(fan)
            a = rng.uniform(-b, b, n)
        elif kind == "emb":
            a = rng.standard_normal(n)
        elif kind == "albert_emb":
            a = rng.standard_normal(n) * 0.02 * 25.0  # HF init std 0.02, scaled so LN sees signal
        elif kind == "ln_w":
            a = 1.0 + 0.1 * rng.standard_normal(n)
        elif kind == "ln_b":
            a = 0.1 * rng.standard_normal(n)
        elif kind == "alpha":
            a = rng.uniform(0.5, 1.5, n)
        elif kind == "dur_w":
            a = 0.02 * rng.standard_normal(n)
        elif kind == "dur_b":
            a = math.log((2.2 / MAX_DUR) / (1.0 - 2.2 / MAX_DUR)) + 0.3 * rng.standard_normal(n)
        elif kind == "f0_w":
            a = 110.0 * rng.standard_normal(n) / math.sqrt(fan)
        elif kind == "f0_b":
            a = np.full(n, 120.0)
        else:
            raise AssertionError(kind)
        out[name] = a.astype(np.float32).reshape(shape)
        if kind in ("conv_v", "convT_v"):
            base = name[: -len("weight_v")]
            g = out[base + "weight_g"]
            v = out[name].astype(np.float64).reshape(shape[0], -1)
            norm = np.sqrt((v * v).sum(axis=1))
            out[base + "weight_g"] = (g.reshape(-1) * norm).astype(np.float32).reshape(g.shape)
    return out


# ------------------------------------------------------------------------------- safetensors

_DT = {"F32": np.float32, "F64": np.float64, "I64": np.int64, "I32": np.int32}
_DT_REV = {np.dtype(v).str: k for k, v in _DT.items()}


def save_safetensors(path: str, tensors: "dict[str, np.ndarray]") -> None:
    """Write a safetensors file (u64-LE header length, JSON directory, LE payload)."""
    header = {}
    off = 0
    blobs = []
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        dt = _DT_REV[arr.dtype.newbyteorder("<").str]
        b = arr.astype(arr.dtype.newbyteorder("<"), copy=False).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    tmp = path + ".partial"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


def load_safetensors(path: str) -> "OrderedDict[str, np.ndarray]":
    """Read a safetensors file; only F32/F64/I64/I32 are accepted (src/st.rs:84-110)."""
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 8:
        raise ValueError("file too short for header length")
    (hlen,) = struct.unpack("<Q", data[:8])
    if 8 + hlen > len(data):
        raise ValueError(f"header length {hlen} exceeds file size")
    header = json.loads(data[8 : 8 + hlen])
    payload = memoryview(data)[8 + hlen :]
    out: "OrderedDict[str, np.ndarray]" = OrderedDict()
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = info["dtype"]
        if dt not in _DT:
            raise ValueError(f"unsupported dtype {dt} for {name}")
        s, e = info["data_offsets"]
        if not (0 <= s <= e <= len(payload)):
            raise ValueError(f"offsets out of range for {name}")
        arr = np.frombuffer(payload[s:e], dtype=np.dtype(_DT[dt]).newbyteorder("<"))
        if arr.size != int(np.prod(info["shape"])):
            raise ValueError(f"size mismatch for {name}")
        out[name] = arr.reshape(info["shape"]).astype(_DT[dt])
    return out


def write_random_checkpoint(path: str, seed: int = 0) -> str:
    """Generate (if absent) the seeded random-init checkpoint at ``path``; returns the path."""
    if not os.path.exists(path):
        save_safetensors(path, random_init(seed))
    return path
