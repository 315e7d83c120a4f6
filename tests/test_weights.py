"""Checkpoint manifest and codec: structural known answers of the reference's state dict."""
import os
import struct

import numpy as np
import pytest


def test_census_matches_reference_state_dict(kk):
    """688 raw keys, 89 weight-normed modules, 81,810,022 params (reference oracle/dump_weights.py
    census) once the 140 absent AdaIN affine params are counted (tests/native_load.rs:33-41)."""
    w = kk.weights
    n, n_wn, numel = w.census()
    m = w.manifest()
    # AdaIN modules: every '*.fc.weight' whose parent is an AdaIN1d (norm1/norm2/adain1/adain2)
    adain = [k[: -len(".fc.weight")] for k in m if k.endswith(".fc.weight") and
             (".norm1." in k or ".norm2." in k or ".adain1." in k or ".adain2." in k)]
    assert len(adain) == 70
    affine_numel = sum(2 * m[p + ".fc.weight"][0][0] // 2 for p in adain)
    assert n + 2 * len(adain) == 688
    assert n_wn == 89
    assert numel + affine_numel == 81_810_022


def test_manifest_shapes_follow_loaders(kk):
    m = kk.weights.manifest()
    assert m["decoder.generator.ups.0.weight_v"][0] == (512, 256, 20)      # ConvT [cin, cout, k]
    assert m["decoder.generator.ups.0.weight_g"][0] == (512, 1, 1)         # weight_norm dim 0
    assert m["decoder.decode.3.pool.weight_v"][0] == (1090, 1, 3)          # depthwise ConvT
    assert m["decoder.generator.m_source.l_linear.weight"][0] == (1, 9)
    assert m["predictor.text_encoder.lstms.0.weight_ih_l0_reverse"][0] == (1024, 640)
    assert m["decoder.generator.resblocks.5.convs1.2.weight_v"][0] == (128, 128, 11)
    assert "decoder.generator.noise_convs.0.weight" in m  # plain conv (not weight-normed)
    assert not any(k.endswith(".norm.weight") or k.endswith(".norm.bias") for k in m)


def test_random_init_deterministic_and_calibrated(kk):
    a = kk.weights.random_init(0)
    b = kk.weights.random_init(0)
    c = kk.weights.random_init(1)
    for k in ("bert.embeddings.word_embeddings.weight", "decoder.generator.conv_post.weight_v"):
        assert np.array_equal(a[k], b[k]) and not np.array_equal(a[k], c[k])
    # duration head: ~2.2 frames per token at zero input
    bias = a["predictor.duration_proj.linear_layer.bias"].astype(np.float64)
    assert 1.5 < (1 / (1 + np.exp(-bias))).sum() < 3.5
    # weight_g = ||v|| * U(0.8, 1.2)
    v = a["decoder.encode.conv1.weight_v"].reshape(1024, -1).astype(np.float64)
    g = a["decoder.encode.conv1.weight_g"].reshape(-1)
    r = g / np.sqrt((v * v).sum(1))
    assert r.min() > 0.79 and r.max() < 1.21


def test_safetensors_round_trip(tmp_path, kk):
    w = kk.weights
    t = {"a": np.arange(6, dtype=np.float32).reshape(2, 3), "b": np.array([1.5], np.float64),
         "c": np.array([-3, 4], np.int64)}
    p = str(tmp_path / "x.safetensors")
    w.save_safetensors(p, t)
    r = w.load_safetensors(p)
    for k in t:
        assert r[k].dtype == t[k].dtype and np.array_equal(r[k], t[k])


def test_corrupt_safetensors_refused(tmp_path, kk):
    w = kk.weights
    p = str(tmp_path / "x.safetensors")
    w.save_safetensors(p, {"a": np.ones(4, np.float32)})
    raw = open(p, "rb").read()
    bad = tmp_path / "trunc.safetensors"
    bad.write_bytes(raw[: len(raw) // 2])
    with pytest.raises(Exception):
        w.load_safetensors(str(bad))
    huge = tmp_path / "hlen.safetensors"
    huge.write_bytes(struct.pack("<Q", 1 << 40) + raw[8:])
    with pytest.raises(ValueError):
        w.load_safetensors(str(huge))
    short = tmp_path / "short.safetensors"
    short.write_bytes(b"abc")
    with pytest.raises(ValueError):
        w.load_safetensors(str(short))
    f16 = tmp_path / "f16.safetensors"
    h = b'{"a":{"dtype":"F16","shape":[2],"data_offsets":[0,4]}}'
    f16.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 4)
    with pytest.raises(ValueError):
        w.load_safetensors(str(f16))


def test_weight_norm_matches_torch(oracle_mod):
    import torch
    rng = np.random.default_rng(0)
    v = rng.standard_normal((6, 5, 3)).astype(np.float32)
    g = rng.uniform(0.5, 2, (6, 1, 1)).astype(np.float32)
    ours = oracle_mod.weight_norm(v, g)
    ref = torch._weight_norm(torch.from_numpy(v), torch.from_numpy(g), 0).numpy()
    assert np.abs(ours - ref).max() <= 1e-6
