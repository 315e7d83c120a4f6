"""PyTorch zip checkpoint reader (kk_pth_*, mirror of src/torchpt.rs) on files written by
torch.save: flat names, exact values for contiguous, strided and offset views, voice packs, and the
refusals the reference makes (compressed entries, unsupported globals, wrong voice shapes)."""
import os
import zipfile
from collections import OrderedDict

import numpy as np
import pytest


@pytest.fixture(scope="module")
def torch():
    import torch as t
    return t


def test_checkpoint_round_trip(kk, torch, tmp_path):
    g = torch.Generator().manual_seed(0)
    base = torch.randn(6, 10, generator=g)
    sd_a = OrderedDict()
    sd_a["module.embeddings.weight"] = torch.randn(5, 3, generator=g)
    sd_a["layer.bias"] = torch.randn(7, generator=g)
    sd_a["proj.weight"] = base.t()                  # strided view
    sd_a["tail.weight"] = base[2:4, 3:9]             # view with a storage offset, shared storage
    sd_b = OrderedDict(w=torch.randn(2, 1, 4, generator=g), s=torch.tensor(3.5))
    path = str(tmp_path / "m.pth")
    torch.save({"bert": sd_a, "decoder": sd_b}, path)
    got = kk.pth.load_kmodel_checkpoint(path)
    want = {"bert.embeddings.weight": sd_a["module.embeddings.weight"], "bert.layer.bias": sd_a["layer.bias"],
            "bert.proj.weight": sd_a["proj.weight"], "bert.tail.weight": sd_a["tail.weight"],
            "decoder.w": sd_b["w"], "decoder.s": sd_b["s"]}
    assert sorted(got) == sorted(want)
    for k, t in want.items():
        assert got[k].shape == tuple(t.shape) and np.array_equal(got[k], t.contiguous().numpy()), k


def test_voice_pack(kk, torch, tmp_path):
    v = torch.randn(510, 1, 256, generator=torch.Generator().manual_seed(1))
    p = str(tmp_path / "af.pt")
    torch.save(v, p)
    assert np.array_equal(kk.pth.load_voice_pack(p), v.numpy())
    torch.save(torch.randn(510, 256), str(tmp_path / "bad.pt"))
    with pytest.raises(kk.pth.PthError, match="unexpected voice pack shape"):
        kk.pth.load_voice_pack(str(tmp_path / "bad.pt"))


def test_refusals(kk, torch, tmp_path):
    p = str(tmp_path / "half.pth")
    torch.save({"m": OrderedDict(w=torch.zeros(3, dtype=torch.float16))}, p)
    with pytest.raises(kk.pth.PthError, match="unsupported pickle global torch.HalfStorage"):
        kk.pth.load_kmodel_checkpoint(p)
    p = str(tmp_path / "param.pth")
    torch.save({"m": OrderedDict(w=torch.nn.Parameter(torch.zeros(3)))}, p)
    with pytest.raises(kk.pth.PthError, match="unsupported pickle global"):
        kk.pth.load_kmodel_checkpoint(p)
    # the same archive with deflated entries
    src = str(tmp_path / "ok.pth")
    torch.save({"m": OrderedDict(w=torch.ones(4))}, src)
    dst = str(tmp_path / "deflated.pth")
    with zipfile.ZipFile(src) as zi, zipfile.ZipFile(dst, "w", zipfile.ZIP_DEFLATED) as zo:
        for info in zi.infolist():
            zo.writestr(info.filename, zi.read(info.filename))
    with pytest.raises(kk.pth.PthError, match="compressed"):
        kk.pth.load_kmodel_checkpoint(dst)
    with pytest.raises(kk.pth.PthError):
        kk.pth.load_kmodel_checkpoint(str(tmp_path / "missing.pth"))


def test_engine_voices_from_model_dir(kk, torch, tmp_path):
    """Engine.voice: voices/<name>.pt under the model directory, explicit .pt paths, and the
    element-wise mean of a comma-separated list (src/engine.rs:115-137)."""
    os.makedirs(tmp_path / "voices")
    g = torch.Generator().manual_seed(2)
    a, b = torch.randn(510, 1, 256, generator=g), torch.randn(510, 1, 256, generator=g)
    torch.save(a, str(tmp_path / "voices" / "af.pt"))
    torch.save(b, str(tmp_path / "bm.pt"))
    e = kk.Engine.__new__(kk.Engine)
    e.model_dir, e.voices = str(tmp_path), {}
    va = e.voice("af")
    assert np.array_equal(va.pack, a.numpy().reshape(510, 256)) and len(va.sha256) == 64
    vb = e.voice(str(tmp_path / "bm.pt"))
    mix = e.voice("af," + str(tmp_path / "bm.pt"))
    assert np.array_equal(mix.pack, ((a + b) / 2).numpy().reshape(510, 256))
    assert mix.sha256 == va.sha256 + "," + vb.sha256
    with pytest.raises(kk.pth.PthError):
        e.voice("nobody")


@pytest.mark.gpu
def test_engine_from_pth_equals_safetensors(kk, torch, ckpt_path, tmp_path):
    """kk_create on the PyTorch checkpoint layout ({submodule: state_dict}) hydrates the same
    weights as from safetensors: identical decoder output."""
    from kokoro_rust_b200 import weights
    flat = weights.load_safetensors(ckpt_path)
    subs = OrderedDict()
    for name, arr in flat.items():
        sub, param = name.split(".", 1)
        subs.setdefault(sub, OrderedDict())[param] = torch.from_numpy(np.ascontiguousarray(arr, np.float32))
    pth = str(tmp_path / "kokoro.pth")
    torch.save(subs, pth)
    rng = np.random.default_rng(9)
    n = 11
    asr = rng.standard_normal((n, 512)).astype(np.float32)
    f0 = np.exp(rng.uniform(np.log(80), np.log(400), 2 * n)).astype(np.float32)
    nc = rng.standard_normal(2 * n).astype(np.float32)
    s_dec = (rng.standard_normal((1, 128)) * 0.1).astype(np.float32)
    outs = []
    for p in (ckpt_path, pth):
        e = kk.GpuKokoro(p, 0, "fp32")
        outs.append(e.decode_batch([asr], [f0], [nc], s_dec, seeds=[3])[0])
        e.close()
    assert np.array_equal(outs[0], outs[1])
