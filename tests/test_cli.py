"""The synth pipeline (src/cli.rs:450-925 semantics) on the host with a stand-in GPU: whole-file
assembly in line order, per-line resume keyed by text + configuration + audio hash, blank /
invalid / oversize lines, per-line mode and the diagnostics manifest."""
import json
import os

import numpy as np
import pytest


class FakeGpu:
    identity = "fake"

    def __init__(self, kk):
        self.kk, self.calls = kk, []

    def forward_batch(self, items):
        self.calls.append(len(items))
        outs = []
        for it in items:
            n = 600 * len(it.ids)
            t = np.arange(n, dtype=np.float64)
            a = (0.5 * np.sin(t * 0.01 * len(it.ids)) * (1 + (it.noise.seed % 7) * 0.01)).astype(np.float32)
            outs.append(self.kk.Output(a, np.ones(len(it.ids), np.int64)))
        return outs


def make_engine(kk):
    e = kk.Engine.__new__(kk.Engine)
    e.gpu = FakeGpu(kk)
    e.model_dir, e.voices = "/nonexistent", {}
    e.vocab = {c: i + 1 for i, c in enumerate("abcdefghijklmnopərstuvwxyz ")}
    e.model_sha256, e.config_sha256 = "m" * 64, "c" * 64
    e.add_voice("af_heart", np.arange(510 * 256, dtype=np.float32).reshape(510, 256) / 1e5)
    return e


def run(kk, eng, inp, out, *extra):
    from kokoro_rust_b200 import cli
    args = cli.build_parser().parse_args(["synth", str(inp), "--model-dir", "unused", "--out-dir", str(out), *extra])
    return cli.synth(args, engine=eng)


def wav_samples(path):
    with open(path, "rb") as f:
        b = f.read()
    assert b[:4] == b"RIFF" and b[8:12] == b"WAVE"
    return np.frombuffer(b[44:], "<i2")


def test_whole_file_in_order_and_resume(kk, tmp_path):
    lines = ["həlo wɜrld", "abc def", "xyzQ", "the end"]
    inp = tmp_path / "book.txt"
    inp.write_text("\n".join(lines) + "\n", encoding="utf-8")
    out = tmp_path / "out"
    eng = make_engine(kk)
    assert run(kk, eng, inp, out) == 0
    assert sum(eng.gpu.calls) == 4
    whole = wav_samples(out / "book.wav")
    state = out / ".kokoro" / "book"
    parts = [wav_samples(state / f"book_{i:05d}.wav") for i in range(1, 5)]
    assert np.array_equal(whole, np.concatenate(parts))
    sc = json.loads((state / "book_00003.json").read_text())
    assert sc["status"] == "ok" and sc["dropped_phoneme_chars"] == ["Q"] and sc["samples"] == 600 * (3 + 2)
    sha1 = kk.wav.sha256_hex((out / "book.wav").read_bytes())
    # everything resumes: no synthesis, the assembled file is kept
    eng.gpu.calls.clear()
    assert run(kk, eng, inp, out) == 0 and eng.gpu.calls == []
    assert kk.wav.sha256_hex((out / "book.wav").read_bytes()) == sha1
    # one edited line is the only one synthesized again
    lines[1] = "abc deff"
    inp.write_text("\n".join(lines) + "\n", encoding="utf-8")
    assert run(kk, eng, inp, out) == 0 and eng.gpu.calls == [1]
    assert kk.wav.sha256_hex((out / "book.wav").read_bytes()) != sha1
    # a damaged line WAV is detected by its hash and redone; a different seed redoes everything
    with open(state / "book_00004.wav", "r+b") as f:
        f.seek(100)
        f.write(b"\x00\x01")
    eng.gpu.calls.clear()
    assert run(kk, eng, inp, out) == 0 and eng.gpu.calls == [1]
    eng.gpu.calls.clear()
    assert run(kk, eng, inp, out, "--seed", "5") == 0 and sum(eng.gpu.calls) == 4


def test_blank_invalid_and_oversize_lines(kk, tmp_path):
    eng = make_engine(kk)
    inp = tmp_path / "b.txt"
    inp.write_text("abc\n\ndef\n", encoding="utf-8")
    assert run(kk, eng, inp, tmp_path / "o1") == 1
    assert not (tmp_path / "o1" / "b.wav").exists()
    sc = json.loads((tmp_path / "o1" / ".kokoro" / "b" / "b_00002.json").read_text())
    assert sc["status"] == "blank" and "blank line" in sc["error"]
    assert run(kk, eng, inp, tmp_path / "o2", "--blank-lines", "skip") == 0
    assert len(wav_samples(tmp_path / "o2" / "b.wav")) == 600 * 5 * 2
    inp.write_text("abc\nde\x07f\n" + "a" * 511 + "\n", encoding="utf-8")
    assert run(kk, eng, inp, tmp_path / "o3") == 1
    st = tmp_path / "o3" / ".kokoro" / "b"
    assert json.loads((st / "b_00002.json").read_text())["status"] == "invalid"
    assert json.loads((st / "b_00003.json").read_text())["status"] == "oversize"
    assert json.loads((st / "b_00001.json").read_text())["status"] == "ok"


def test_per_line_mode_and_manifest(kk, tmp_path):
    eng = make_engine(kk)
    inp = tmp_path / "p.txt"
    inp.write_bytes(b"\xef\xbb\xbfabc\r\nxyz\r\n")
    out = tmp_path / "o"
    assert run(kk, eng, inp, out, "--per-line", "--diagnostics", "--format", "float32") == 0
    assert (out / "p_00001.wav").exists() and (out / "p_00002.wav").exists() and not (out / "p.wav").exists()
    m = json.loads((out / "p.manifest.json").read_text())
    assert m["bom_stripped"] and m["crlf_lines"] == 2 and m["counts"] == {"done": 2, "resumed": 0, "failed": 0}
    assert [e["line"] for e in m["lines"]] == [1, 2] and m["config"]["format"] == "Float32"
    # a later run without --diagnostics marks the old manifest as out of date
    assert run(kk, eng, inp, out, "--per-line", "--format", "float32") == 0
    m = json.loads((out / "p.manifest.json").read_text())
    assert m["complete"] is False and "stale" in m


def test_input_rules(kk, tmp_path):
    from kokoro_rust_b200 import cli
    p = tmp_path / "bad.txt"
    p.write_bytes(b"ok\n\xff\xfe\n")
    with pytest.raises(cli.JobError, match="not valid UTF-8: line 2"):
        cli.read_input(str(p))
    assert cli.control_char("a\tb") is None and cli.control_char("ab\x1b") == (3, "\x1b")
    args = cli.build_parser().parse_args(["synth", str(p), "--model-dir", "x", "--input-format", "text"])
    with pytest.raises(cli.JobError, match="text frontend"):
        cli.synth(args)


@pytest.mark.gpu
def test_cli_end_to_end_on_gpu(kk, ckpt_path, tmp_path):
    """The whole pipeline on the GPU from a model directory in the reference's layout
    (kokoro-v1_0.pth, config.json with the phoneme vocabulary, voices/<name>.pt)."""
    import torch
    from collections import OrderedDict
    from kokoro_rust_b200 import cli, weights
    md = tmp_path / "model"
    os.makedirs(md / "voices")
    subs = OrderedDict()
    for name, arr in weights.load_safetensors(ckpt_path).items():
        sub, param = name.split(".", 1)
        subs.setdefault(sub, OrderedDict())[param] = torch.from_numpy(np.ascontiguousarray(arr, np.float32))
    torch.save(subs, str(md / "kokoro-v1_0.pth"))
    vocab = {c: i + 1 for i, c in enumerate("abdefhijklmnopstuvwzðŋɑɔəɛɪʊʃʒθ ")}
    (md / "config.json").write_text(json.dumps({"vocab": vocab}), encoding="utf-8")
    torch.save(torch.randn(510, 1, 256, generator=torch.Generator().manual_seed(4)) * 0.1,
               str(md / "voices" / "af_heart.pt"))
    inp = tmp_path / "lines.txt"
    inp.write_text("həloʊ wɜld\nðɪs ɪz ə tɛst\nbaɪ\n", encoding="utf-8")
    out = tmp_path / "out"
    args = cli.build_parser().parse_args(["synth", str(inp), "--model-dir", str(md), "--out-dir", str(out),
                                          "--diagnostics"])
    assert cli.synth(args) == 0
    m = json.loads((out / "lines.manifest.json").read_text())
    assert m["counts"] == {"done": 3, "resumed": 0, "failed": 0} and m["output"]["lines"] == 3
    total = sum(json.loads((out / ".kokoro" / "lines" / f"lines_{i:05d}.json").read_text())["samples"]
                for i in (1, 2, 3))
    assert m["output"]["samples"] == total > 0
    assert cli.synth(args) == 0  # second run: everything resumed
    assert json.loads((out / "lines.manifest.json").read_text())["counts"]["resumed"] == 3


def test_job_level_errors_exit_2(kk, tmp_path):
    """Failures outside a line (unreadable input, a model directory without a checkpoint) end the
    job with status 2."""
    from kokoro_rust_b200 import cli
    assert cli.main(["synth", str(tmp_path / "missing.txt"), "--model-dir", str(tmp_path)]) == 2
    inp = tmp_path / "l.txt"
    inp.write_text("abc\n", encoding="utf-8")
    assert cli.main(["synth", str(inp), "--model-dir", str(tmp_path), "--out-dir", str(tmp_path / "o")]) == 2
