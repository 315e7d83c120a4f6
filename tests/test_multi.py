"""One engine process per GPU behind the Engine interface (multi.MultiEngine), on the host with
stand-in engines (tests/multi_standin.py): requests spread over the workers by LPT come back in
request order and equal to a single engine's results, per-request errors keep their place, a
worker that exits fails only the requests it held, and the synth pipeline over two workers writes
the same WAV as over one engine."""
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
STANDIN = os.path.join(HERE, "multi_standin.py")


def _standin():
    import importlib.util
    spec = importlib.util.spec_from_file_location("kk_standin_local", STANDIN)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _reqs(n, seed=0):
    rng = np.random.default_rng(seed)
    alphabet = list("abcdefghijklmnopərstuvwxyz ")
    out = []
    for i in range(n):
        m = int(rng.integers(1, 300))
        out.append(("".join(rng.choice(alphabet, m)), 1000 + i))
    return out


def test_spread_in_order_and_equal_to_one_engine(kk):
    from kokoro_rust_b200.multi import MultiEngine
    reqs = _reqs(24)
    reqs[5] = ("", 5)                   # empty: a per-request validation error
    reqs[11] = ("a" * 600, 11)          # oversize
    one = _standin().make_engine(kk, 0)
    ref = one.synth_batch(reqs, "af_heart", 1.0, kk.BatchPolicy(max_phonemes=900, max_items=8))
    with MultiEngine("/nonexistent.safetensors", [0, 1], standin=STANDIN) as m:
        assert m.identity() == "fake" and m.model_sha256 == "m" * 64
        got = m.synth_batch(reqs, "af_heart", 1.0, kk.BatchPolicy(max_phonemes=900, max_items=8))
        assert m.voice("af_heart").pack.shape == (510, 256)
    assert len(got) == len(reqs)
    devices = set()
    for r, g in zip(ref, got):
        if isinstance(r, Exception):
            assert isinstance(g, Exception) and type(r).__name__ in str(g)
        else:
            assert np.array_equal(r.audio, g.audio) and r.dropped == g.dropped
            devices.add(int(g.pred_dur[0]))
    assert devices == {0, 1}            # both workers took requests


def test_lost_worker_fails_only_its_requests(kk):
    from kokoro_rust_b200.multi import MultiEngine
    from kokoro_rust_b200.shard import LineError
    with MultiEngine("/nonexistent.safetensors", [0, 1], standin=STANDIN) as m:
        reqs = [("abc!", 1), ("abcdef", 2), ("de", 3), ("xyz", 4)]   # '!' ends its worker
        got = m.synth_batch(reqs, "af_heart", 1.0)
        lost = [i for i, g in enumerate(got) if isinstance(g, LineError)]
        assert 0 in lost and len(lost) < len(reqs)
        assert all(not isinstance(g, Exception) for i, g in enumerate(got) if i not in lost)
        assert len(m.live()) == 1
        # the next call runs everything on the remaining worker
        got = m.synth_batch([("abc", 1), ("defg", 2)], "af_heart", 1.0)
        assert all(not isinstance(g, Exception) for g in got)
        m.synth_batch([("q!", 1)], "af_heart", 1.0)
        assert m.live() == []
        with pytest.raises(RuntimeError, match="no GPU worker left"):
            m.synth_batch([("abc", 1)], "af_heart", 1.0)


def test_worker_that_cannot_start_is_reported(kk, tmp_path):
    from kokoro_rust_b200.multi import MultiEngine
    bad = tmp_path / "bad_standin.py"
    bad.write_text("def make_engine(kk, device):\n    raise RuntimeError('no device ' + str(device))\n")
    with pytest.raises(RuntimeError, match="no device 1"):
        MultiEngine("/nonexistent.safetensors", [0, 1], standin=str(bad))


def test_worker_that_never_answers_is_ended(kk, tmp_path):
    from kokoro_rust_b200.multi import MultiEngine
    slow = tmp_path / "slow_standin.py"
    slow.write_text("import time\ndef make_engine(kk, device):\n    time.sleep(3600)\n")
    with pytest.raises(RuntimeError, match="did not answer within 2 s"):
        MultiEngine("/nonexistent.safetensors", [0], standin=str(slow), start_timeout=2.0)


def test_synth_pipeline_over_two_workers_matches_one_engine(kk, tmp_path):
    from kokoro_rust_b200 import cli
    from kokoro_rust_b200.multi import MultiEngine
    lines = [r[0] for r in _reqs(40, seed=3)]
    inp = tmp_path / "book.txt"
    inp.write_text("\n".join(lines) + "\n", encoding="utf-8")

    def run(engine, out):
        args = cli.build_parser().parse_args(["synth", str(inp), "--model-dir", "unused", "--out-dir", str(out),
                                              "--batch-window", "16"])
        return cli.synth(args, engine=engine)

    assert run(_standin().make_engine(kk, 0), tmp_path / "one") == 0
    with MultiEngine("/nonexistent.safetensors", [0, 1], standin=STANDIN) as m:
        assert run(m, tmp_path / "two") == 0
    a = (tmp_path / "one" / "book.wav").read_bytes()
    b = (tmp_path / "two" / "book.wav").read_bytes()
    assert a == b
