"""bench.py's reference arm (`--impl reference`), the line that times the CPU restatement for the
driver: its JSON keys and values follow the bench contract, the timed CPU work is `steps` samples
after at least three warm-up samples, and ranks other than 0 print nothing and do no work. The
oracle timing is replaced by a stand-in here (the real one takes minutes of CPU); the GPU box runs
the real one."""
import contextlib
import importlib.util
import io
import json
import os
import sys
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("kk_bench_ref_arm", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _run(monkeypatch, argv, env=None):
    b = _bench()
    calls = []

    def fake_time_oracle(ckpt, lines, style, threads):
        calls.append((len(lines), threads))
        return 2.5, 0.5  # 2.5 audio-s in 0.5 wall-s

    stub = types.SimpleNamespace(weights=types.SimpleNamespace(write_random_checkpoint=lambda path, seed: None))
    monkeypatch.setattr(b, "time_oracle", fake_time_oracle)
    monkeypatch.setattr(b, "import_package", lambda: stub)
    monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
    monkeypatch.setenv("KK_FETCH_THREADS", "4")
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE"):
        monkeypatch.delenv(k, raising=False)
    for k, v in (env or {}).items():
        monkeypatch.setenv(k, v)
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        b.main()
    return out.getvalue(), calls


def test_reference_arm_line_follows_the_contract(monkeypatch):
    text, calls = _run(monkeypatch, ["--impl", "reference", "--steps", "2", "--warmup", "1"])
    lines = [l for l in text.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    # warm-up is raised to 3; every sample is one median-length line on all host threads
    assert calls == [(1, os.cpu_count() or 1)] * (3 + 2)
    assert d["impl"] == "reference"
    assert d["metric"] == "audio-sec per wall-sec (full ragged forward)"  # the GPU arm's config-4 metric
    assert d["unit"] == "audio-s/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert abs(d["value"] - 5.0) < 1e-12  # 2 x 2.5 audio-s in 2 x 0.5 s
    assert abs(d["ms_per_step"] - 500.0) < 1e-9
    assert d["scaling"] == "weak" and d["vs_baseline"] is None and d["data"] == "synthetic"
    assert isinstance(d["config"]["workload"], str) and d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] == (os.cpu_count() or 1)
    assert cb["unit"] == d["unit"] and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing(monkeypatch):
    text, calls = _run(monkeypatch, ["--impl", "reference", "--gpus", "2", "--steps", "1"],
                       {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1", "LOCAL_WORLD_SIZE": "2"})
    assert text.strip() == "" and calls == []
