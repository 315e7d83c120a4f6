"""Shared fixtures: the package (directory ``kokoro-rust_b200``), the CPU oracle (test
infrastructure), a seeded random-init checkpoint and the ``gpu`` marker."""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "kokoro-rust_b200")


def import_package():
    if "kokoro_rust_b200" in sys.modules:
        return sys.modules["kokoro_rust_b200"]
    spec = importlib.util.spec_from_file_location("kokoro_rust_b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["kokoro_rust_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def import_oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import kokoro_oracle  # noqa: E402

    return kokoro_oracle


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def kk():
    return import_package()


@pytest.fixture(scope="session")
def oracle_mod():
    return import_oracle()


@pytest.fixture(scope="session")
def ckpt_path(tmp_path_factory, kk):
    from kokoro_rust_b200 import weights

    p = str(tmp_path_factory.mktemp("ckpt") / "kokoro_seed0.safetensors")
    return weights.write_random_checkpoint(p, seed=0)


@pytest.fixture(scope="session")
def state_dict(ckpt_path):
    from kokoro_rust_b200 import weights

    return weights.load_safetensors(ckpt_path)


@pytest.fixture(scope="session")
def oracle(state_dict, oracle_mod):
    return oracle_mod.KokoroOracle(state_dict, threads=min(8, os.cpu_count() or 1))


@pytest.fixture(scope="session")
def bench_mod():
    """bench.py's workload definitions (config 2's input distributions)."""
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import bench  # noqa: E402

    return bench


def spec_mean_abs_db(a, b, n=1024, hop=256):
    """G-SPEC (reference tests/common_gates.rs:12-49): periodic Hann 1024, hop 256, frames fully
    inside, 20 log10(max(|X|, 1e-5)), mean |dB_a - dB_b|."""
    w = 0.5 - 0.5 * np.cos(2 * np.pi * np.arange(n) / n)
    frames = 1 + (len(a) - n) // hop
    fa = np.stack([np.fft.rfft(a[f * hop:f * hop + n].astype(np.float64) * w) for f in range(frames)])
    fb = np.stack([np.fft.rfft(b[f * hop:f * hop + n].astype(np.float64) * w) for f in range(frames)])
    da = 20 * np.log10(np.maximum(np.abs(fa), 1e-5))
    db = 20 * np.log10(np.maximum(np.abs(fb), 1e-5))
    return float(np.abs(da - db).mean())


@pytest.fixture(scope="session")
def spec_db():
    return spec_mean_abs_db


def config1():
    """64 ids uniform in [1, 177] from numpy's default_rng(0) framed by pad 0, the
    256-d style N(0, 0.1^2) from the same generator after the ids, durations forced to [0, 3 x 64, 0]
    (192 frames, 115,200 samples)."""
    rng = np.random.default_rng(0)
    ids = np.concatenate([[0], rng.integers(1, 178, 64), [0]]).astype(np.int64)
    ref_s = (rng.standard_normal(256) * 0.1).astype(np.float32)
    dur = np.array([0] + [3] * 64 + [0], np.int64)
    return ids, ref_s, dur


@pytest.fixture(scope="session")
def gspec(oracle_mod, state_dict):
    """The reference's G-SPEC gate (tests/common_gates.rs:1-10): a full-forward waveform passes at a
    mean |dB| distance of at most twice the floor pair's, the floor pair being two runs of the same
    CPU implementation that differ only in thread count (1 and 8) on one fixed floor case. The
    floor case here is BASELINE config 1 (counter noise seed 0). Returns {"floor": dB, "gate": dB,
    "config1": the 8-thread oracle's config-1 output (audio, durations, F0 / N, t_en / asr)}."""
    import torch
    threads = min(8, os.cpu_count() or 1)
    ids, ref_s, dur = config1()
    outs = [oracle_mod.KokoroOracle(state_dict, threads=th).forward(ids, ref_s, 1.0, seed=0, forced_dur=dur,
                                                                    want=("f0", "asr"))
            for th in (1, threads)]
    torch.set_num_threads(threads)
    floor = spec_mean_abs_db(outs[0]["audio"], outs[1]["audio"])
    return {"floor": floor, "gate": 2.0 * floor, "config1": outs[1]}


def synth_item(rng, n_tokens, style_sd=0.1):
    """Token ids uniform in [1, 177] framed by pad 0, style ~ N(0, 0.1^2)."""
    ids = np.concatenate([[0], rng.integers(1, 178, n_tokens), [0]]).astype(np.int64)
    ref_s = (rng.standard_normal(256) * style_sd).astype(np.float32)
    return ids, ref_s
