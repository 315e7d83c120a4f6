"""Parity on BASELINE's own configurations, against the CPU oracle through the C ABI.

* Config 1 exactly (fp32): 64 ids uniform in [1, 177] from ``numpy.random.default_rng(0)`` framed by
  pad 0, style N(0, 0.1^2) from the same generator (drawn after the ids), speed 1, durations forced
  to ``[0, 3 x 64, 0]`` (192 frames, 115,200 samples), counter noise seed 0.
  - vocoder: the oracle's own asr / F0 / N through ``kk_decode_batch``, waveform max-abs <= 1e-3;
  - full forward: F0 / N curves within 1e-4 relative L2, the text encoder output ``t_en`` and its
    frame alignment ``asr`` within 1e-4 relative L2 (the reference's ``text_encoder_b``,
    src/gpu_batch.rs:457-481), waveform under the reference's G-SPEC gate: at most twice the
    spectral distance between two oracle runs on this case that differ only in thread count (the
    gate's floor pair, tests/common_gates.rs:1-10; config 1 is the floor case). The waveform itself
    drifts in phase: an F0 that differs in the sixth digit (accumulation order) moves the phase of
    near-zero STFT bins across +-pi, which the noise convolutions consume; the oracle against
    itself at 1 and 8 threads shows the same;
  - BF16 mode: ``t_en`` / ``asr`` within 2e-2 relative L2 (bf16 conv operands, fp32 LayerNorm,
    the split-operand LSTM recurrence).
* Config 2's shape: 4 items of T = 400 frames with config 2's input distributions (the bench's
  ``config2_inputs``): fp32 max-abs <= 1e-3, BF16 SNR >= 40 dB (each item's margin printed).
* Durations of a 510-token item (the longest the reference accepts), fp32, bit-exact outside
  round-half-even ties closer than 1e-4.
"""
import os
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3


from conftest import config1


@pytest.fixture(scope="module")
def c1_ref(gspec):
    return gspec["config1"]


@pytest.fixture(scope="module")
def eng32(kk, ckpt_path):
    e = kk.GpuKokoro(ckpt_path, 0, "fp32")
    yield e
    e.close()


@pytest.fixture(scope="module")
def eng16(kk, ckpt_path):
    e = kk.GpuKokoro(ckpt_path, 0, "bf16")
    yield e
    e.close()


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(np.asarray(b, np.float64)))


def forward_dumps(kk, eng, ids, ref_s, dur):
    """Forced-duration forward of one item with the engine's stage dumps (KK_DEBUG_DUMP_DIR)."""
    d = tempfile.mkdtemp()
    os.environ["KK_DEBUG_DUMP_DIR"] = d
    try:
        out = eng.forward_batch([kk.BatchItem(ids, ref_s, 1.0, kk.ItemNoise(seed=0))], forced_dur=[dur])[0]
    finally:
        del os.environ["KK_DEBUG_DUMP_DIR"]

    def load(name):
        rows, cols, ld = (int(v) for v in open(os.path.join(d, name + ".shape")).read().split())
        return np.fromfile(os.path.join(d, name + ".f32"), np.float32).reshape(rows, ld)[:, :cols]
    return out, load


def test_config1_vocoder_fp32(eng32, c1_ref):
    ids, ref_s, dur = config1()
    asr = c1_ref["asr"].T  # [N, 512] time-major
    a = eng32.decode_batch([asr], [c1_ref["f0"]], [c1_ref["n"]], ref_s[None, :128], seeds=[0])[0]
    r = c1_ref["audio"]
    err = float(np.abs(a - r).max())
    print(f"config 1 vocoder: {a.shape[0]} samples, max-abs {err:.3g}")
    assert a.shape == r.shape == (115_200,)
    assert err <= FP32_TOL


def test_config1_forward_fp32(kk, eng32, c1_ref, gspec, spec_db):
    ids, ref_s, dur = config1()
    out, load = forward_dumps(kk, eng32, ids, ref_s, dur)
    assert out.audio.shape == (115_200,) and np.array_equal(out.pred_dur, dur)
    N, T = int(dur.sum()), len(ids)
    e_f0 = rel_l2(load("f0").reshape(-1)[:2 * N], c1_ref["f0"])
    e_n = rel_l2(load("nc").reshape(-1)[:2 * N], c1_ref["n"])
    e_ten = rel_l2(load("t_en")[:T], c1_ref["t_en"])
    e_asr = rel_l2(load("xcat0")[:N, :512], c1_ref["asr"].T)
    d = spec_db(out.audio, c1_ref["audio"])
    print(f"config 1 forward fp32: F0 {e_f0:.3g} N {e_n:.3g} t_en {e_ten:.3g} asr {e_asr:.3g} (rel-L2), "
          f"spectral {d:.3f} dB (G-SPEC floor pair {gspec['floor']:.3f} dB, gate {gspec['gate']:.3f} dB), "
          f"max-abs {np.abs(out.audio - c1_ref['audio']).max():.3g}")
    assert e_f0 <= 1e-4 and e_n <= 1e-4
    assert e_ten <= 1e-4 and e_asr <= 1e-4
    assert d <= gspec["gate"]


def test_config1_text_encoder_bf16(kk, eng16, c1_ref):
    ids, ref_s, dur = config1()
    out, load = forward_dumps(kk, eng16, ids, ref_s, dur)
    N, T = int(dur.sum()), len(ids)
    e_ten = rel_l2(load("t_en")[:T], c1_ref["t_en"])
    e_asr = rel_l2(load("xcat0")[:N, :512], c1_ref["asr"].T)
    print(f"config 1 text encoder bf16: t_en {e_ten:.3g} asr {e_asr:.3g} (rel-L2)")
    assert out.audio.shape == (115_200,) and np.isfinite(out.audio).all()
    assert e_ten <= 2e-2 and e_asr <= 2e-2


@pytest.fixture(scope="module")
def c2_case(oracle, oracle_mod, bench_mod):
    """Four items of config 2's shape (T = 400 frames), with the oracle's waveforms."""
    import torch
    asr, f0s, ns, s_dec = bench_mod.config2_inputs(seed=2000, B=4, T=400)
    seeds = [21, 22, 23, 24]
    refs = [oracle.decode(torch.from_numpy(a.T.copy()), f, n, torch.from_numpy(s), oracle_mod.counter_noise(sd, 600 * 400 * 9))
            for a, f, n, s, sd in zip(asr, f0s, ns, s_dec, seeds)]
    return asr, f0s, ns, s_dec, seeds, refs


def test_config2_shape_fp32(eng32, c2_case):
    asr, f0s, ns, s_dec, seeds, refs = c2_case
    outs = eng32.decode_batch(asr, f0s, ns, s_dec, seeds=seeds)
    for i, (a, r) in enumerate(zip(outs, refs)):
        err = float(np.abs(a - r).max())
        print(f"config 2 item {i}: {a.shape[0]} samples, fp32 max-abs {err:.3g}")
        assert a.shape == r.shape == (240_000,)
        assert err <= FP32_TOL


def test_config2_shape_bf16_snr(eng16, c2_case):
    asr, f0s, ns, s_dec, seeds, refs = c2_case
    outs = eng16.decode_batch(asr, f0s, ns, s_dec, seeds=seeds)
    for i, (a, r) in enumerate(zip(outs, refs)):
        snr = float(10 * np.log10((r.astype(np.float64) ** 2).sum() / ((a - r).astype(np.float64) ** 2).sum()))
        print(f"config 2 item {i}: bf16 SNR {snr:.2f} dB (margin {snr - 40.0:.2f} dB over 40 dB)")
        assert a.shape == r.shape and snr >= 40.0


def test_durations_510_tokens_fp32(kk, eng32, oracle):
    rng = np.random.default_rng(510)
    ids = np.concatenate([[0], rng.integers(1, 178, 510), [0]]).astype(np.int64)
    ref_s = (rng.standard_normal(256) * 0.1).astype(np.float32)
    dur, q = oracle.durations(ids, ref_s, 1.0)
    out = eng32.forward_batch([kk.BatchItem(ids, ref_s, 1.0, kk.ItemNoise(seed=1))])[0]
    tie = np.abs(q - np.floor(q) - 0.5) < 1e-4
    print(f"512 ids: {int(dur.sum())} frames, {int(tie.sum())} ties exempt, "
          f"{int((out.pred_dur != dur).sum())} differences")
    assert out.pred_dur.shape == dur.shape
    assert np.array_equal(out.pred_dur[~tie], dur[~tie])
    assert out.audio.shape == (600 * int(out.pred_dur.sum()),)
