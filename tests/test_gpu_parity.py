"""CUDA engine vs the CPU oracle through the C ABI (fp32 path, small cases; BASELINE's own
configurations are in test_gpu_configs.py, batch semantics in test_gpu_batching.py).

* vocoder comparison (decoder + generator on identical asr / F0 / N / style / noise inputs):
  waveform max-abs <= 1e-3;
* replayed noise equals the counter stream it was drawn from;
* full forward with forced durations: the waveform is compared spectrally under the reference's
  G-SPEC gate (tests/common_gates.rs: at most twice the distance of the floor pair, the oracle at 1
  and at 8 threads on the floor case, config 1): the harmonic source integrates F0 over every
  sample, so an F0 that differs by fp32 accumulation order (~1e-6 relative) moves phases of
  near-zero STFT bins across the +-pi branch cut, for the oracle against itself as much as for the
  engine;
* predicted integer durations bit-exact outside round-half-even ties closer than 1e-4;
* memory statistics of a forward and the free-VRAM batch budget built from them.
"""
import numpy as np
import pytest

from conftest import spec_mean_abs_db, synth_item

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3


@pytest.fixture(scope="module")
def eng32(kk, ckpt_path):
    e = kk.GpuKokoro(ckpt_path, 0, "fp32")
    yield e
    e.close()


def vocoder_inputs(rng, n_frames):
    """Config-2 style inputs: asr N(0,1), F0 log-uniform 80-400 Hz with a zeroed (unvoiced) run,
    N N(0,1), style N(0, 0.1^2)."""
    asr = rng.standard_normal((n_frames, 512)).astype(np.float32)
    f0 = np.exp(rng.uniform(np.log(80), np.log(400), 2 * n_frames)).astype(np.float32)
    run = max(1, (2 * n_frames) // 5)
    s = rng.integers(0, 2 * n_frames - run + 1)
    f0[s:s + run] = 0.0
    n = rng.standard_normal(2 * n_frames).astype(np.float32)
    s_dec = (rng.standard_normal(128) * 0.1).astype(np.float32)
    return asr, f0, n, s_dec


def test_decode_matches_oracle(kk, eng32, oracle, oracle_mod):
    import torch
    rng = np.random.default_rng(3)
    frames = [23, 9]
    inp = [vocoder_inputs(rng, n) for n in frames]
    seeds = [11, 12]
    outs = eng32.decode_batch([x[0] for x in inp], [x[1] for x in inp], [x[2] for x in inp],
                              np.stack([x[3] for x in inp]), seeds=seeds)
    for (asr, f0, n, s_dec), seed, a in zip(inp, seeds, outs):
        noise = oracle_mod.counter_noise(seed, 600 * asr.shape[0] * 9)
        r = oracle.decode(torch.from_numpy(asr.T.copy()), f0, n, torch.from_numpy(s_dec), noise)
        err = np.abs(a - r).max()
        print("decode max-abs", err, "ref rms", np.sqrt((r ** 2).mean()))
        assert a.shape == r.shape
        assert err <= FP32_TOL


def test_decode_replayed_noise_matches_counter(kk, eng32, oracle_mod):
    rng = np.random.default_rng(4)
    asr, f0, n, s_dec = vocoder_inputs(rng, 7)
    a = eng32.decode_batch([asr], [f0], [n], s_dec[None], seeds=[5])[0]
    noise = oracle_mod.counter_noise(5, 600 * 7 * 9)
    b = eng32.decode_batch([asr], [f0], [n], s_dec[None], noise=[noise])[0]
    assert np.abs(a - b).max() <= 1e-5


def test_forward_forced_durations(kk, eng32, oracle, gspec):
    rng = np.random.default_rng(1)
    ids, ref_s = synth_item(rng, 12)
    dur = np.concatenate([[0], np.full(12, 3), [0]])
    outs = eng32.forward_batch([kk.BatchItem(ids, ref_s, 1.0, kk.ItemNoise(seed=7))], forced_dur=[dur])
    ref = oracle.forward(ids, ref_s, 1.0, seed=7, forced_dur=dur)
    a, r = outs[0].audio, ref["audio"]
    assert a.shape == r.shape == (600 * 36,)
    assert np.array_equal(outs[0].pred_dur, dur)
    d = spec_mean_abs_db(a, r)
    print(f"forced forward: spectral {d:.3f} dB (G-SPEC gate {gspec['gate']:.3f} dB), max-abs {np.abs(a - r).max():.3g}")
    assert d <= gspec["gate"]


def test_predicted_durations_bit_exact(kk, eng32, oracle):
    rng = np.random.default_rng(2)
    items, refs = [], []
    for n in (9, 17, 5):
        ids, ref_s = synth_item(rng, n)
        items.append(kk.BatchItem(ids, ref_s, 1.0, kk.ItemNoise(seed=n)))
        refs.append(oracle.forward(ids, ref_s, 1.0, seed=n, want=("dur_q",)))
    outs = eng32.forward_batch(items)
    for o, r in zip(outs, refs):
        margin = np.abs(r["dur_q"] - np.floor(r["dur_q"]) - 0.5)
        tie = margin < 1e-4
        assert np.array_equal(o.pred_dur[~tie], r["dur"][~tie]), (o.pred_dur, r["dur"])


def test_memory_stats_and_free_vram_budget(kk, eng32):
    """kk_memory_stats after a forward: the call's token and frame totals, a peak working set
    within the arena, and a free-VRAM policy built from them."""
    rng = np.random.default_rng(5)
    items, durs = [], []
    for n in (7, 20):
        ids, ref_s = synth_item(rng, n)
        items.append(kk.BatchItem(ids, ref_s, 1.0, kk.ItemNoise(seed=n)))
        durs.append(np.concatenate([[0], np.full(n, 2), [0]]))
    eng32.forward_batch(items, forced_dur=durs)
    st = eng32.memory_stats()
    assert st["tokens"] == sum(len(it.ids) for it in items)
    assert st["frames"] == sum(int(d.sum()) for d in durs)
    assert 0 < st["peak_bytes"] <= st["arena_bytes"]
    free, total = eng32.device_memory()
    assert 0 < free <= total
    p = kk.BatchPolicy.from_free_vram(eng32)
    assert p.max_phonemes >= kk.engine.MAX_PHONEMES + 2
