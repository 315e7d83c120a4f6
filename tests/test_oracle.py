"""The CPU oracle against independent formulations and published known answers."""
import numpy as np
import pytest
import torch


def test_splitmix64_published_sequence(oracle_mod):
    """splitmix64 (Vigna) from state 0: e220a8397b1dcdaf 6e789e6aa1b965f4 06c45d188009454f
    f88bb8a8724c81ec; splitmix_at(seed, i) is output i of the stream (src/vocoder.rs:22-27)."""
    got = [int(x) for x in oracle_mod.splitmix_at(0, np.arange(4, dtype=np.uint64))]
    assert got == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F, 0xF88BB8A8724C81EC]


def test_mix_seed_engine_and_oracle_agree(kk, oracle_mod):
    for s, i in ((0, 0), (42, 7), (2**64 - 1, 123456), (7, 2**40)):
        assert kk.mix_seed(s, i) == oracle_mod.mix_seed(s, i)


def test_counter_noise_is_standard_normal(oracle_mod):
    n = oracle_mod.counter_noise(3, 200_001)
    assert n.shape == (200_001,) and n.dtype == np.float32
    assert abs(float(n.mean())) < 0.01 and abs(float(n.std()) - 1.0) < 0.01
    assert np.array_equal(n[:1000], oracle_mod.counter_noise(3, 1000))
    assert not np.array_equal(n[:1000], oracle_mod.counter_noise(4, 1000))


def test_durations_round_half_even_and_clamp(oracle_mod):
    # logits whose sigmoid sum is exactly representable: sigma(0) = 0.5
    def row(k):  # k entries at 0 (0.5 each), rest at -inf-ish
        r = np.full(50, -100.0, np.float32)
        r[:k] = 0.0
        return r
    logits = np.stack([row(5), row(7), row(1), row(0), row(9)])  # sums 2.5, 3.5, 0.5, ~0, 4.5
    d, q = oracle_mod.durations_from_logits(logits, 1.0)
    assert list(d) == [2, 4, 1, 1, 4]  # ties to even; clamp >= 1
    d2, _ = oracle_mod.durations_from_logits(logits, 0.5)  # speed divides
    assert list(d2) == [5, 7, 1, 1, 9]


def test_stft_matches_numpy_rfft(oracle_mod):
    """torch.stft(n_fft 20, hop 5, periodic Hann, centre, reflect) magnitude and phase."""
    rng = np.random.default_rng(0)
    x = np.tanh(rng.standard_normal(600)).astype(np.float32)
    spec = oracle_mod.stft20(x)
    assert spec.shape == (22, 1 + 600 // 5)
    xp = np.pad(x.astype(np.float64), 10, mode="reflect")
    w = 0.5 - 0.5 * np.cos(2 * np.pi * np.arange(20) / 20)
    fr = np.stack([xp[5 * f:5 * f + 20] * w for f in range(spec.shape[1])])
    X = np.fft.rfft(fr, axis=1)
    assert np.abs(spec[:11].T - np.abs(X)).max() < 1e-5
    m = np.abs(X) > 1e-3  # phase where it is defined
    dph = np.angle(np.exp(1j * (spec[11:].T - np.angle(X))))
    assert np.abs(dph[m]).max() < 1e-4


def test_istft_matches_torch_istft(oracle_mod):
    rng = np.random.default_rng(1)
    F = 41
    post = rng.standard_normal((22, F)).astype(np.float32) * 0.5
    ours = oracle_mod.istft20(post)
    mag = np.exp(post[:11].astype(np.float64))
    ph = np.sin(post[11:].astype(np.float64))
    X = torch.from_numpy(mag * np.exp(1j * ph))
    ref = torch.istft(X, n_fft=20, hop_length=5, win_length=20,
                      window=torch.hann_window(20, periodic=True, dtype=torch.float64), center=True).numpy()
    assert ours.shape == ref.shape == (5 * (F - 1),)
    assert np.abs(ours - ref).max() < 1e-5


def test_frames_to_samples_known_answer(oracle_mod):
    """130 frames -> 78,000 samples: iSTFT over 120 * 130 + 1 frames at hop 5."""
    post = np.zeros((22, 120 * 130 + 1), np.float32)
    assert oracle_mod.istft20(post).shape == (78_000,)


def test_sinegen_unvoiced_and_rand_ini_dead(oracle_mod):
    L = 8
    lw = np.linspace(-1, 1, 9).astype(np.float32)
    f0 = np.zeros(L, np.float32)  # unvoiced everywhere, zero noise -> tanh(lb)
    har = oracle_mod.sinegen_har(f0, np.zeros(300 * L * 9, np.float32), lw, 0.25)
    assert np.allclose(har, np.tanh(np.float32(0.25)))
    f0v = np.full(L, 220.0, np.float32)  # voiced: bounded, periodic-ish, not constant
    har = oracle_mod.sinegen_har(f0v, np.zeros(300 * L * 9, np.float32), lw, 0.0)
    assert np.abs(har).max() < 1 and har.std() > 0.01


def test_oracle_decode_shapes_and_determinism(oracle, oracle_mod):
    rng = np.random.default_rng(5)
    N = 6
    asr = torch.from_numpy(rng.standard_normal((512, N)).astype(np.float32))
    f0 = np.exp(rng.uniform(np.log(80), np.log(400), 2 * N)).astype(np.float32)
    n = rng.standard_normal(2 * N).astype(np.float32)
    s = torch.from_numpy((rng.standard_normal(128) * 0.1).astype(np.float32))
    noise = oracle_mod.counter_noise(1, 600 * N * 9)
    a = oracle.decode(asr, f0, n, s, noise)
    b = oracle.decode(asr, f0, n, s, noise)
    assert a.shape == (600 * N,) and np.array_equal(a, b) and np.isfinite(a).all()
