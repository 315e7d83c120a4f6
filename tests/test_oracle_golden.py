"""The CPU oracle against golden vectors produced by the REFERENCE's own CUDA kernels
(kernels/kokoro.cu compiled from source for sm_100a by oracle/build_ref.py and run on a B200 by
tests/golden/make_ref_golden.py). This pins the oracle's arithmetic to the reference's.

Tolerances: the oracle evaluates transcendentals correctly rounded (via f64) where the reference
calls CUDA's sinf / tanhf / logf, so values agree to a few ulp; the phase_pre cumulative sum (the
bit-exactness-critical path) and the frame arithmetic are compared exactly."""
import os

import numpy as np
import pytest
import torch

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_kernels.npz"))


def test_counter_noise_matches_reference_gen_noise(oracle_mod):
    n = oracle_mod.counter_noise(int(G["src_seed"][0]), G["src_noise"].shape[0])
    assert np.abs(n - G["src_noise"]).max() <= 2e-6 * max(1.0, float(np.abs(G["src_noise"]).max()))


def test_sine_phase_pre_bit_exact(oracle_mod):
    pp = oracle_mod.sine_phase_pre(G["src_f0"])
    assert pp.shape == G["src_pp"].shape
    assert np.array_equal(pp, G["src_pp"])


def test_har_source_matches_reference(oracle_mod):
    har = oracle_mod.har_from_phase(G["src_f0"], G["src_pp"], G["src_noise"], G["src_lw"], float(G["src_lb"][0]))
    assert np.abs(har - G["src_har"]).max() <= 2e-6


def test_stft_matches_reference(oracle_mod):
    spec = oracle_mod.stft20(G["src_har"])
    ref = G["src_spec"]
    assert spec.shape == ref.shape
    mag, rmag = spec[:11], ref[:11]
    assert np.abs(mag - rmag).max() <= 1e-6 * max(1.0, float(rmag.max()))
    ok = rmag > 1e-4 * float(rmag.max())
    dph = np.angle(np.exp(1j * (spec[11:].astype(np.float64) - ref[11:])))
    assert np.abs(dph[ok]).max() <= 1e-5


def test_istft_matches_reference(oracle_mod):
    a = oracle_mod.istft20(G["istft_post"])
    assert a.shape == G["istft_audio"].shape
    assert np.abs(a - G["istft_audio"]).max() <= 1e-5 * max(1.0, float(np.abs(G["istft_audio"]).max()))


def test_adain_stats_and_apply_match_reference(oracle_mod):
    x = G["adain_x"]
    C = x.shape[0]
    y_ref = G["adain_y"]
    for b, (s, n) in enumerate(zip(G["adain_starts"], G["adain_lens"])):
        seg = x[:, s:s + n]
        mean, rstd = oracle_mod.chan_stats(seg)
        assert np.abs(mean - G["adain_mean"][b]).max() <= 1e-6 * max(1.0, float(np.abs(mean).max()))
        assert np.abs(rstd - G["adain_rstd"][b]).max() <= 1e-5 * float(np.abs(rstd).max())
        gb = G["adain_gb"][b]
        y = oracle_mod.adain_apply(seg, mean, rstd, G["adain_nw"], G["adain_nb"], gb[:C], gb[C:], 0.2)
        assert np.abs(y - y_ref[:, s:s + n]).max() <= 1e-5
    gaps = np.ones(x.shape[1], bool)
    for s, n in zip(G["adain_starts"], G["adain_lens"]):
        gaps[s:s + n] = False
    assert np.all(y_ref[:, gaps] == 0)  # gap columns zeroed


def test_lstm_matches_reference(oracle_mod):
    out = G["lstm_out"]
    H = G["lstm_whf"].shape[1]
    for s, n in zip(G["lstm_starts"], G["lstm_lens"]):
        for d, (gx, whh, bhh) in enumerate(((G["lstm_gxf"], G["lstm_whf"], G["lstm_bhf"]),
                                            (G["lstm_gxb"], G["lstm_whb"], G["lstm_bhb"]))):
            h = oracle_mod.lstm_dir(torch.from_numpy(gx[s:s + n]), torch.from_numpy(whh), torch.from_numpy(bhh), d == 1)
            assert np.abs(h.numpy() - out[s:s + n, d * H:(d + 1) * H]).max() <= 1e-5


def test_layernorm_gelu_softmax_match_reference(oracle_mod):
    y = oracle_mod.ln_rows(G["ln_x"], G["ln_g"], G["ln_b"], 1e-12)
    assert np.abs(y - G["ln_y"]).max() <= 2e-6 * max(1.0, float(np.abs(G["ln_y"]).max()))
    g = oracle_mod.gelu_new(torch.from_numpy(G["gelu_x"])).numpy()
    assert np.abs(g - G["gelu_y"]).max() <= 2e-6 * max(1.0, float(np.abs(G["gelu_y"]).max()))
    s = torch.softmax(torch.from_numpy(G["softmax_x"]) * 0.125, -1).numpy()
    assert np.abs(s - G["softmax_y"]).max() <= 1e-6


def test_strided_and_transposed_convs_match_reference():
    y = torch.nn.functional.conv1d(torch.from_numpy(G["conv_x"])[None], torch.from_numpy(G["conv_w"]),
                                   torch.from_numpy(G["conv_b"]), stride=6, padding=3)[0].numpy()
    assert np.abs(y - G["conv_y"]).max() <= 1e-5
    C = G["pool_x"].shape[0]
    yp = torch.nn.functional.conv_transpose1d(torch.from_numpy(G["pool_x"])[None],
                                              torch.from_numpy(G["pool_w"]).reshape(C, 1, 3),
                                              torch.from_numpy(G["pool_b"]), stride=2, padding=1, output_padding=1,
                                              groups=C)[0].numpy()
    assert np.abs(yp - G["pool_y"]).max() <= 1e-5
