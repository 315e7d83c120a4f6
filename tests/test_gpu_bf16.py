"""BF16 precision mode (tcgen05 convolutions, linears and attention with bf16 operands and fp32
accumulation; LSTM recurrence with bf16 hi / lo split operands) against the CPU oracle, end to end.

Bounds, measured on this checkpoint and stated with headroom:
* predicted integer durations equal the oracle's (ALBERT, duration LSTMs in BF16), except where
  the oracle's unrounded duration lies within 0.02 of a rounding tie; every duration, ties included,
  is within 1 frame of the oracle's;
* F0 / N curves (the predictor's outputs, forced durations) within 2.5e-2 / 8e-2 relative L2
  (measured about 1.2e-2 / 4e-2: bf16 operands through ALBERT, the predictor LSTMs and the
  AdaIN resblocks; the reference's own mixed-precision build moves F0 by the same order);
* the vocoder (decoder + generator on identical inputs) at >= 40 dB SNR (measured 42 dB).
"""
import os
import tempfile

import numpy as np
import pytest

from conftest import synth_item
from test_gpu_parity import vocoder_inputs

pytestmark = pytest.mark.gpu

GAP_N = 2  # frame-domain rows between items (kk_common.cuh)


@pytest.fixture(scope="module")
def eng16(kk, ckpt_path):
    e = kk.GpuKokoro(ckpt_path, 0, "bf16")
    yield e
    e.close()


@pytest.fixture(scope="module")
def cases(kk, oracle):
    """Items spanning the three attention buckets (<= 128, <= 256, <= 512 tokens)."""
    rng = np.random.default_rng(21)
    items, refs = [], []
    for i, n in enumerate((9, 60, 140, 300)):
        ids, ref_s = synth_item(rng, n)
        items.append(kk.BatchItem(ids, ref_s, 1.0, kk.ItemNoise(seed=100 + i)))
        refs.append(oracle.forward(ids, ref_s, 1.0, seed=100 + i, want=("dur_q", "f0")))
    return items, refs


def test_bf16_durations_match_oracle(eng16, cases):
    items, refs = cases
    outs = eng16.forward_batch(items)
    for o, r in zip(outs, refs):
        tie = np.abs(r["dur_q"] - np.floor(r["dur_q"]) - 0.5) < 0.02
        assert np.array_equal(o.pred_dur[~tie], r["dur"][~tie]), (o.pred_dur, r["dur"])
        assert np.abs(o.pred_dur - r["dur"]).max() <= 1


def test_bf16_f0_n_curves(eng16, cases):
    items, refs = cases
    d = tempfile.mkdtemp()
    os.environ["KK_DEBUG_DUMP_DIR"] = d  # the engine writes its f0 / nc buffers here
    try:
        eng16.forward_batch(items, forced_dur=[r["dur"] for r in refs])
    finally:
        del os.environ["KK_DEBUG_DUMP_DIR"]
    f0 = np.fromfile(os.path.join(d, "f0.f32"), np.float32)
    nc = np.fromfile(os.path.join(d, "nc.f32"), np.float32)
    a = 0
    for r in refs:
        n = int(r["dur"].sum())
        g0, gn = f0[2 * a:2 * (a + n)], nc[2 * a:2 * (a + n)]
        rf, rn = r["f0"].reshape(-1), r["n"].reshape(-1)
        e0 = np.linalg.norm(g0 - rf) / np.linalg.norm(rf)
        en = np.linalg.norm(gn - rn) / np.linalg.norm(rn)
        print(f"frames {n}: f0 rel-L2 {e0:.3g}, n rel-L2 {en:.3g}")
        assert e0 <= 2.5e-2 and en <= 8e-2
        a += n + GAP_N


def test_bf16_vocoder_snr(eng16, oracle, oracle_mod):
    import torch
    rng = np.random.default_rng(3)
    inp = [vocoder_inputs(rng, n) for n in (23, 9, 200)]
    seeds = [11, 12, 13]
    outs = eng16.decode_batch([x[0] for x in inp], [x[1] for x in inp], [x[2] for x in inp],
                              np.stack([x[3] for x in inp]), seeds=seeds)
    for (asr, f0, n, s_dec), seed, a in zip(inp, seeds, outs):
        noise = oracle_mod.counter_noise(seed, 600 * asr.shape[0] * 9)
        r = oracle.decode(torch.from_numpy(asr.T.copy()), f0, n, torch.from_numpy(s_dec), noise)
        snr = 10 * np.log10((r ** 2).sum() / ((a - r) ** 2).sum())
        print(f"frames {asr.shape[0]}: vocoder SNR {snr:.1f} dB")
        assert a.shape == r.shape and snr >= 40.0


def test_bf16_attention_kernel_effect(kk, eng16, cases):
    """What the tensor-core attention (bf16 Q, K, V, P) changes against the reference's f32
    attention (src/gpu.rs:199-230), everything else of the BF16 mode equal: durations and F0 against
    the oracle with each attention kernel (KK_OPT_ATTENTION_F32 selects the fp32 one)."""
    items, refs = cases
    res = {}
    for name, opt in (("tcgen05", 0), ("f32", 1)):
        eng16.set_option(kk.engine.KK_OPT_ATTENTION_F32, opt)
        try:
            outs = eng16.forward_batch(items)
            d = tempfile.mkdtemp()
            os.environ["KK_DEBUG_DUMP_DIR"] = d
            try:
                eng16.forward_batch(items, forced_dur=[r["dur"] for r in refs])
            finally:
                del os.environ["KK_DEBUG_DUMP_DIR"]
        finally:
            eng16.set_option(kk.engine.KK_OPT_ATTENTION_F32, 0)
        f0 = np.fromfile(os.path.join(d, "f0.f32"), np.float32)
        diff = sum(int((o.pred_dur != r["dur"]).sum()) for o, r in zip(outs, refs))
        a, e0 = 0, []
        for r in refs:
            n = int(r["dur"].sum())
            rf = r["f0"].reshape(-1)
            e0.append(float(np.linalg.norm(f0[2 * a:2 * (a + n)] - rf) / np.linalg.norm(rf)))
            a += n + GAP_N
        res[name] = (diff, max(e0))
        print(f"attention {name}: {diff} of {sum(len(r['dur']) for r in refs)} durations differ from the oracle, "
              f"F0 rel-L2 max {max(e0):.3g}")
    assert res["tcgen05"][1] <= 2.5e-2 and res["f32"][1] <= 2.5e-2
