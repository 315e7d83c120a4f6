"""Batch semantics of the ragged layout (the reference's batching contract, docs/design/BATCHING.md:
batching never changes an item's result) and the failure paths, through the C ABI.

* batch vs single (fp32): an item alone and the same item in the middle of a 3-item batch give equal
  predicted durations and bit-identical audio (forced durations short enough that every AdaIN
  statistic is one chunk, so no f64 atomic order enters);
* gap canary: with every device buffer filled with NaN before use, outputs are unchanged (fp32
  bit-identical; BF16 within 1e-3 of the unpoisoned run) and finite, so no kernel reads a gap row or
  any other element before it is written;
* negative control: with the gap mask switched off (KK_OPT_NEGCTL_NOMASK, the reference's
  KOKORO_BATCH_NEGCTL_NOMASK, src/gpu_batch.rs:62-66 and tests/bf16x_regression.rs:47-55) the
  batched item no longer equals the single one, so the batch test above detects leakage;
* ItemNoise::Fixed with predicted durations (src/gpu_batch.rs:337-340): replayed draws equal to an
  item's counter stream reproduce the counter run, items may mix both kinds, and a draw count that
  does not match the predicted durations is refused;
* bounded waits: a wait on a barrier nothing arrives on gives up with KK_ERR_TIMEOUT and the engine
  stays usable.
"""
import numpy as np
import pytest

from conftest import synth_item

pytestmark = pytest.mark.gpu


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


def three_items(kk):
    """Three short items with forced durations of 2 frames per token (at most 16 frames each)."""
    rng = np.random.default_rng(31)
    items, durs = [], []
    for i, n in enumerate((6, 4, 5)):
        ids, ref_s = synth_item(rng, n)
        items.append(kk.BatchItem(ids, ref_s, 1.0, kk.ItemNoise(seed=40 + i)))
        durs.append(np.concatenate([[0], np.full(n, 2), [0]]).astype(np.int64))
    return items, durs


def test_batch_vs_single_fp32(kk, eng32):
    items, durs = three_items(kk)
    single = eng32.forward_batch([items[1]], forced_dur=[durs[1]])[0]
    batch = eng32.forward_batch(items, forced_dur=durs)
    assert np.array_equal(batch[1].audio, single.audio)
    # predicted durations: alone and batched
    p1 = eng32.forward_batch([items[1]])[0]
    pb = eng32.forward_batch(items)
    assert np.array_equal(pb[1].pred_dur, p1.pred_dur)
    assert np.array_equal(pb[1].audio, p1.audio) or np.abs(pb[1].audio - p1.audio).max() <= 1e-6


def test_gap_canary_fp32(kk, eng32):
    items, durs = three_items(kk)
    ref = eng32.forward_batch(items, forced_dur=durs)
    eng32.set_option(kk.engine.KK_OPT_GAP_CANARY, 1)
    try:
        got = eng32.forward_batch(items, forced_dur=durs)
        pred = eng32.forward_batch(items)
    finally:
        eng32.set_option(kk.engine.KK_OPT_GAP_CANARY, 0)
    for g, r in zip(got, ref):
        assert np.isfinite(g.audio).all()
        assert np.array_equal(g.audio, r.audio)
    for p in pred:
        assert np.isfinite(p.audio).all()


def test_gap_canary_bf16(kk, eng16):
    items, durs = three_items(kk)
    ref = eng16.forward_batch(items, forced_dur=durs)
    eng16.set_option(kk.engine.KK_OPT_GAP_CANARY, 1)
    try:
        got = eng16.forward_batch(items, forced_dur=durs)
    finally:
        eng16.set_option(kk.engine.KK_OPT_GAP_CANARY, 0)
    for g, r in zip(got, ref):
        assert np.isfinite(g.audio).all()
        assert np.abs(g.audio - r.audio).max() <= 1e-3


def test_negative_control_nomask_changes_outputs(kk, eng32):
    items, durs = three_items(kk)
    single = eng32.forward_batch([items[1]], forced_dur=[durs[1]])[0]
    eng32.set_option(kk.engine.KK_OPT_NEGCTL_NOMASK, 1)
    try:
        leaky = eng32.forward_batch(items, forced_dur=durs)
    finally:
        eng32.set_option(kk.engine.KK_OPT_NEGCTL_NOMASK, 0)
    d = float(np.abs(leaky[1].audio - single.audio).max())
    print(f"no-mask negative control: batched item differs from the single run by max-abs {d:.3g}")
    assert d > 1e-3
    again = eng32.forward_batch(items, forced_dur=durs)  # the mask is back
    assert np.array_equal(again[1].audio, single.audio)


def test_negative_control_refused_in_bf16(kk, eng16):
    with pytest.raises(kk.KokoroError) as e:
        eng16.set_option(kk.engine.KK_OPT_NEGCTL_NOMASK, 1)
    assert e.value.status == kk.engine.KK_ERR_INVALID_ARG


def test_fixed_noise_with_predicted_durations(kk, eng32, oracle_mod):
    rng = np.random.default_rng(32)
    items = []
    for i, n in enumerate((7, 11)):
        ids, ref_s = synth_item(rng, n)
        items.append(kk.BatchItem(ids, ref_s, 1.0, kk.ItemNoise(seed=50 + i)))
    ref = eng32.forward_batch(items)  # counter noise, predicted durations
    frames = [int(o.pred_dur.sum()) for o in ref]
    fixed = [kk.BatchItem(it.ids, it.ref_s, 1.0,
                          kk.ItemNoise(sine=oracle_mod.counter_noise(it.noise.seed, 600 * 9 * f),
                                       rand_ini=rng.uniform(0, 1, 9).astype(np.float32)))
             for it, f in zip(items, frames)]
    got = eng32.forward_batch(fixed)  # every item replayed, no forced durations
    for g, r in zip(got, ref):
        assert np.array_equal(g.pred_dur, r.pred_dur)
        assert np.abs(g.audio - r.audio).max() <= 1e-5
    mixed = eng32.forward_batch([fixed[0], items[1]])  # ItemNoise::Fixed and ::Counter in one batch
    for g, r in zip(mixed, ref):
        assert np.abs(g.audio - r.audio).max() <= 1e-5
    short = kk.BatchItem(items[0].ids, items[0].ref_s, 1.0,
                         kk.ItemNoise(sine=oracle_mod.counter_noise(1, 600 * 9 * (frames[0] - 1))))
    with pytest.raises(kk.KokoroError) as e:
        eng32.forward_batch([short, items[1]])
    assert e.value.status == kk.engine.KK_ERR_INVALID_ARG and "fixed noise size mismatch for item 0" in str(e.value)


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_bounded_wait_expires_and_engine_recovers(kk, eng32, eng16, precision):
    eng = eng32 if precision == "fp32" else eng16
    items, durs = three_items(kk)
    before = eng.forward_batch(items, forced_dur=durs)
    with pytest.raises(kk.KokoroError) as e:
        eng.wait_selftest(5000)  # 5 us on a barrier nothing arrives on
    assert e.value.status == kk.engine.KK_ERR_TIMEOUT and "error flag 2" in str(e.value)
    after = eng.forward_batch(items, forced_dur=durs)  # the next call runs normally
    for a, b in zip(after, before):
        assert np.isfinite(a.audio).all()
        assert np.abs(a.audio - b.audio).max() <= (0.0 if precision == "fp32" else 1e-3)


def test_batch_vs_single_bf16(kk, eng16):
    """BF16 mode: every layer runs the same arithmetic whatever the batch (the layouts hold at
    least 64 rows, so no layer of a small batch falls back to the fp32 kernel; the style
    projections are fp32 for every batch). Durations are equal; the audio differs only through the
    fused AdaIN sums of the tensor-core epilogue, which add f32 partial sums of absolute 128-row
    tiles: a last-bit change of a statistic flips the bf16 rounding of a few convolution inputs, a
    bf16-sized perturbation, so the bound is the BF16 mode's own (SNR >= 40 dB). The reference's own
    BF16x product depends on the batch composition too, durations included
    (docs/design/BATCHING.md:7-13); element-wise f64 sums would make this mode batch-invariant bit
    for bit (measured) at 4-5 ms per config-4 forward, and are not used."""
    items, durs = three_items(kk)
    single = eng16.forward_batch([items[1]], forced_dur=[durs[1]])[0]
    batch = eng16.forward_batch(items, forced_dur=durs)
    r = single.audio.astype(np.float64)
    err = float(((batch[1].audio - r) ** 2).sum())
    snr = 10 * np.log10((r ** 2).sum() / err) if err > 0 else float("inf")
    print(f"bf16 batch vs single: max-abs {np.abs(batch[1].audio - r).max():.3g}, SNR {snr:.1f} dB")
    assert snr >= 40.0
    p1 = eng16.forward_batch([items[1]])[0]
    pb = eng16.forward_batch(items)
    assert np.array_equal(pb[1].pred_dur, p1.pred_dur)


def test_bf16_reproducible_across_runs(kk, eng16):
    """The same batch twice gives the same audio bit for bit (the reference's reproducibility gate,
    tests/bf16x_regression.rs:35-46): every reduction of the path has a fixed order, and the AdaIN
    sums' f64 accumulation of f32 partials does not depend on the order of the atomic adds."""
    items, durs = three_items(kk)
    a = eng16.forward_batch(items)
    b = eng16.forward_batch(items)
    for x, y in zip(a, b):
        assert np.array_equal(x.pred_dur, y.pred_dur)
        assert np.array_equal(x.audio, y.audio)
