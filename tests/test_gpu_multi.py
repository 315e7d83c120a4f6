"""The per-GPU worker processes of multi.MultiEngine on real B200s: every visible GPU gets a worker
holding its own engine; synth_batch over them returns, in request order, the audio the in-process
engine gives for the same requests, although every worker batches only its own share.

* FP32 mode: durations equal and audio bit-identical (batching never changes an item's result:
  every kernel of the fp32 path computes an item's rows in an order that does not depend on where
  the item sits in the batch, and its AdaIN sums are exact f64 sums of item-relative f32 chunks);
* BF16 mode: durations equal; the waveforms are reported, not compared (the fused per-tile AdaIN
  sums group rows by tile, so a different batch moves a statistic in the last bit, which flips the
  bf16 rounding of a few convolution inputs and, through F0, drifts the source phase; the
  reference's own BF16x product is batch-composition dependent too, durations included, and its
  regression tests report such lines instead of comparing them, tests/bf16x_regression.rs:74-79).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def requests():
    rng = np.random.default_rng(11)
    pack = (rng.standard_normal((510, 256)) * 0.1).astype(np.float32)
    reqs = [(rng.integers(1, 178, int(n)), 500 + i) for i, n in enumerate(rng.integers(8, 200, 12))]
    reqs[4] = ([], 4)  # empty: a per-request error in both
    return pack, reqs


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_multi_engine_matches_in_process_engine(kk, ckpt_path, gspec, spec_db, precision):
    import torch
    from kokoro_rust_b200.multi import MultiEngine
    n_gpu = torch.cuda.device_count()
    pack, reqs = requests()
    one = kk.Engine(ckpt_path, 0, precision)
    one.add_voice("v", pack)
    ref = one.synth_batch(reqs, "v", 1.0)
    one.gpu.close()
    with MultiEngine(ckpt_path, list(range(n_gpu)), precision) as m:
        m.add_voice("v", pack)
        got = m.synth_batch(reqs, "v", 1.0)
    worst = 0.0
    for r, g in zip(ref, got):
        if isinstance(r, Exception):
            assert isinstance(g, Exception)
            continue
        assert np.array_equal(r.pred_dur, g.pred_dur)
        assert r.audio.shape == g.audio.shape
        assert np.isfinite(g.audio).all()
        if precision == "fp32" or n_gpu == 1:
            assert np.array_equal(r.audio, g.audio)
        elif r.audio.shape[0] >= 1024:
            worst = max(worst, spec_db(r.audio, g.audio))
    print(f"{n_gpu} GPU worker(s), {precision}: worst spectral distance {worst:.3f} dB "
          f"(the G-SPEC gate of the fp32 path: {gspec['gate']:.3f} dB)")
    if precision == "fp32" or n_gpu == 1:  # one worker batches exactly as the in-process engine
        assert worst <= gspec["gate"]
