"""The per-GPU worker processes of multi.MultiEngine on real B200s: every visible GPU gets a worker
holding its own engine; synth_batch over them returns, in request order, the audio the in-process
engine gives for the same requests (same durations, bf16 waveforms within the bf16 path's SNR
bar)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_multi_engine_matches_in_process_engine(kk, ckpt_path):
    import torch
    from kokoro_rust_b200.multi import MultiEngine
    n_gpu = torch.cuda.device_count()
    rng = np.random.default_rng(11)
    pack = (rng.standard_normal((510, 256)) * 0.1).astype(np.float32)
    reqs = [(rng.integers(1, 178, int(n)), 500 + i) for i, n in enumerate(rng.integers(8, 200, 12))]
    reqs[4] = ([], 4)  # empty: a per-request error in both
    one = kk.Engine(ckpt_path, 0, "bf16")
    one.add_voice("v", pack)
    ref = one.synth_batch(reqs, "v", 1.0)
    one.gpu.close()
    with MultiEngine(ckpt_path, list(range(n_gpu)), "bf16") as m:
        m.add_voice("v", pack)
        got = m.synth_batch(reqs, "v", 1.0)
    for r, g in zip(ref, got):
        if isinstance(r, Exception):
            assert isinstance(g, Exception)
            continue
        assert np.array_equal(r.pred_dur, g.pred_dur)
        assert r.audio.shape == g.audio.shape
        err = float(np.sum((r.audio.astype(np.float64) - g.audio) ** 2))
        sig = float(np.sum(r.audio.astype(np.float64) ** 2))
        assert err == 0.0 or 10 * np.log10(sig / err) >= 40.0
