"""PCM_16 conversion on the device (KK_OPT_OUTPUT_PCM16 + kk_fetch_audio_pcm16) against the host
WAV encoder (kk_wav_encode, the rule of src/wav.rs:76-84) applied to the same forward's f32 audio:
bit-exact samples and equal clip counts. The forward is deterministic (counter noise, fixed
durations), so the f32 and PCM_16 runs produce the same audio."""
import numpy as np
import pytest

from conftest import synth_item

pytestmark = pytest.mark.gpu


def test_device_pcm16_equals_host_encoding(kk, ckpt_path):
    rng = np.random.default_rng(11)
    items, durs = [], []
    for i, n in enumerate([7, 30, 15]):
        ids, ref_s = synth_item(rng, n, style_sd=0.3)
        items.append(kk.BatchItem(ids, ref_s, 1.0, kk.ItemNoise(seed=100 + i)))
        durs.append(np.concatenate([[0], rng.integers(1, 4, n), [0]]).astype(np.int64))
    e = kk.GpuKokoro(ckpt_path, 0, "bf16")
    try:
        f = e.forward_batch(items, forced_dur=durs)
        # scale up so some samples clip
        items2 = [kk.BatchItem(it.ids, it.ref_s * 4.0, 1.0, it.noise) for it in items]
        f2 = e.forward_batch(items2, forced_dur=durs)
        p = e.forward_batch(items, forced_dur=durs, pcm16=True)
        p2 = e.forward_batch(items2, forced_dur=durs, pcm16=True)
    finally:
        e.close()
    for fa, pa in zip(f + f2, p + p2):
        enc = kk.wav.encode(fa.audio, 24000, kk.wav.Format.Pcm16)
        assert pa.audio.dtype == np.int16 and pa.audio.size == fa.audio.size
        assert np.frombuffer(enc.bytes[44:], "<i2").tobytes() == pa.audio.astype("<i2").tobytes()
        assert pa.clipped == enc.clipped
        assert kk.wav.encode_pcm16_samples(pa.audio, 24000) == enc.bytes
