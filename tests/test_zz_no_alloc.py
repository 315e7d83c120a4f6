"""kk_decode_batch_noalloc: the vocoder entry point for callers that cannot allocate device memory
(a streaming audio thread must not wait on cudaMalloc; a GPU shared under a fixed memory budget
must not let the engine's arena grow). It runs on a static device scratch array, so this test
checks it against kk_decode_batch on two calls in a row (the second call reuses the scratch the
first one left behind), checks that it allocates nothing (the engine's arena stays as it was, at
zero bytes on an engine that never ran an allocating call, and the device's free memory does not
move across calls once the library's code is loaded), and checks that batches above its stated
limit are refused."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3  # the fp32 vocoder tolerance used by the parity tests


def inputs(rng, frames):
    asr = [rng.standard_normal((n, 512)).astype(np.float32) for n in frames]
    f0 = []
    for n in frames:
        c = np.exp(rng.uniform(np.log(80), np.log(400), 2 * n)).astype(np.float32)
        c[: max(1, n // 4)] = 0.0  # an unvoiced run
        f0.append(c)
    nc = [rng.standard_normal(2 * n).astype(np.float32) for n in frames]
    s_dec = (rng.standard_normal((len(frames), 128)) * 0.1).astype(np.float32)
    return asr, f0, nc, s_dec


@pytest.fixture(scope="module")
def eng(kk, ckpt_path):
    e = kk.GpuKokoro(ckpt_path, 0, "bf16")
    yield e
    e.close()


def test_noalloc_matches_decode_batch_twice(eng):
    rng = np.random.default_rng(7)
    for frames, seeds in (([40, 30], [3, 4]), ([118], [9])):  # second call: the 120-frame maximum
        asr, f0, nc, s_dec = inputs(rng, frames)
        ref = eng.decode_batch(asr, f0, nc, s_dec, seeds=seeds)
        got = eng.decode_batch_noalloc(asr, f0, nc, s_dec, seeds=seeds)
        assert len(got) == len(ref)
        for g, r, n in zip(got, ref, frames):
            assert g.shape == r.shape == (600 * n,)
            assert np.isfinite(g).all()
            assert np.abs(g - r).max() <= TOL


def test_noalloc_refuses_batches_above_its_limit(kk, eng):
    rng = np.random.default_rng(8)
    asr, f0, nc, s_dec = inputs(rng, [119])  # 119 + 2 gap frames > 120
    with pytest.raises(kk.KokoroError) as e:
        eng.decode_batch_noalloc(asr, f0, nc, s_dec, seeds=[1])
    assert e.value.status == kk.engine.KK_ERR_INVALID_ARG and "120 frames" in str(e.value)
    asr, f0, nc, s_dec = inputs(rng, [2] * 9)
    with pytest.raises(kk.KokoroError) as e:
        eng.decode_batch_noalloc(asr, f0, nc, s_dec, seeds=list(range(9)))
    assert e.value.status == kk.engine.KK_ERR_INVALID_ARG and "8 items" in str(e.value)
    asr, f0, nc, s_dec = inputs(rng, [12])  # still usable after a refusal
    got = eng.decode_batch_noalloc(asr, f0, nc, s_dec, seeds=[2])[0]
    ref = eng.decode_batch(asr, f0, nc, s_dec, seeds=[2])[0]
    assert np.abs(got - ref).max() <= TOL


def test_noalloc_allocates_nothing(kk, ckpt_path, eng):
    rng = np.random.default_rng(9)
    fresh = kk.GpuKokoro(ckpt_path, 0, "bf16")  # an engine that only ever calls the no-allocation entry
    try:
        for frames in ([50, 40], [118]):
            asr, f0, nc, s_dec = inputs(rng, frames)
            fresh.decode_batch_noalloc(asr, f0, nc, s_dec, seeds=list(range(len(frames))))
            st = fresh.memory_stats()
            assert st["arena_bytes"] == 0 and st["peak_bytes"] == 0, st
        free0, _ = fresh.device_memory()
        for frames in ([60, 20], [118]):
            asr, f0, nc, s_dec = inputs(rng, frames)
            fresh.decode_batch_noalloc(asr, f0, nc, s_dec, seeds=list(range(len(frames))))
            assert fresh.device_memory()[0] == free0
        assert fresh.memory_stats()["arena_bytes"] == 0
    finally:
        fresh.close()
    # an engine whose arena already holds a larger call: the no-allocation calls leave it as it is
    asr, f0, nc, s_dec = inputs(rng, [200, 150])
    eng.decode_batch(asr, f0, nc, s_dec, seeds=[1, 2])
    before = eng.memory_stats()
    free0, _ = eng.device_memory()
    for frames in ([30, 30, 30], [118]):
        asr, f0, nc, s_dec = inputs(rng, frames)
        eng.decode_batch_noalloc(asr, f0, nc, s_dec, seeds=list(range(len(frames))))
    after = eng.memory_stats()
    assert after["arena_bytes"] == before["arena_bytes"] and after["peak_bytes"] == before["peak_bytes"]
    assert eng.device_memory()[0] == free0
