"""Host-side scheduling mirror of the reference engine (src/engine.rs:46-241)."""
import numpy as np
import pytest


def ref_plan(lens, max_ph, max_items):
    """Restatement of plan_batches (src/engine.rs:165-183) used as the expected answer."""
    order = sorted(range(len(lens)), key=lambda i: (lens[i], i))
    out, cur, s = [], [], 0
    for i in order:
        if cur and (len(cur) >= max_items or s + lens[i] > max_ph):
            out.append(cur)
            cur, s = [], 0
        s += lens[i]
        cur.append(i)
    return out + ([cur] if cur else [])


def test_plan_batches_budget_and_order(kk):
    rng = np.random.default_rng(0)
    lens = list(rng.integers(2, 512, 300))
    p = kk.BatchPolicy(max_phonemes=4000, max_items=64)
    plan = kk.plan_batches(lens, p)
    assert plan == ref_plan(lens, 4000, 64)
    assert sorted(i for b in plan for i in b) == list(range(300))
    for b in plan:
        assert len(b) <= 64 and (len(b) == 1 or sum(lens[i] for i in b) <= 4000)
    flat = [lens[i] for b in plan for i in b]
    assert flat == sorted(flat)
    assert kk.plan_batches([], p) == []
    assert kk.plan_batches([9999], p) == [[0]]  # oversize single item still gets a batch


class FakeGpu:
    """Fails any batch larger than `limit` with OOM (the split-in-half trigger)."""

    def __init__(self, kk, limit):
        self.kk, self.limit, self.calls = kk, limit, []

    def forward_batch(self, items):
        self.calls.append(len(items))
        if len(items) > self.limit:
            raise self.kk.KokoroError(2, "device arena: cannot allocate")
        return [self.kk.Output(np.full(600 * len(it.ids), float(len(it.ids)), np.float32),
                               np.full(len(it.ids), 1, np.int64)) for it in items]


def make_engine(kk, limit):
    e = kk.Engine.__new__(kk.Engine)
    e.gpu = FakeGpu(kk, limit)
    e.voices = {}
    e.add_voice("v", np.arange(510 * 256, dtype=np.float32).reshape(510, 256))
    return e


def test_synth_batch_splits_in_half_and_keeps_order(kk):
    e = make_engine(kk, limit=3)
    rng = np.random.default_rng(1)
    reqs = [(list(rng.integers(1, 178, n)), i) for i, n in enumerate(rng.integers(1, 60, 17))]
    reqs[4] = ([], 4)                  # empty -> per-item error
    reqs[9] = (list(range(1, 600)), 9)  # oversize -> per-item error
    res = e.synth_batch(reqs, "v", 1.0, kk.BatchPolicy(max_phonemes=10_000, max_items=64))
    assert len(res) == 17
    for i, r in enumerate(res):
        if i in (4, 9):
            assert isinstance(r, Exception)
        else:
            n_ids = len(reqs[i][0]) + 2
            assert r.audio.shape == (600 * n_ids,) and r.audio[0] == n_ids  # its own output
    # split-in-half order of src/engine.rs:229-234: a failing batch is replaced by its halves,
    # first half first
    expect, stack = [], [15]
    while stack:
        n = stack.pop()
        expect.append(n)
        if n > 3:
            stack += [n - n // 2, n // 2]
    assert e.gpu.calls == expect


def test_single_item_failure_is_reported(kk):
    e = make_engine(kk, limit=0)
    res = e.synth_batch([([1, 2, 3], 0), ([4, 5], 1)], "v")
    assert all(isinstance(r, kk.KokoroError) for r in res)


def test_voice_rules(kk):
    e = make_engine(kk, limit=10)
    v = e.voice("v")
    assert np.array_equal(v.ref_s(1), v.pack[0]) and np.array_equal(v.ref_s(510), v.pack[509])
    with pytest.raises(ValueError):
        v.ref_s(0)
    with pytest.raises(ValueError):
        v.ref_s(511)
    e.add_voice("w", np.zeros((510, 256), np.float32))
    assert np.allclose(e.voice("v,w").pack, v.pack / 2)


class FakeMem:
    """memory_stats / device_memory of a GpuKokoro, for the free-VRAM budget arithmetic."""

    def __init__(self, free, arena=0, peak=0, tokens=0, frames=0):
        self.free, self.st = free, {"weight_bytes": 330 << 20, "arena_bytes": arena, "peak_bytes": peak,
                                    "tokens": tokens, "frames": frames}

    def memory_stats(self):
        return dict(self.st)

    def device_memory(self):
        return self.free, 180 << 30


def test_free_vram_budget(kk):
    E = kk.engine
    # before any forward: the built-in per-frame and per-phoneme figures
    p = kk.BatchPolicy.from_free_vram(FakeMem(free=100 << 30), headroom=0.5)
    frames = (100 << 30) * 0.5 / E.DEFAULT_BYTES_PER_FRAME
    assert p.max_phonemes == int(frames / E.DEFAULT_FRAMES_PER_PHONEME)
    # the arena the engine already holds is reusable; a faster speed means fewer frames per phoneme
    p2 = kk.BatchPolicy.from_free_vram(FakeMem(free=60 << 30, arena=40 << 30), headroom=0.5, speed=2.0)
    assert p2.max_phonemes == int(frames / (E.DEFAULT_FRAMES_PER_PHONEME / 2.0))
    # after a forward: that call's bytes per frame and frames per phoneme (never below the default)
    m = FakeMem(free=50 << 30, arena=10 << 30, peak=16 << 30, tokens=10_000, frames=40_000)
    p3 = kk.BatchPolicy.from_free_vram(m, headroom=1.0)
    assert p3.max_phonemes == int((60 << 30) / ((16 << 30) / 40_000) / 4.0)
    m = FakeMem(free=50 << 30, arena=10 << 30, peak=16 << 30, tokens=40_000, frames=40_000)
    assert kk.BatchPolicy.from_free_vram(m, headroom=1.0).max_phonemes == int(
        (60 << 30) / ((16 << 30) / 40_000) / E.DEFAULT_FRAMES_PER_PHONEME)
    # a calibration call with an implausibly small working set cannot inflate the budget
    m = FakeMem(free=50 << 30, arena=10 << 30, peak=1 << 20, tokens=40_000, frames=40_000)
    assert kk.BatchPolicy.from_free_vram(m, headroom=1.0).max_phonemes == int(
        (60 << 30) / (E.DEFAULT_BYTES_PER_FRAME * 0.5) / E.DEFAULT_FRAMES_PER_PHONEME)
    # a nearly full device still admits one maximal item (the OOM split handles the rest)
    assert kk.BatchPolicy.from_free_vram(FakeMem(free=1 << 20)).max_phonemes == kk.engine.MAX_PHONEMES + 2
    plan = kk.plan_batches([100] * 50, kk.BatchPolicy(max_phonemes=p.max_phonemes, max_items=p.max_items))
    assert sum(len(b) for b in plan) == 50
