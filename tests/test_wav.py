"""WAV output (src/wav.rs) through the C ABI: header, PCM_16 / float32 encoding, in-order assembly
with per-part sha256 checks, on the reference's own test cases (src/wav.rs:195-277), checked against
the numpy restatement in oracle/ and Python's hashlib."""
import hashlib
import os

import numpy as np
import pytest


def ref_lines():
    """The three lines of the reference's wav tests (src/wav.rs:207-213)."""
    return [
        (np.sin(np.arange(1000, dtype=np.float32) * np.float32(0.01)) * np.float32(0.5)).astype(np.float32),
        np.array([0.25, -1.5, 1.5, 0.0, -0.3333], np.float32),  # includes clipped samples
        ((np.arange(777) % 17).astype(np.float32) - 8.0) / np.float32(9.0),
    ]


@pytest.fixture(scope="module")
def wav(kk):
    return kk.wav


@pytest.mark.parametrize("fmt", [0, 1], ids=["pcm16", "float32"])
def test_encode_matches_oracle_on_reference_lines(wav, oracle_mod, fmt):
    for a in ref_lines():
        e = wav.encode(a, 24000, wav.Format(fmt))
        want, clipped = oracle_mod.wav_encode(a, 24000, fmt)
        assert e.bytes == want
        assert e.clipped == clipped
    assert wav.encode(ref_lines()[1], 24000, wav.Format.Pcm16).clipped == 2


def test_pcm16_rounding_clamping_and_nan(wav, oracle_mod):
    rng = np.random.default_rng(5)
    # exact half-way products, values just inside / outside the range, and non-finite samples
    ties = (np.arange(-40, 40, dtype=np.float32) + np.float32(0.5)) / np.float32(32767.0)
    edge = np.array([1.0, -1.0, 1.0000153, -1.0000306, 32768 / 32767, -32768.5 / 32767, np.inf, -np.inf, np.nan,
                     0.0, -0.0], np.float32)
    a = np.concatenate([ties, edge, rng.uniform(-1.2, 1.2, 5000).astype(np.float32)])
    e = wav.encode(a, 24000, wav.Format.Pcm16)
    want, clipped = oracle_mod.wav_encode(a, 24000, 0)
    assert e.bytes == want and e.clipped == clipped
    pcm = np.frombuffer(e.bytes[44:], "<i2")
    assert pcm[len(ties) + 8] == 0  # NaN stored as 0


def test_assembly_equals_encoding_the_concatenated_samples(wav, tmp_path):
    for fmt in (wav.Format.Pcm16, wav.Format.Float32):
        d = tmp_path / f"exact-{fmt.name}"
        d.mkdir()
        ls = ref_lines()
        parts = wav.write_lines(ls, str(d), 24000, fmt)
        dest = str(d / "book.wav")
        a = wav.assemble(parts, fmt, 24000, dest, sync=False)
        want = wav.encode(np.concatenate(ls), 24000, fmt).bytes
        got = open(dest, "rb").read()
        assert got == want
        assert a.samples == sum(x.size for x in ls)
        assert a.sha256 == hashlib.sha256(want).hexdigest()
        assert wav.read_canonical(dest, fmt, 24000) == a.data_bytes
        assert not os.path.exists(d / ".book.wav.partial")


def test_riff_size_limit_is_enforced_not_wrapped(wav):
    wav.check_riff_size(wav.MAX_DATA_BYTES)
    with pytest.raises(wav.WavError):
        wav.check_riff_size(wav.MAX_DATA_BYTES + 1)
    with pytest.raises(wav.WavError):
        wav.check_riff_size(0xFFFFFFFF + 10)
    h = wav.header(wav.Format.Pcm16, 24000, wav.MAX_DATA_BYTES)
    assert int.from_bytes(h[4:8], "little") == 0xFFFFFFFF
    with pytest.raises(wav.WavError):
        wav.header(wav.Format.Float32, 24000, wav.MAX_DATA_BYTES + 2)


def test_corrupt_or_mismatched_parts_leave_the_destination_untouched(wav, tmp_path):
    ls = ref_lines()
    dest = tmp_path / "book.wav"
    dest.write_bytes(b"previous good output")

    def unchanged():
        assert dest.read_bytes() == b"previous good output"
        assert not (tmp_path / ".book.wav.partial").exists()

    def fresh(name):
        d = tmp_path / name
        d.mkdir()
        return wav.write_lines(ls, str(d), 24000, wav.Format.Pcm16)

    parts = fresh("changed")  # a sample changed after synthesis: caught by the hash
    b = bytearray(open(parts[1][0], "rb").read())
    b[44] ^= 1
    open(parts[1][0], "wb").write(bytes(b))
    with pytest.raises(wav.WavError, match="changed since it was synthesized"):
        wav.assemble(parts, wav.Format.Pcm16, 24000, str(dest), sync=False)
    unchanged()
    parts = fresh("truncated")
    b = open(parts[2][0], "rb").read()
    open(parts[2][0], "wb").write(b[:-3])
    with pytest.raises(wav.WavError):
        wav.assemble(parts, wav.Format.Pcm16, 24000, str(dest), sync=False)
    unchanged()
    parts = fresh("missing")
    os.remove(parts[0][0])
    with pytest.raises(wav.WavError):
        wav.assemble(parts, wav.Format.Pcm16, 24000, str(dest), sync=False)
    unchanged()
    parts = fresh("format")
    with pytest.raises(wav.WavError):
        wav.assemble(parts, wav.Format.Float32, 24000, str(dest), sync=False)
    with pytest.raises(wav.WavError):
        wav.assemble(parts, wav.Format.Pcm16, 22050, str(dest), sync=False)
    unchanged()


@pytest.mark.parametrize("n", [0, 1, 55, 56, 63, 64, 65, 119, 120, 1000, 1 << 16])
def test_sha256_matches_hashlib(wav, n):
    data = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8).tobytes()
    assert wav.sha256_hex(data) == hashlib.sha256(data).hexdigest()
