"""The BF16 mode's tcgen05 attention kernel on its own (kk_attention_selftest) against a float64
restatement with the kernel's roundings: Q, K and V rounded to bf16; scores in fp32 (exact products
of bf16 values accumulated in fp32); p = exp(s / 8 - max) in fp32, rounded to bf16 for the P V
product; normalised by the fp32 sum of the unrounded p (src/gpu_batch.rs:429-442 computes the same
softmax(Q K^T / 8) V per item and head in fp32). Tolerance: relative L2 <= 1e-4 (fp32 accumulation
order), and max-abs error <= 2^-8 x max |v|: where the kernel's fp32 exp and the reference's differ
by one ulp next to a bf16 rounding boundary, one p flips by one bf16 ulp (2^-8 relative, p <= 1),
which moves an output by at most 2^-8 max |v| (the row sum is >= 1).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).to(torch.float32).numpy()


def reference(qkv, lens):
    out = np.zeros((qkv.shape[0], 768), np.float64)
    r0 = 0
    for T in lens:
        blk = qkv[r0:r0 + T]
        for h in range(12):
            q = bf16(blk[:, h * 64:(h + 1) * 64]).astype(np.float64)
            k = bf16(blk[:, 768 + h * 64:768 + (h + 1) * 64]).astype(np.float64)
            v = bf16(blk[:, 1536 + h * 64:1536 + (h + 1) * 64]).astype(np.float64)
            s = (q @ k.T).astype(np.float32) * np.float32(0.125)
            m = s.max(1, keepdims=True)
            p = np.exp((s - m).astype(np.float64)).astype(np.float32)
            l = p.astype(np.float64).sum(1, keepdims=True)
            out[r0:r0 + T, h * 64:(h + 1) * 64] = (bf16(p).astype(np.float64) @ v) / l
        r0 += T
    return out


@pytest.mark.parametrize("lens", [[1, 7, 16, 100, 128], [129, 200, 256], [257, 300, 511, 512], [37, 512, 128, 5]])
def test_tc_attention_matches_reference(kk, lens):
    import kokoro_rust_b200.engine as E
    rng = np.random.default_rng(sum(lens))
    qkv = (rng.standard_normal((sum(lens), 2304)) * 1.5).astype(np.float32)
    got = E.attention_selftest(0, lens, qkv).astype(np.float64)
    ref = reference(qkv, lens)
    err = np.abs(got - ref)
    vmax = np.abs(bf16(qkv[:, 1536:])).max()
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-4
    assert err.max() <= 2.0 ** -8 * vmax, (err.max(), vmax)


@pytest.mark.parametrize("lens", [[1, 7, 16, 100, 128], [257, 300, 511, 512]])
def test_tc_attention_bf16_rows_equal_f32_rows(kk, lens):
    """The BF16 mode's QKV projection writes bf16 rows (round to nearest even) for the attention:
    the same ctx bit for bit as the f32 rows the attention rounds itself."""
    import kokoro_rust_b200.engine as E
    rng = np.random.default_rng(7 + sum(lens))
    qkv = (rng.standard_normal((sum(lens), 2304)) * 1.5).astype(np.float32)
    bits = torch.from_numpy(qkv).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = E.attention_selftest(0, lens, bits, bf16_rows=True)
    want = E.attention_selftest(0, lens, qkv)
    assert np.array_equal(got, want)


def test_tc_attention_rejects_long_items(kk):
    import kokoro_rust_b200.engine as E
    with pytest.raises(E.KokoroError):
        E.attention_selftest(0, [513], np.zeros((513, 2304), np.float32))
