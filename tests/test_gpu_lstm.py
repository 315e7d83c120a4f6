"""The BiLSTM recurrence kernels on their own (kk_lstm_selftest) against a float64 restatement of
kernels/kokoro.cu:400-450 (gates = gx + (W_hh h + b_hh), order i, f, g, o; c = f c + i g;
h = o tanh(c); the reverse direction runs each item backwards), on ragged items.

Tolerances (max-abs on h, which lies in (-1, 1)): 1e-5 for both kernels. The fp32 cluster kernel
rounds in fp32 over up to 100 recurrent steps; the BF16 mode's tcgen05 kernel splits both operands
of the recurrent product into fp16 big and scaled small parts (22 significant bits each, exact
products, fp32 accumulation: the "3xTF32" split-operand method with fp16 halves), so it must reach
the same fp32-level error, and the test prints both errors side by side.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def reference(lens, gx, whh, bhh):
    out = np.zeros((gx.shape[0], 512))
    r0 = 0
    for T in lens:
        for d in range(2):
            W = whh[d].astype(np.float64)
            b = bhh[d].astype(np.float64)
            h = np.zeros(256)
            c = np.zeros(256)
            steps = range(T) if d == 0 else range(T - 1, -1, -1)
            for t in steps:
                g = gx[r0 + t, d * 1024:(d + 1) * 1024].astype(np.float64) + (W @ h + b)
                i, f, gg, o = g[:256], g[256:512], g[512:768], g[768:]
                sig = lambda x: 1.0 / (1.0 + np.exp(-x))  # noqa: E731
                c = sig(f) * c + sig(i) * np.tanh(gg)
                h = sig(o) * np.tanh(c)
                out[r0 + t, d * 256:(d + 1) * 256] = h
        r0 += T
    return out


@pytest.mark.parametrize("tc,tol", [(0, 1e-5), (1, 1e-5)], ids=["fp32", "tcgen05"])
def test_lstm_recurrence_matches_reference(kk, tc, tol):
    import kokoro_rust_b200.engine as E
    rng = np.random.default_rng(7)
    lens = [100, 1, 37, 64, 99, 3, 17, 80, 55, 2, 91, 33]
    rows = sum(lens)
    gx = (rng.standard_normal((rows, 2048)) * 0.8).astype(np.float32)
    whh = (rng.standard_normal((2, 1024, 256)) / 16.0).astype(np.float32)
    bhh = (rng.standard_normal((2, 1024)) * 0.1).astype(np.float32)
    got = E.lstm_selftest(0, tc, lens, gx, whh, bhh)
    ref = reference(lens, gx, whh, bhh)
    err = np.abs(got - ref).max()
    print(f"lstm {'tcgen05' if tc else 'fp32'}: max-abs error {err:.3g} against float64")
    assert err <= tol, err


def test_lstm_selftest_rejects_oversized_group(kk):
    import kokoro_rust_b200.engine as E
    with pytest.raises(E.KokoroError):
        E.lstm_selftest(0, 0, [2] * 33, np.zeros((66, 2048), np.float32), np.zeros((2, 1024, 256), np.float32),
                        np.zeros((2, 1024), np.float32))
