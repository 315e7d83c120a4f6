"""The bf16 tcgen05 convolution kernel on its own, through kk_conv_selftest, against a float64
convolution of the same bf16-rounded operands, on both input routes: the producer warps transform
the input inside the conv ("fused"), or a prologue kernel writes bf16 window planes that the conv
bulk-copies ("pre", the route of layers with more than 128 output channels).

The kernel stages its input as bf16 after the layer's prologue (gap mask, AdaIN folded to
x * A + B, leaky ReLU or Snake, nearest x2 upsample) and its weights as bf16, accumulates in fp32
in tensor memory and applies the epilogue (bias, accumulate, shortcut-and-scale, gelu) and the fused
AdaIN statistics in fp32. The reference below rounds the same prologue values to bf16 and
convolves in float64, so the remaining differences are fp32 accumulation order and rare one-ulp
bf16 flips where the kernel's fast sine (Snake) lands on the other side of a rounding boundary.
Tolerances: relative L2 error <= 2e-5 (1e-4 with Snake), max-abs error <= 2e-3 x rms of the
output (one flipped bf16 input moves an output by about |w| x 2^-8 x |x|), statistics within
1e-4 relative (sums) of the reference's sums of the kernel's own outputs.
"""
import zlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

IN_NOMASK, IN_MASK, IN_ADAIN_LEAKY, IN_ADAIN_SNAKE, IN_LEAKY_MASK = range(5)
OUT_STORE, OUT_ADD, OUT_PLUS, OUT_GELU = range(4)


def bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).to(torch.float32).numpy()


def layout(rng, n_items, lo, hi, gap=2):
    """Item of every row: [gap][item 0][gap][item 1]...[gap]; returns the row->item table."""
    tab = [-1] * gap
    for b in range(n_items):
        tab += [b] * int(rng.integers(lo, hi))
        tab += [-1] * gap
    return np.asarray(tab, np.int32)


def prologue(x_dom, items, mode, slope, coef, alpha):
    v = x_dom.astype(np.float32).copy()
    if mode == IN_NOMASK:
        return v
    keep = items >= 0
    b = np.where(keep, items, 0)
    if mode in (IN_ADAIN_LEAKY, IN_ADAIN_SNAKE):
        A = coef[b, :, 0].astype(np.float64)
        B = coef[b, :, 1].astype(np.float64)
        t = (v.astype(np.float64) * A + B).astype(np.float32)  # fmaf: one rounding
        if mode == IN_ADAIN_LEAKY:
            v = np.where(t < 0, t * np.float32(slope), t).astype(np.float32)
        else:
            al = alpha.astype(np.float32)
            sn = np.sin((al * t).astype(np.float32).astype(np.float64)).astype(np.float32)
            ia = (np.float32(1.0) / al).astype(np.float32)
            v = (ia.astype(np.float64) * (sn * sn).astype(np.float32).astype(np.float64) +
                 t.astype(np.float64)).astype(np.float32)
    elif mode == IN_LEAKY_MASK:
        v = np.where(v < 0, v * np.float32(slope), v).astype(np.float32)
    v[~keep] = 0.0
    return v


def gelu_new(a):
    a = a.astype(np.float64)
    return 0.5 * a * (1.0 + np.tanh(0.7978845608028654 * (a + 0.044715 * a ** 3)))


def reference(x, w, bias, items_in, rows_out, pad, dil, up2, in_mode, slope, out_mode, oscale, coef, alpha, sc, y0):
    cout, cin, K = w.shape
    rows_in = len(items_in)
    src = np.arange(rows_in) // 2 if up2 else np.arange(rows_in)
    xin = bf16(prologue(x[src, :cin], items_in, in_mode, slope, coef, alpha))
    xt = torch.from_numpy(xin.T[None].astype(np.float64))
    wt = torch.from_numpy(bf16(w).astype(np.float64))
    # explicit zero padding on both sides (the kernel reads zeros outside [0, rows_in))
    need = rows_out - 1 + (K - 1) * dil + 1
    xp = torch.zeros((1, cin, max(need, rows_in + pad)), dtype=torch.float64)
    xp[:, :, pad:pad + rows_in] = xt
    acc = torch.nn.functional.conv1d(xp[:, :, :need], wt, dilation=dil)[0].numpy().T  # [rows_out][cout]
    r = acc + (bias.astype(np.float64) if bias is not None else 0.0)
    if out_mode == OUT_ADD:
        r = y0[:, :cout].astype(np.float64) + r
    elif out_mode == OUT_PLUS:
        r = (r + sc[:, :cout].astype(np.float64)) * oscale
    elif out_mode == OUT_GELU:
        r = gelu_new(r)
    return r


CASES = [
    # name, cin, cout, K, dil, in_mode, out_mode, up2, stats, ldx_extra, ldy_extra
    ("snake_k3_store_stats", 128, 128, 3, 1, IN_ADAIN_SNAKE, OUT_STORE, 0, True, 0, 0),
    ("snake_k11_d5_plus_stats", 128, 128, 11, 5, IN_ADAIN_SNAKE, OUT_PLUS, 0, True, 0, 0),
    ("snake_k7_d3_add", 256, 256, 7, 3, IN_ADAIN_SNAKE, OUT_ADD, 0, False, 0, 0),
    ("linear_768_2304", 768, 2304, 1, 1, IN_NOMASK, OUT_STORE, 0, False, 0, 0),
    ("linear_768_2048_gelu", 768, 2048, 1, 1, IN_NOMASK, OUT_GELU, 0, False, 0, 0),
    ("adain_leaky_up2_514_1024_stats", 514, 1024, 3, 1, IN_ADAIN_LEAKY, OUT_STORE, 1, True, 2, 0),
    ("mask_1090_512_stats", 1090, 512, 3, 1, IN_MASK, OUT_STORE, 0, True, 2, 0),
    ("leaky_k7_128_22_padded_rows", 128, 22, 7, 1, IN_LEAKY_MASK, OUT_STORE, 0, False, 0, 6),
    ("mask_k1_22_128", 22, 128, 1, 1, IN_MASK, OUT_STORE, 0, False, 2, 0),
    ("k2_132_256", 132, 256, 2, 1, IN_NOMASK, OUT_STORE, 0, False, 0, 4),
]


@pytest.mark.parametrize("pre", [0, 1], ids=["fused", "pre"])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_tc_conv_matches_fp64_on_bf16_operands(kk, case, pre):
    import kokoro_rust_b200.engine as E
    name, cin, cout, K, dil, in_mode, out_mode, up2, stats, ldx_extra, ldy_extra = case
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    n_items = 4
    items_in = layout(rng, n_items, 60, 260) if not up2 else np.repeat(layout(rng, n_items, 30, 130), 2)
    rows_in = len(items_in)
    rows_out = rows_in
    items_out = items_in
    pad = (K - 1) * dil // 2
    xrows = (rows_in + 1) // 2 if up2 else rows_in
    x = rng.standard_normal((xrows, cin + ldx_extra)).astype(np.float32)
    w = (rng.standard_normal((cout, cin, K)) / np.sqrt(cin * K)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(cout)).astype(np.float32)
    coef = np.stack([1.0 + 0.3 * rng.standard_normal((n_items, cin)), 0.2 * rng.standard_normal((n_items, cin))],
                    -1).astype(np.float32)
    alpha = (1.0 + 0.5 * rng.random(cin)).astype(np.float32)
    sc = rng.standard_normal((rows_out, cout + 4)).astype(np.float32) if out_mode == OUT_PLUS else None
    y0 = rng.standard_normal((rows_out, cout + ldy_extra)).astype(np.float32)
    oscale = float(1 / np.sqrt(2.0))
    res = E.conv_selftest(0, x=x, w=w, item_in=items_in, item_out=items_out, rows_out=rows_out, pad=pad, dil=dil,
                          up2=up2, in_mode=in_mode, slope=0.2, out_mode=out_mode, oscale=oscale, bias=bias,
                          coef=coef, alpha=alpha, sc=sc, y=y0.copy(), n_items=n_items, want_stats=stats, pre=pre)
    y, st = res if stats else (res, None)
    ref = reference(x, w, bias, items_in, rows_out, pad, dil, up2, in_mode, 0.2, out_mode, oscale, coef, alpha, sc,
                    y0)
    got = y[:, :cout].astype(np.float64)
    err = np.abs(got - ref)
    rms = np.sqrt(np.mean(ref ** 2))
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    tol_rel = 1e-4 if in_mode == IN_ADAIN_SNAKE else 2e-5
    assert rel <= tol_rel, (name, rel)
    assert err.max() <= 2e-3 * rms, (name, err.max(), rms)
    if ldy_extra:  # columns from cout rounded up to 16 bytes on are untouched (TMA writes 16-byte units)
        c16 = (cout + 3) // 4 * 4
        np.testing.assert_array_equal(y[:, c16:], y0[:, c16:])
    if stats:
        for b in range(n_items):
            rows = got[items_out == b]
            np.testing.assert_allclose(st[b, :, 0], rows.sum(0), rtol=1e-4, atol=1e-4 * np.abs(rows).sum(0).max())
            np.testing.assert_allclose(st[b, :, 1], (rows ** 2).sum(0), rtol=1e-4)


def test_tc_conv_rejects_unaligned_row_strides(kk):
    """Every operand moves by TMA, so row strides must be multiples of 16 bytes."""
    import kokoro_rust_b200.engine as E
    tab = np.zeros(300, np.int32)
    w = np.zeros((22, 64, 3), np.float32)
    with pytest.raises(E.KokoroError, match="not supported"):
        E.conv_selftest(0, x=np.zeros((300, 64), np.float32), w=w, item_in=tab, item_out=tab, rows_out=300, pad=1,
                        y=np.zeros((300, 22), np.float32))
    with pytest.raises(E.KokoroError, match="not supported"):
        E.conv_selftest(0, x=np.zeros((300, 66), np.float32), w=w, item_in=tab, item_out=tab, rows_out=300, pad=1,
                        y=np.zeros((300, 24), np.float32))


def test_tc_conv_rejects_tiny_row_counts(kk):
    import kokoro_rust_b200.engine as E
    x = np.zeros((32, 64), np.float32)
    w = np.zeros((64, 64, 3), np.float32)
    with pytest.raises(E.KokoroError, match="not supported"):
        E.conv_selftest(0, x=x, w=w, item_in=np.zeros(32, np.int32), item_out=np.zeros(32, np.int32), rows_out=32,
                        pad=1)
