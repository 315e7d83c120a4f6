"""Same-box kernel baseline: the reference's own tensor-core convolution against this engine's
tcgen05 convolution, on the generator shapes of config 2 (B = 32 items of 400 frames). MEASUREMENT
INFRASTRUCTURE ONLY: nothing of the product imports it.

The reference kernels are kernels/kokoro.cu compiled from source for sm_100a by oracle/build_ref.py
(oracle/_ref/kokoro_ref.cubin): `conv1d_wmma_bf16_snake` (AdaIN + Snake prologue, y = conv) and
`conv1d_wmma_bf16_snake_res` (y += conv), kernels/kokoro.cu:660-777, launched as the reference's host
code launches them (src/gpu.rs:455-488: grid ceil(T / 128) x ceil(Cout / 128), 256 threads,
shared memory = the [128 + (K - 1) dil][48] bf16 window rounded to 128 B + 8 KB). This engine's side
is the same convolution through kk_conv_selftest (input mode 3 = AdaIN + Snake with the gap mask,
output mode 0 = store / 1 = accumulate), which times repeated launches with CUDA events on its
stream. Both read f32 activations and write f32 outputs; the reference keeps them channel-major
[C][T], this engine time-major [T][C].

A small case first checks that the two kernels compute the same convolution (same weights, inputs
and AdaIN parameters; relative L2 difference of the outputs, both with bf16 operands).

Run on a GPU box from the repository root:
    python oracle/time_ref_conv.py --out ref_conv.json
    python oracle/time_ref_conv.py --single 3     # one launch of this engine's conv, for ncu
"""
import argparse
import ctypes
import importlib.util
import json
import os
import sys

import numpy as np
import torch
from cuda.bindings import driver as cu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUBIN = os.path.join(ROOT, "oracle", "_ref", "kokoro_ref.cubin")

P, I = ctypes.c_void_p, ctypes.c_int


def ck(r):
    err = r[0] if isinstance(r, tuple) else r
    if err != cu.CUresult.CUDA_SUCCESS:
        raise RuntimeError(str(err))
    return r[1] if isinstance(r, tuple) and len(r) > 1 else None


class RefConv:
    """The reference's fused bf16 WMMA convolution, launched from its cubin on torch's stream."""

    def __init__(self):
        torch.zeros(1, device="cuda")
        self.mod = ck(cu.cuModuleLoadData(open(CUBIN, "rb").read()))
        self.fns = {}

    def fn(self, name):
        if name not in self.fns:
            self.fns[name] = ck(cu.cuModuleGetFunction(self.mod, name.encode()))
        return self.fns[name]

    @staticmethod
    def layout_a(w):
        """torch-layout weights [Cout][Cin][K] -> the kernel's A layout [cot][slice][k][64][16] bf16
        (the arrangement bf16_layout_a writes, kernels/kokoro.cu:644-659)."""
        cout, cin, K = w.shape
        n_cot, ns = (cout + 63) // 64, (cin + 15) // 16
        wp = np.zeros((n_cot * 64, ns * 16, K), np.float32)
        wp[:cout, :cin] = w
        a = wp.reshape(n_cot, 64, ns, 16, K).transpose(0, 2, 4, 1, 3)  # cot, slice, k, row, col
        return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).cuda()

    def launch(self, res, x, wa, b, y, cin, T, cout, K, dil, pad, pro):
        name = "conv1d_wmma_bf16_snake_res" if res else "conv1d_wmma_bf16_snake"
        tw = 128 + (K - 1) * dil
        smem = (tw * 48 * 2 + 127) // 128 * 128 + 8 * 256 * 4
        f = self.fn(name)
        if smem > 48 * 1024:
            ck(cu.cuFuncSetAttribute(f, cu.CUfunction_attribute.CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                     smem))
        ptrs = [x, wa, b, y]
        vals = tuple(t.data_ptr() for t in ptrs) + (cin, T, cout, K, dil, pad) + tuple(t.data_ptr() for t in pro)
        types = (P,) * 4 + (I,) * 6 + (P,) * len(pro)
        stream = cu.CUstream(torch.cuda.current_stream().cuda_stream)
        ck(cu.cuLaunchKernel(f, (T + 127) // 128, (cout + 127) // 128, 1, 256, 1, 1, smem, stream, (vals, types), 0))


def item_table(n_items, rows_per_item, gap):
    t = np.full(n_items * (rows_per_item + gap), -1, np.int32)
    for b in range(n_items):
        t[b * (rows_per_item + gap): b * (rows_per_item + gap) + rows_per_item] = b
    return t


def adain_params(rng, n_items, C):
    """AdaIN + Snake parameters in the reference's form and folded to this engine's x * A + B."""
    mean = rng.standard_normal((n_items, C)).astype(np.float32) * 0.1
    rstd = (1.0 + rng.random((n_items, C))).astype(np.float32)
    gb = (rng.standard_normal((n_items, 2 * C)) * 0.1).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    nb = (0.1 * rng.standard_normal(C)).astype(np.float32)
    alpha = (0.5 + rng.random(C)).astype(np.float32)
    g1 = 1.0 + gb[:, :C].astype(np.float64)
    A = g1 * rstd * nw
    B = g1 * (nb - mean.astype(np.float64) * rstd * nw) + gb[:, C:]
    coef = np.stack([A, B], axis=-1).astype(np.float32)
    return dict(mean=mean, rstd=rstd, gb=gb, nw=nw, nb=nb, alpha=alpha, coef=coef)


def run_ref(rc, res, xd, w, bias, items, prm, K, dil, iters, warm, want_y=False):
    """xd: the input in the reference's layout [C][T] on the device; returns (y [T][Cout] or None,
    ms per launch)."""
    cin, T = xd.shape
    cout = w.shape[0]
    yd = torch.zeros((cout, T), dtype=torch.float32, device="cuda")
    wa = rc.layout_a(w)
    bd = torch.from_numpy(bias).cuda()
    pro = [torch.from_numpy(items).cuda()] + [torch.from_numpy(prm[k]).cuda()
                                              for k in ("mean", "rstd", "nw", "nb", "gb", "alpha")]
    pad = (K - 1) * dil // 2
    rc.launch(res, xd, wa, bd, yd, cin, T, cout, K, dil, pad, pro)
    torch.cuda.synchronize()
    y0 = yd.t().cpu().numpy().copy() if want_y else None
    for _ in range(warm):
        rc.launch(res, xd, wa, bd, yd, cin, T, cout, K, dil, pad, pro)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(iters):
        rc.launch(res, xd, wa, bd, yd, cin, T, cout, K, dil, pad, pro)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(iters, 1)
    del yd
    return y0, ms


def engine_module():
    """The package (directory kokoro-rust_b200) loaded under an importable name."""
    if "kokoro_rust_b200" not in sys.modules:
        pkg = os.path.join(ROOT, "kokoro-rust_b200")
        spec = importlib.util.spec_from_file_location("kokoro_rust_b200", os.path.join(pkg, "__init__.py"),
                                                      submodule_search_locations=[pkg])
        mod = importlib.util.module_from_spec(spec)
        sys.modules["kokoro_rust_b200"] = mod
        spec.loader.exec_module(mod)
    return sys.modules["kokoro_rust_b200"].engine


def run_ours(res, x_tm, w, bias, items, prm, K, dil, iters):
    eng = engine_module()
    T = x_tm.shape[0]
    out = eng.conv_selftest(0, x=x_tm, w=w, item_in=items, item_out=items, rows_out=T, pad=(K - 1) * dil // 2,
                            dil=dil, in_mode=3, out_mode=1 if res else 0, bias=bias, coef=prm["coef"],
                            alpha=prm["alpha"], n_items=int(items.max()) + 1, timing_iters=iters)
    return out if iters > 0 else (out, 0.0)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--out", default=None)
    ap.add_argument("--single", type=int, default=0, metavar="K",
                    help="only one launch of this engine's conv (128 channels, dilation 1, y = conv) on "
                         "8 items of 48,000 rows: the small case for an ncu capture")
    args = ap.parse_args()
    rng = np.random.default_rng(7)
    if args.single:
        C, K = 128, args.single
        items = item_table(8, 48000, 240)
        x = rng.standard_normal((len(items), C), dtype=np.float32)
        bias = (0.1 * rng.standard_normal(C)).astype(np.float32)
        prm = adain_params(rng, 8, C)
        w = (rng.standard_normal((C, C, K)) * 0.05).astype(np.float32)
        y, _ = run_ours(False, x, w, bias, items, prm, K, 1, 0)
        print(json.dumps({"case": "single", "K": K, "rows": len(items), "mean_abs_y": float(np.abs(y).mean())}))
        return
    rc = RefConv()
    lines = []

    # ---- agreement on a small ragged case (both kernels, one shape)
    C, K, dil = 128, 7, 3
    items = item_table(2, 1000, 96)
    x = rng.standard_normal((len(items), C)).astype(np.float32)
    w = (rng.standard_normal((C, C, K)) * 0.05).astype(np.float32)
    bias = (0.1 * rng.standard_normal(C)).astype(np.float32)
    prm = adain_params(rng, 2, C)
    y_ref, _ = run_ref(rc, False, torch.from_numpy(x).cuda().t().contiguous(), w, bias, items, prm, K, dil, 0, 0,
                       want_y=True)
    y_our, _ = run_ours(False, x, w, bias, items, prm, K, dil, 0)
    rel = float(np.linalg.norm(y_our - y_ref) / np.linalg.norm(y_ref))
    check = {"case": "agreement", "C": C, "K": K, "dil": dil, "rows": len(items), "rel_l2": rel}
    print(json.dumps(check), flush=True)
    if not rel < 2e-2:
        raise SystemExit(f"the two convolutions disagree: relative L2 {rel}")

    # ---- config-2 generator shapes: 32 items x 400 frames, 2-frame gaps
    stages = [("stage0 (20N rows, 256 ch)", 256, item_table(32, 20 * 400, 20 * 2)),
              ("stage1 (120N rows, 128 ch)", 128, item_table(32, 120 * 400, 120 * 2))]
    rows = []
    for sname, C, items in stages:
        T = len(items)
        x = rng.standard_normal((T, C), dtype=np.float32)
        xd = torch.from_numpy(x).cuda().t().contiguous()
        bias = (0.1 * rng.standard_normal(C)).astype(np.float32)
        prm = adain_params(rng, 32, C)
        for K in (3, 7, 11):
            w = (rng.standard_normal((C, C, K)) * 0.05).astype(np.float32)
            for dil, res in ((1, False), (3, False), (5, False), (1, True)):
                flops = 2.0 * K * C * C * T
                _, ms_r = run_ref(rc, res, xd, w, bias, items, prm, K, dil, args.iters, args.warmup)
                _, ms_o = run_ours(res, x, w, bias, items, prm, K, dil, args.iters)
                r = {"stage": sname, "C": C, "rows": T, "K": K, "dil": dil, "residual": res,
                     "ref_ms": ms_r, "ours_ms": ms_o, "ref_tflops": flops / ms_r / 1e9,
                     "ours_tflops": flops / ms_o / 1e9, "speedup": ms_r / ms_o}
                rows.append(r)
                print(json.dumps(r), flush=True)
        del xd
    tot_r = sum(r["ref_ms"] for r in rows)
    tot_o = sum(r["ours_ms"] for r in rows)
    summary = {"case": "summary", "shapes": len(rows), "ref_ms_total": tot_r, "ours_ms_total": tot_o,
               "speedup": tot_r / tot_o, "gpu": torch.cuda.get_device_name(0)}
    print(json.dumps(summary), flush=True)
    if args.out:
        with open(args.out, "w") as f:
            json.dump({"agreement": check, "rows": rows, "summary": summary}, f, indent=1)


if __name__ == "__main__":
    main()
