"""Micro-benchmark of the tcgen05 convolution kernel on representative config-4 layer shapes, through
the diagnostics entry point kk_conv_selftest (one B200, synthetic inputs larger than L2).

    python kokoro-rust_b200/conv_bench.py [shape-substring ...]   # e.g. k11_128 k1_768

Environment: ITERS (timed launches per shape, default 10; 0 = one untimed launch, for profilers),
PRE (1 = the pre-transform route: prologue kernel + bf16 window planes, default 0 = fused
producers). Each line: device ms per launch (CUDA events), algorithmic TFLOP/s and GB/s, and the
fraction of the max(FLOPs / tensor peak, bytes / HBM peak) floor with the peaks of
MEASURED_PEAKS.json.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

# name, cin, cout, K, dil, in_mode, out_mode, stats, rows, item length range
SHAPES = [
    ("k3_128_snake_store_st", 128, 128, 3, 1, 3, 0, True, 1 << 20, (20000, 40000)),
    ("k11_128_snake_plus_st", 128, 128, 11, 1, 3, 2, True, 1 << 20, (20000, 40000)),
    ("k7_128_snake_add", 128, 128, 7, 1, 3, 1, False, 1 << 20, (20000, 40000)),
    ("k7_256_snake_store_st", 256, 256, 7, 1, 3, 0, True, 300000, (4000, 8000)),
    ("k3_256_snake_store_st", 256, 256, 3, 1, 3, 0, True, 300000, (4000, 8000)),
    ("k11_256_snake_plus_st", 256, 256, 11, 1, 3, 2, True, 300000, (4000, 8000)),
    ("k1_768_2304", 768, 2304, 1, 1, 0, 0, False, 34676, (60, 260)),
    ("k1_2048_768_plus", 2048, 768, 1, 1, 0, 2, False, 34676, (60, 260)),
    ("k3_1090_1024_mask_st", 1090, 1024, 3, 1, 1, 0, True, 69805, (100, 500)),
]


def load_engine():
    import importlib.util
    spec = importlib.util.spec_from_file_location("kokoro_rust_b200", os.path.join(HERE, "__init__.py"),
                                                  submodule_search_locations=[HERE])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["kokoro_rust_b200"] = mod
    spec.loader.exec_module(mod)
    return mod.engine


def main(argv):
    E = load_engine()
    iters = int(os.environ.get("ITERS", "10"))
    pre = int(os.environ.get("PRE", "0"))
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    P = (peaks.get("bf16_tflops_sustained") or 1381.3) * 1e12
    H = (peaks.get("hbm_gbs") or 6548.5) * 1e9
    rng = np.random.default_rng(0)
    for name, cin, cout, K, dil, im, om, st, rows, il in SHAPES:
        if argv and not any(o in name for o in argv):
            continue
        tab, b = [-1, -1], 0
        while len(tab) < rows:
            n = int(rng.integers(*il))
            tab += [b] * n + [-1, -1]
            b += 1
        tab = np.asarray(tab[:rows], np.int32)
        ldx = (cin + 3) // 4 * 4
        x = rng.standard_normal((rows, ldx), dtype=np.float32)
        w = (rng.standard_normal((cout, cin, K), dtype=np.float32) / np.sqrt(cin * K)).astype(np.float32)
        coef = np.stack([np.ones((b, cin)), np.zeros((b, cin))], -1).astype(np.float32)
        sc = rng.standard_normal((rows, cout), dtype=np.float32) if om == 2 else None
        out = E.conv_selftest(0, x=x, w=w, item_in=tab, item_out=tab, rows_out=rows, pad=(K - 1) * dil // 2,
                              dil=dil, in_mode=im, out_mode=om, bias=np.zeros(cout, np.float32), coef=coef,
                              alpha=np.ones(cin, np.float32), sc=sc, n_items=b, want_stats=st,
                              timing_iters=iters, pre=pre)
        if iters == 0:
            print(json.dumps({"shape": name, "launched": True}))
            continue
        ms = out[1]
        fl = 2.0 * rows * cin * cout * K
        by = 4.0 * (rows * cin + rows * cout * (2 if om in (1, 2) else 1)) + 2.0 * cin * cout * K
        floor = max(fl / P, by / H) * 1e3
        print(json.dumps({"shape": name, "route": "pre" if pre else "fused", "ms": round(ms, 4),
                          "TFLOPs": round(fl / ms / 1e9, 1), "GBs": round(by / ms / 1e6),
                          "floor_ms": round(floor, 4), "frac": round(floor / ms, 3)}))


if __name__ == "__main__":
    main(sys.argv[1:])
