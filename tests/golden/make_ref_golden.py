"""Generate tests/golden/ref_kernels.npz: outputs of the REFERENCE's CUDA kernels (kernels/kokoro.cu
compiled from source by oracle/build_ref.py) on seeded inputs, run on a B200. The CPU tests check
the oracle against these vectors (tests/test_oracle_golden.py).

Run on a GPU box from the repository root:  python tests/golden/make_ref_golden.py
Launch shapes follow the reference's host code (src/gpu.rs, src/gpu_batch.rs).
"""
import ctypes
import json
import os
import sys

import numpy as np
import torch
from cuda.bindings import driver as cu

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
CUBIN = os.path.join(ROOT, "oracle", "_ref", "kokoro_ref.cubin")
OUT = os.path.join(ROOT, "tests", "golden", "ref_kernels.npz")

P, I, L, F, D, U = ctypes.c_void_p, ctypes.c_int, ctypes.c_long, ctypes.c_float, ctypes.c_double, ctypes.c_ulonglong


def ck(r):
    err = r[0] if isinstance(r, tuple) else r
    if err != cu.CUresult.CUDA_SUCCESS:
        raise RuntimeError(str(err))
    return r[1] if isinstance(r, tuple) and len(r) > 1 else None


class Ref:
    def __init__(self):
        torch.zeros(1, device="cuda")  # primary context current on this thread
        data = open(CUBIN, "rb").read()
        self.mod = ck(cu.cuModuleLoadData(data))
        self.keep = []

    def fn(self, name):
        return ck(cu.cuModuleGetFunction(self.mod, name.encode()))

    def dev(self, a):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        self.keep.append(t)
        return t

    def launch(self, name, grid, block, args, smem=0, coop=False):
        vals = tuple(a.data_ptr() if isinstance(a, torch.Tensor) else a[0] for a in args)
        types = tuple(P if isinstance(a, torch.Tensor) else a[1] for a in args)
        f = self.fn(name)
        if smem > 48 * 1024:
            ck(cu.cuFuncSetAttribute(f, cu.CUfunction_attribute.CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, smem))
        if coop:
            ck(cu.cuLaunchCooperativeKernel(f, *grid, *block, smem, 0, (vals, types)))
        else:
            ck(cu.cuLaunchKernel(f, *grid, *block, smem, 0, (vals, types), 0))
        torch.cuda.synchronize()


def cfg1(n):
    return ((n + 255) // 256, 1, 1), (256, 1, 1)


def splitmix_at(seed, ctr):
    m = (1 << 64) - 1
    x = (seed + (ctr + 1) * 0x9E3779B97F4A7C15) & m
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & m
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & m
    return x ^ (x >> 31)


def main():
    r = Ref()
    rng = np.random.default_rng(2024)
    g = {}
    tw = np.zeros(440)
    for k in range(11):
        for n in range(20):
            a = 2.0 * np.pi * ((k * n) % 20) / 20.0
            tw[k * 20 + n], tw[220 + k * 20 + n] = np.cos(a), np.sin(a)
    win = (0.5 - 0.5 * np.cos(2.0 * np.pi * np.arange(20) / 20.0)).astype(np.float32)
    tw_d, win_d = r.dev(tw), r.dev(win)

    # ---- A. harmonic source: gen_noise, sine_phase_pre, sine_har_source, stft20_ld
    Lc = 20
    S, Dn = 300 * Lc, Lc
    f0 = np.exp(rng.uniform(np.log(80), np.log(400), Lc)).astype(np.float32)
    f0[5:9] = 0.0
    f0[12] = -30.0
    lw = rng.uniform(-1, 1, 9).astype(np.float32)
    lb = np.float32(rng.uniform(-0.2, 0.2))
    seed = 12345
    rand_ini = np.array([(splitmix_at(seed, h) >> 40) * (1.0 / 16777216.0) for h in range(9)], np.float32)
    noise = r.dev(np.zeros(S * 9, np.float32))
    nn = S * 9
    r.launch("gen_noise", *cfg1(nn // 2 + 1), [(seed, U), noise, (nn, L)])
    f0_d = r.dev(f0)
    pp = r.dev(np.zeros(9 * Dn, np.float32))
    near = np.float32(1.0 / 300.0)
    down = np.float32(1.0 / (1.0 / 300.0))
    r.launch("sine_phase_pre", (1, 1, 1), (32, 1, 1),
             [f0_d, (Lc, I), (S, I), (Dn, I), (float(near), F), (float(down), F), r.dev(rand_ini), pp])
    har = r.dev(np.zeros(S, np.float32))
    r.launch("sine_har_source", *cfg1(S), [f0_d, (Lc, I), (S, I), (Dn, I), (float(near), F), (float(near), F), pp,
                                           noise, r.dev(lw), (float(lb), F), har])
    Fr = 1 + S // 5
    spec = r.dev(np.zeros(22 * Fr, np.float32))
    r.launch("stft20_ld", *cfg1(Fr), [har, (S, I), spec, (Fr, I), (Fr, I), tw_d, win_d])
    g.update(src_f0=f0, src_lw=lw, src_lb=np.array([lb]), src_seed=np.array([seed], np.uint64),
             src_noise=noise.cpu().numpy(), src_pp=pp.cpu().numpy().reshape(9, Dn), src_har=har.cpu().numpy(),
             src_spec=spec.cpu().numpy().reshape(22, Fr))

    # ---- B. iSTFT: istft_frames_ld + istft_ola
    Fi = 241
    post = (rng.standard_normal((22, Fi)) * 0.5).astype(np.float32)
    fr = r.dev(np.zeros(Fi * 20, np.float64))
    r.launch("istft_frames_ld", *cfg1(Fi), [r.dev(post), (Fi, I), (Fi, I), fr, tw_d, win_d])
    ln_ = 5 * (Fi - 1)
    aud = r.dev(np.zeros(ln_, np.float32))
    r.launch("istft_ola", *cfg1(ln_), [fr, (Fi, I), aud, (ln_, I), win_d])
    g.update(istft_post=post, istft_audio=aud.cpu().numpy())

    # ---- C. AdaIN statistics + apply over two segments of a gap-separated layout
    C, Lx = 16, 100
    starts, lens = np.array([0, 45], np.int32), np.array([40, 50], np.int32)
    x = (rng.standard_normal((C, Lx)) * 2 + 1).astype(np.float32)
    col = np.full(Lx, -1, np.int32)
    for b in range(2):
        col[starts[b]:starts[b] + lens[b]] = b
    mean, rstd = r.dev(np.zeros(2 * C, np.float32)), r.dev(np.zeros(2 * C, np.float32))
    x_d = r.dev(x)
    r.launch("chan_stats_seg", (C, 2, 1), (256, 1, 1),
             [x_d, (Lx, I), r.dev(starts), r.dev(lens), (1e-5, F), mean, rstd, (C, I)])
    gb = (rng.standard_normal((2, 2 * C)) * 0.3).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, C).astype(np.float32)
    nb = (rng.standard_normal(C) * 0.1).astype(np.float32)
    y = r.dev(np.zeros(C * Lx, np.float32))
    r.launch("adain_apply_seg", *cfg1(C * Lx), [x_d, y, r.dev(col), mean, rstd, r.dev(nw), r.dev(nb), r.dev(gb),
                                                (C, I), (Lx, I), (0.2, F)])
    g.update(adain_x=x, adain_starts=starts, adain_lens=lens, adain_gb=gb, adain_nw=nw, adain_nb=nb,
             adain_mean=mean.cpu().numpy().reshape(2, C), adain_rstd=rstd.cpu().numpy().reshape(2, C),
             adain_y=y.cpu().numpy().reshape(C, Lx))

    # ---- D. batched BiLSTM recurrence (cooperative launch, grid (H, 2) x 128)
    H, B = 32, 2
    ls, ss = np.array([7, 5], np.int32), np.array([0, 9], np.int32)
    rows = 16
    gxf = rng.standard_normal((rows, 4 * H)).astype(np.float32)
    gxb = rng.standard_normal((rows, 4 * H)).astype(np.float32)
    whf = (rng.uniform(-1, 1, (4 * H, H)) / np.sqrt(H)).astype(np.float32)
    whb = (rng.uniform(-1, 1, (4 * H, H)) / np.sqrt(H)).astype(np.float32)
    bhf = (rng.uniform(-1, 1, 4 * H) / np.sqrt(H)).astype(np.float32)
    bhb = (rng.uniform(-1, 1, 4 * H) / np.sqrt(H)).astype(np.float32)
    hbuf = r.dev(np.zeros(2 * B * 2 * H, np.float32))
    cst = r.dev(np.zeros(B * 2 * H, np.float32))
    out = r.dev(np.zeros(rows * 2 * H, np.float32))
    r.launch("lstm_seq_batched", (H, 2, 1), (128, 1, 1),
             [r.dev(gxf), r.dev(gxb), r.dev(whf), r.dev(whb), r.dev(bhf), r.dev(bhb), hbuf, cst, out, r.dev(ss),
              r.dev(ls), (B, I), (int(ls.max()), I), (H, I)], coop=True)
    g.update(lstm_gxf=gxf, lstm_gxb=gxb, lstm_whf=whf, lstm_whb=whb, lstm_bhf=bhf, lstm_bhb=bhb, lstm_starts=ss,
             lstm_lens=ls, lstm_out=out.cpu().numpy().reshape(rows, 2 * H))

    # ---- E. row LayerNorm (eps 1e-12), gelu_new, softmax_rows
    xl = (rng.standard_normal((3, 768)) * 3 + 1).astype(np.float32)
    gl = rng.uniform(0.5, 1.5, 768).astype(np.float32)
    bl = (rng.standard_normal(768) * 0.1).astype(np.float32)
    xl_d = r.dev(xl)
    r.launch("layer_norm_rows", (3, 1, 1), (256, 1, 1), [xl_d, r.dev(gl), r.dev(bl), (0, P), (3, I), (768, I),
                                                          (1e-12, F)])
    xg = (rng.standard_normal(1000) * 3).astype(np.float32)
    xg_d = r.dev(xg)
    r.launch("gelu_new", *cfg1(1000), [xg_d, (1000, L)])
    xs = (rng.standard_normal((4, 300)) * 4).astype(np.float32)
    xs_d = r.dev(xs)
    r.launch("softmax_rows", (4, 1, 1), (256, 1, 1), [xs_d, (300, I), (0.125, F)])
    g.update(ln_x=xl, ln_g=gl, ln_b=bl, ln_y=xl_d.cpu().numpy(), gelu_x=xg, gelu_y=xg_d.cpu().numpy(),
             softmax_x=xs, softmax_y=xs_d.cpu().numpy())

    # ---- F. strided conv (noise_convs.0 shape: 22 -> 64 here, k12 s6 p3), weights [Cin][K][Cout]
    Ci, Tc, Co, Kc, st, pd = 22, 361, 64, 12, 6, 3
    xc = rng.standard_normal((Ci, Tc)).astype(np.float32)
    wc = (rng.standard_normal((Co, Ci, Kc)) / np.sqrt(Ci * Kc)).astype(np.float32)
    bc = (rng.standard_normal(Co) * 0.1).astype(np.float32)
    To = (Tc + 2 * pd - Kc) // st + 1
    yc = r.dev(np.zeros(Co * To, np.float32))
    xw = 127 * st + (Kc - 1) + 1
    smem = (4 * xw + 4 * Kc * 64) * 4
    r.launch("conv1d_strided", ((To + 127) // 128, (Co + 63) // 64, 1), (128, 1, 1),
             [r.dev(xc), r.dev(np.ascontiguousarray(wc.transpose(1, 2, 0))), r.dev(bc), yc, (Ci, I), (Tc, I), (Co, I),
              (Kc, I), (1, I), (pd, I), (st, I), (To, I)], smem=smem)
    g.update(conv_x=xc, conv_w=wc, conv_b=bc, conv_y=yc.cpu().numpy().reshape(Co, To))

    # ---- G. depthwise ConvTranspose1d k3 s2 p1 op1 (the AdainResBlk1d pool)
    Cd, Td = 8, 20
    xd = rng.standard_normal((Cd, Td)).astype(np.float32)
    wd = rng.standard_normal((Cd, 3)).astype(np.float32)
    bd = rng.standard_normal(Cd).astype(np.float32)
    yd = r.dev(np.zeros(Cd * 2 * Td, np.float32))
    r.launch("dw_convT_k3s2", *cfg1(Cd * 2 * Td), [r.dev(xd), r.dev(wd), r.dev(bd), yd, (Cd, I), (Td, I)])
    g.update(pool_x=xd, pool_w=wd, pool_b=bd, pool_y=yd.cpu().numpy().reshape(Cd, 2 * Td))

    np.savez_compressed(OUT, **g)
    meta = {"source": "reference kernels/kokoro.cu built by oracle/build_ref.py for sm_100a",
            "device": torch.cuda.get_device_name(0), "arrays": sorted(g)}
    json.dump(meta, open(OUT.replace(".npz", ".json"), "w"), indent=1)
    print("wrote", OUT, len(g), "arrays")


if __name__ == "__main__":
    main()
