"""Benchmark of the batched ragged Kokoro-82M forward on B200 (driver contract).

A step is one pass of the hot path over one batch of synthetic input. Default workload (N = 1):
the full ragged forward over 251 synthetic lines (token lengths lognormal,
median 110, sigma 0.6, clamped to [8, 510]; ids uniform in [1, 177]; one style per file;
model-predicted durations). Under torchrun (weak scaling) the job is 251 x N lines of the same
distribution, sharded across the ranks longest-processing-time first (``shard.shard_lpt``, cost =
tokens), so every rank runs about 251 lines of equal token count; there is no collective on the hot
path (the process group carries only the barrier, the max-over-ranks timing and the per-rank
report). ``--workload config5`` is the book-scale job: 20,000 lines built once, LPT-sharded across
the ranks, each rank's share bin-packed into ragged batches by ``plan_batches`` under the free-VRAM
budget (``BatchPolicy.from_free_vram``); a step is the rank's whole share. ``--workload config2``
times the vocoder-only op (decoder + generator, B = 32, T = 400); ``--workload config3`` runs the
full forward on the text-side configuration (256 sequences, lengths uniform in [16, 510]) and adds
``text_side``: tokens/s and TFLOP/s of the ALBERT, duration and text-encoder stages, from the
profiled step's stage boundaries (``stage_ms``).

Metric: audio-seconds per wall-second (audio-s = samples / 24000), whole job. ``value`` uses
device-resident inputs with the audio left on the device, timed by CUDA events on the engine's
stream (max over ranks). ``e2e`` is the host wall clock (``time.perf_counter``) around the public
API call a user makes, ``forward_batch(items, fetch=True)``: Python packing, validation, the
host-to-device copies, the forward and the audio read-back into numpy arrays, max over ranks.
``per_rank`` reports every rank's device time, audio, clock and stage times, including
``frame layout``: the device time from the end of the duration stage to the frame-layout tables
being on the device (durations read-back, host layout build, upload).

``--impl reference`` times the reference's CPU path. The reference crate has no CPU forward of
its own ("there is no CPU mode", docs/USAGE.md:100) and its Rust toolchain is absent here, so the
reference arm is the CPU restatement of its algorithm (oracle/kokoro_oracle.py) on the host
cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "kokoro-rust_b200")


def import_package():
    if "kokoro_rust_b200" in sys.modules:
        return sys.modules["kokoro_rust_b200"]
    spec = importlib.util.spec_from_file_location("kokoro_rust_b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["kokoro_rust_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


# ------------------------------------------------------------------------------ workloads

def config4_lines(seed: int, n_lines: int = 251):
    """251 synthetic lines: lognormal token lengths (median 110, sigma 0.6) clamped to [8, 510],
    ids uniform in [1, 177], one style vector per file (N(0, 0.1^2))."""
    rng = np.random.default_rng(seed)
    lens = np.clip(np.rint(np.exp(np.log(110.0) + 0.6 * rng.standard_normal(n_lines))), 8, 510).astype(int)
    toks = [rng.integers(1, 178, n) for n in lens]
    style = (rng.standard_normal(256) * 0.1).astype(np.float32)
    return toks, style


def rank_shard(toks, world: int, rank: int):
    """This rank's share of the lines: longest-processing-time-first over token counts
    (``shard.shard_lpt``), line indices ascending."""
    kk = import_package()
    return kk.shard.shard_lpt([len(t) for t in toks], world)[rank]


def config3_lines(seed: int, n_lines: int = 256):
    """The text-side configuration: 256 sequences with token lengths uniform in [16, 510], ids
    uniform in [1, 177], one style vector (N(0, 0.1^2))."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(16, 511, n_lines)
    toks = [rng.integers(1, 178, n) for n in lens]
    style = (rng.standard_normal(256) * 0.1).astype(np.float32)
    return toks, style


# Text-side FLOPs per token from the layer shapes: ALBERT (embedding projection + 12 layers of QKV,
# attention output and FFN GEMMs) 132.3 M, its attention 36,864 * T (QK^T and PV, 12 layers, T =
# the sequence's length), text encoder (3 convs k 5 + BiLSTM) 11.0 M, duration side (bert_encoder,
# 3 AdaLN + BiLSTM layers, predictor LSTM, logits) 15.5 M.
TEXT_FLOP_PER_TOKEN = 132.3e6 + 11.0e6 + 15.5e6
ATTN_FLOP_PER_TOKEN_PER_T = 36864.0
TEXT_STAGES = ("stage:albert", "stage:durations", "stage:text encoder")
PROF_STEPS = 3  # profiled steps (per-launch CUDA events) after the timed ones, averaged per class


def config2_inputs(seed: int, B: int = 32, T: int = 400):
    """Vocoder-only inputs: asr N(0,1) [B][T][512]; F0 log-uniform 80-400 Hz with 20% of frames
    zeroed in contiguous runs; N N(0,1); style N(0, 0.1^2)."""
    rng = np.random.default_rng(seed)
    asr = [rng.standard_normal((T, 512)).astype(np.float32) for _ in range(B)]
    f0s, ns = [], []
    for _ in range(B):
        f0 = np.exp(rng.uniform(np.log(80), np.log(400), 2 * T)).astype(np.float32)
        zero = int(0.2 * 2 * T)
        left = zero
        while left > 0:  # a few contiguous unvoiced runs
            run = min(left, int(rng.integers(10, 60)))
            s = int(rng.integers(0, 2 * T - run))
            f0[s:s + run] = 0.0
            left -= run
        f0s.append(f0)
        ns.append(rng.standard_normal(2 * T).astype(np.float32))
    s_dec = (rng.standard_normal((B, 128)) * 0.1).astype(np.float32)
    return asr, f0s, ns, s_dec


# ------------------------------------------------------------------------------ clocks

CLOCK_Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
           "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
           "clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = tempfile.mktemp(prefix="kk_clocks_", suffix=".csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={CLOCK_Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 9:
                    rows.append(p)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------ CPU (oracle) leg

def cpu_sample_lines(toks, n: int):
    """A bounded sample of the workload: n lines of median length (the CPU path is ~2000x
    slower, so the sample keeps the default run within minutes)."""
    order = np.argsort([len(t) for t in toks])
    mid = len(order) // 2
    return [toks[i] for i in order[mid - n // 2: mid - n // 2 + n]]


def load_oracle(ckpt: str, threads: int):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch
    import kokoro_oracle as ko
    kk = import_package()
    torch.set_num_threads(threads)
    return ko, ko.KokoroOracle(kk.weights.load_safetensors(ckpt), threads=threads)


def time_oracle(ckpt: str, lines, style, threads: int):
    """Seconds of audio and wall seconds of the CPU restatement on the given lines."""
    kk = import_package()
    _ko, o = load_oracle(ckpt, threads)
    audio_s = 0.0
    t0 = time.perf_counter()
    for i, t in enumerate(lines):
        ids = np.concatenate([[0], t, [0]])
        out = o.forward(ids, style, 1.0, seed=kk.mix_seed(0, i))
        audio_s += out["audio"].shape[0] / 24000.0
    return audio_s, time.perf_counter() - t0


def time_oracle_configs(ckpt: str, threads: int):
    """The CPU restatement on BASELINE configs 1 and 2: config 1 whole (one utterance, 64 ids from
    default_rng(0), durations forced to [0, 3 x 64, 0]: 4.8 audio-s), config 2 on a bounded sample
    (2 of its 32 items of T = 400 frames: 20 audio-s)."""
    import torch
    ko, o = load_oracle(ckpt, threads)
    rng = np.random.default_rng(0)
    ids = np.concatenate([[0], rng.integers(1, 178, 64), [0]])
    ref_s = (rng.standard_normal(256) * 0.1).astype(np.float32)
    dur = np.array([0] + [3] * 64 + [0])
    t0 = time.perf_counter()
    a1 = o.forward(ids, ref_s, 1.0, seed=0, forced_dur=dur)["audio"].shape[0] / 24000.0
    t1 = time.perf_counter() - t0
    asr, f0s, ns, s_dec = config2_inputs(seed=2000, B=2, T=400)
    t0 = time.perf_counter()
    a2 = 0.0
    for b in range(2):
        a2 += o.decode(torch.from_numpy(asr[b].T.copy()), f0s[b], ns[b], torch.from_numpy(s_dec[b]),
                       ko.counter_noise(b, 600 * 400 * 9)).shape[0] / 24000.0
    t2 = time.perf_counter() - t0
    return {"config1": {"value": a1 / t1, "unit": "audio-s/s", "cores": threads, "kind": "port",
                        "sample": f"config 1 whole: 1 utterance, 192 frames, fp32 ({a1:.1f} audio-s in {t1:.2f} s)"},
            "config2": {"value": a2 / t2, "unit": "audio-s/s", "cores": threads, "kind": "port",
                        "sample": f"config 2, 2 of 32 items of T=400, decoder + generator ({a2:.1f} audio-s in "
                                  f"{t2:.2f} s)"}}


def traffic_ratio():
    """DRAM bytes over algorithmic bytes of the tcgen05 conv class, from the committed small-case ncu
    capture (one kernel, a few launches; profiles/tc_conv_kernel_dram_small_case.md), or None."""
    try:
        for ln in open(os.path.join(ROOT, "profiles", "tc_conv_kernel_dram_small_case.md")):
            if ln.startswith("dram_over_algorithmic:"):
                return float(ln.split(":")[1])
    except (OSError, ValueError):
        pass
    return None


# ------------------------------------------------------------------------------ conv kernel micro-benchmark

# Representative generator / decoder / ALBERT layer shapes of config 4 for ``--workload conv``:
# name, cin, cout, K, dil, in_mode (0 as is, 1 gap mask, 3 AdaIN + Snake), out_mode (0 store,
# 1 add, 2 shortcut), fused AdaIN statistics, rows, item length range (rows)
CONV_SHAPES = [
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


def conv_bench(shapes, iters: int, pre: int):
    """The tcgen05 convolution alone on the layer shapes above, through kk_conv_selftest (one B200,
    synthetic inputs larger than L2): one JSON line per shape with the device ms per launch (CUDA
    events), algorithmic TFLOP/s and GB/s, and the fraction of the max(FLOPs / tensor peak, bytes /
    HBM peak) floor. iters = 0 launches each shape once, untimed (for profilers)."""
    E = import_package().engine
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    P = (peaks.get("bf16_tflops_sustained") or 1381.3) * 1e12
    H = (peaks.get("hbm_gbs") or 6548.5) * 1e9
    rng = np.random.default_rng(0)
    for name, cin, cout, K, dil, im, om, st, rows, il in CONV_SHAPES:
        if shapes and not any(o in name for o in shapes):
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


# ------------------------------------------------------------------------------ main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config4", choices=["config4", "config3", "config2", "config5", "conv"])
    ap.add_argument("--precision", default=os.environ.get("KK_PRECISION", "bf16"), choices=["bf16", "fp32"])
    ap.add_argument("--cpu-lines", type=int, default=3, help="lines in the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--launch-log", default=None, help="write every profiled launch (class, ms, FLOPs, bytes) of the PROF_STEPS profiled steps as CSV")
    ap.add_argument("--items", type=int, default=32, help="config2: utterances per batch")
    ap.add_argument("--frames", type=int, default=400, help="config2: frames per utterance")
    ap.add_argument("--lines", type=int, default=20000, help="config5: lines of the book")
    ap.add_argument("--conv-shapes", nargs="*", default=[], help="conv: shape-name substrings (default all)")
    ap.add_argument("--conv-iters", type=int, default=10, help="conv: timed launches per shape (0: one, untimed)")
    ap.add_argument("--conv-pre", type=int, default=0, help="conv: 1 = the pre-transform route")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload == "conv":  # kernel micro-benchmark, not the contract line
        conv_bench(args.conv_shapes, args.conv_iters, args.conv_pre)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    # the library's host-side audio fetch uses up to 16 threads: share the host's cores among the
    # ranks of this node
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
    os.environ.setdefault("KK_FETCH_THREADS", str(max(1, min(16, (os.cpu_count() or 8) // max(1, local_world)))))
    kk = import_package()

    ckpt_dir = os.environ.get("KK_CKPT_DIR", tempfile.gettempdir())
    ckpt = os.path.join(ckpt_dir, "kokoro_b200_seed0.safetensors")

    if args.impl == "reference":
        if rank != 0:
            return
        kk.weights.write_random_checkpoint(ckpt, 0)
        toks, style = config4_lines(seed=1000)
        threads = os.cpu_count() or 1
        lines = cpu_sample_lines(toks, 1)
        for _ in range(args.warmup):
            time_oracle(ckpt, lines, style, threads)
        tot_a = tot_t = 0.0
        for _ in range(args.steps):
            a, t = time_oracle(ckpt, lines, style, threads)
            tot_a += a
            tot_t += t
        v = tot_a / tot_t
        print(json.dumps({
            "impl": "reference", "metric": "audio-sec per wall-sec (full ragged forward)", "value": v,
            "unit": "audio-s/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000 * tot_t / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config4 sample: 1 median-length line per step (CPU restatement, oracle/)"},
            "cpu_baseline": {"value": v, "unit": "audio-s/s", "cores": threads, "kind": "port",
                             "sample": "1 median-length line of config 4 per step"},
            "e2e": {"value": v, "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    if local_rank == 0:
        # one process per node writes the node's checkpoint file and brings the library up to date,
        # before the node's other ranks read or load them
        kk.weights.write_random_checkpoint(ckpt, 0)
        if world > 1:
            kk.engine.load_library()
    if world > 1:
        dist.barrier()
    eng = kk.GpuKokoro(ckpt, local_rank, args.precision)

    def barrier_sync():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    toks = None
    if args.workload in ("config4", "config3", "config5"):
        if args.workload == "config4":
            # 251 lines per rank: 251 x N lines built once, LPT-sharded by tokens (N = 1: all 251);
            # the style (one voice per file) is config 4's at every N, so the per-rank work does
            # not change with N (the generator draws the style after the lines)
            all_toks, _ = config4_lines(seed=1000, n_lines=251 * world)
            _, style = config4_lines(seed=1000)
            mine = rank_shard(all_toks, world, rank)
            workload_desc = ("config4: full ragged forward, 251 synthetic lines per rank (lognormal lengths median "
                             "110 sigma 0.6 clamped [8,510]; 251 x N lines LPT-sharded by tokens), predicted "
                             "durations, one batch per rank")
        elif args.workload == "config5":
            all_toks, style = config4_lines(seed=5000, n_lines=args.lines)
            mine = rank_shard(all_toks, world, rank)
            workload_desc = (f"config5: book-scale job, {args.lines} synthetic lines (config-4 length distribution) "
                             "LPT-sharded by tokens across the ranks, each rank's share in plan_batches ragged "
                             "batches under the free-VRAM budget; a step is the rank's whole share")
        else:
            all_toks, style = config3_lines(seed=3000 + rank)
            mine = list(range(len(all_toks)))
            workload_desc = ("config3: 256 sequences per rank, token lengths uniform in [16,510], full ragged "
                             "forward with predicted durations, one batch; text side reported from stage times")
        toks = [all_toks[i] for i in mine]
        items = [kk.BatchItem(np.concatenate([[0], all_toks[i], [0]]), style, 1.0,
                              kk.ItemNoise(seed=kk.mix_seed(0, i))) for i in mine]
        batches = [list(range(len(items)))]
        if args.workload == "config5":
            # calibrate the budget on one batch, then bin-pack the share (src/engine.rs:165-183)
            eng.forward_batch(items[:64], fetch=False)
            policy = kk.BatchPolicy.from_free_vram(eng)
            batches = kk.engine.plan_batches([len(it.ids) for it in items], policy)

        def step(fetch):
            """One pass over this rank's share: (audio-s, device ms)."""
            a = ms = 0.0
            for bi in batches:
                outs = eng.forward_batch([items[k] for k in bi], fetch=fetch)
                a += sum(o.audio.shape[0] for o in outs) / 24000.0
                ms += eng.last_times()["total_ms"]
            return a, ms
    else:
        asr, f0s, ns, s_dec = config2_inputs(seed=2000 + rank, B=args.items, T=args.frames)
        batches = [list(range(args.items))]

        def step(fetch):
            eng.decode_batch(asr, f0s, ns, s_dec, seeds=list(range(len(asr))), fetch=fetch)
            return sum(a.shape[0] for a in asr) * 600 / 24000.0, eng.last_times()["total_ms"]
        workload_desc = f"config2: vocoder-only (decoder + generator), B={args.items}, T={args.frames} frames"

    # ---- warm-up and the device-resident timed region (value)
    eng.set_option(kk.engine.KK_OPT_KEEP_AUDIO_ON_DEVICE, 1)
    for _ in range(args.warmup):
        step(False)
    barrier_sync()
    l0 = eng.launch_count()
    audio_s = 0.0
    dev_ms = 0.0
    with ClockSampler(local_rank) as clk:
        w0 = time.perf_counter()
        for _ in range(args.steps):
            a, ms = step(False)
            audio_s += a
            dev_ms += ms
        barrier_sync()
        wall = time.perf_counter() - w0
    launches = eng.launch_count() - l0
    clocks = clk.summary()
    # PROF_STEPS more steps with per-launch CUDA events (kernel classes, roofline), averaged so that
    # one step's power-cap clock swing does not set the figure; not part of `value`
    eng.set_option(kk.engine.KK_OPT_PROFILE, 1)
    eng.profile_reset()
    prof_ms = 0.0
    for _ in range(PROF_STEPS):
        prof_ms += step(False)[1] / PROF_STEPS
    prof = {k: (v[0] // PROF_STEPS, v[1] / PROF_STEPS, v[2] / PROF_STEPS) for k, v in eng.profile().items()}
    plog = eng.profile_launches()
    eng.set_option(kk.engine.KK_OPT_PROFILE, 0)
    barrier_sync()
    t = torch.tensor([dev_ms, audio_s], dtype=torch.float64, device=f"cuda:{local_rank}")
    if world > 1:
        tm = t.clone()
        dist.all_reduce(tm[0:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(tm[1:2], op=dist.ReduceOp.SUM)
        t = tm
    max_ms, total_audio = float(t[0]), float(t[1])
    ms_ = eng.memory_stats()
    mem = dict(ms_, bytes_per_frame=ms_["peak_bytes"] / max(ms_["frames"], 1),
               frames_per_token=ms_["frames"] / max(ms_["tokens"], 1))
    value = total_audio / (max_ms / 1000.0)

    # ---- end to end through the public API (host buffers in, numpy audio out), host wall clock
    eng.set_option(kk.engine.KK_OPT_KEEP_AUDIO_ON_DEVICE, 0)
    step(True)
    barrier_sync()
    e2e_s = 0.0
    e2e_audio = 0.0
    e2e_dev_ms = 0.0
    h2d = d2h = 0
    for _ in range(args.steps):
        w = time.perf_counter()
        a, ms = step(True)
        e2e_s += time.perf_counter() - w
        e2e_audio += a
        e2e_dev_ms += ms
        lt = eng.last_times()
        h2d, d2h = lt["h2d_bytes"], lt["d2h_bytes"]
    barrier_sync()
    te = torch.tensor([e2e_s, e2e_audio], dtype=torch.float64, device=f"cuda:{local_rank}")
    if world > 1:
        dist.all_reduce(te[0:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(te[1:2], op=dist.ReduceOp.SUM)
    e2e_value = float(te[1]) / float(te[0])

    # ---- per-rank report (after the timed regions; an object all-gather over the process group)
    stages = {k[len("stage:"):]: v[1] for k, v in prof.items() if k.startswith("stage:")}
    mine_rep = {"rank": rank, "device_ms": dev_ms, "audio_s": audio_s, "ms_per_step": dev_ms / args.steps,
                "lines": sum(len(b) for b in batches),
                "batches": len(batches), "tokens": int(sum(len(t) + 2 for t in toks)) if toks else None,
                "e2e_wall_s": e2e_s, "sm_mhz": clocks.get("sm_mhz"), "reasons": clocks.get("reasons"),
                "stage_ms": {k: round(v, 3) for k, v in stages.items()}}
    per_rank = [mine_rep]
    if world > 1:
        per_rank = [None] * world
        dist.all_gather_object(per_rank, mine_rep)

    if rank == 0:
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        except Exception:
            pass
        conv_cls = max((k for k in prof if k.startswith("conv")), key=lambda k: prof[k][1], default=None)
        roof = None
        if conv_cls:
            n_l, ms, fl = prof[conv_cls]
            achieved = fl / (ms / 1000.0) / 1e12
            peak = peaks.get("bf16_tflops_sustained") or 1381.3
            roof = {"bound": "tensor", "kernel": conv_cls, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "traffic": None, "launches": n_l, "avg_launch_ms": ms / max(n_l, 1),
                    "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained (kernel timed inside a long step)",
                    "share_of_step": ms / prof_ms}
            # per-launch floor max(FLOPs / tensor peak, algorithmic bytes / HBM peak): many of the
            # 128/256-channel k=3 layers move more bytes than their FLOPs can cover
            hbm = peaks.get("hbm_gbs") or 6650.0
            recs = [r for r in plog if r[0] == conv_cls]
            floor_ms = sum(max(r[2] / (peak * 1e12), r[3] / (hbm * 1e9)) * 1e3 for r in recs) / PROF_STEPS
            hbm_ms = sum(r[1] for r in recs if r[3] / (hbm * 1e9) > r[2] / (peak * 1e12)) / PROF_STEPS
            tot = sum(r[1] for r in recs) / PROF_STEPS
            alg_bytes = sum(r[3] for r in recs) / PROF_STEPS
            # DRAM bytes per launch: this run's algorithmic bytes per launch times the DRAM /
            # algorithmic ratio measured by ncu on a small case of the same kernel
            ratio = traffic_ratio()
            n_rec = max(len(recs) // PROF_STEPS, 1)
            if ratio is not None and recs:
                roof["traffic"] = ratio * alg_bytes / n_rec
                roof["traffic_source"] = ("algorithmic bytes per launch of this run x DRAM/algorithmic ratio "
                                          f"{ratio:.3f} from profiles/tc_conv_kernel_dram_small_case.md (ncu)")
            roof["algorithmic_bytes_per_launch"] = alg_bytes / n_rec
            roof["mixed_floor"] = {"floor_ms": floor_ms, "ms": tot, "frac": floor_ms / max(tot, 1e-9),
                                   "hbm_bound_time_share": hbm_ms / max(tot, 1e-9),
                                   "bytes": alg_bytes, "hbm_peak_gbs": hbm}
        if args.launch_log:
            with open(args.launch_log, "w") as f:
                f.write("class,ms,flops,bytes\n")
                for r in plog:
                    f.write(f"{r[0]},{r[1]:.6f},{r[2]:.6g},{r[3]:.6g}\n")
        cpu = cpu_cfg = None
        if not args.no_cpu_baseline and args.workload == "config4" and world == 1:  # N = 1 only
            threads = torch.get_num_threads()
            lines = cpu_sample_lines(toks, args.cpu_lines)
            a, tt = time_oracle(ckpt, lines, style, threads)
            cpu = {"value": a / tt, "unit": "audio-s/s", "cores": threads, "kind": "port",
                   "sample": f"{len(lines)} median-length lines of config 4 ({a:.1f} audio-s in {tt:.1f} s)"}
            cpu_cfg = time_oracle_configs(ckpt, threads)
        kprof = {k: v for k, v in prof.items() if not k.startswith("stage:")}
        text_side = None
        if args.workload == "config3":
            # rank 0's own shard, from the profiled step's stage boundaries
            n_tok = sum(len(t) + 2 for t in toks)
            fl = sum((len(t) + 2) * (TEXT_FLOP_PER_TOKEN + ATTN_FLOP_PER_TOKEN_PER_T * (len(t) + 2)) for t in toks)
            t_ms = sum(stages.get(s[len("stage:"):], 0.0) for s in TEXT_STAGES)
            text_side = {"tokens": n_tok, "stages": [s[len("stage:"):] for s in TEXT_STAGES], "ms": t_ms,
                         "tokens_per_s": n_tok / max(t_ms, 1e-9) * 1000.0, "tflop": fl / 1e12,
                         "tflops": fl / max(t_ms, 1e-9) / 1e9}
        res = {
            "metric": "audio-sec per wall-sec" + {"config4": " (full ragged forward)",
                                                  "config3": " (full ragged forward, text-side configuration)",
                                                  "config5": " (full ragged forward, book-scale job)",
                                                  "config2": " (vocoder-only decoder+generator)"}[args.workload],
            "value": value, "unit": "audio-s/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": max_ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if "tcgen05" in eng.identity else "f32", "data": "synthetic",
            "config": {"workload": workload_desc, "precision": args.precision, "engine": eng.identity,
                       "audio_s_per_step": total_audio / args.steps / world,
                       "l2": "inputs larger than L2: each step moves tens of GB of activations (L2 126 MB)",
                       "parallelism": f"dp{world} (LPT shards, no collectives)",
                       "wall_s_rank0": wall},
            "roofline": roof,
            "cpu_baseline": cpu,
            **({"cpu_baseline_configs": cpu_cfg} if cpu_cfg else {}),
            "e2e": {"value": e2e_value, "unit": "audio-s/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "timing": "host wall clock (time.perf_counter) around forward_batch(items, fetch=True), max over "
                              "ranks", "device_ms_per_step_rank0": e2e_dev_ms / args.steps,
                    "wall_ms_per_step_rank0": 1000.0 * e2e_s / args.steps},
            "gpu_launches": launches,
            "kernel_profile_steps": PROF_STEPS,
            "kernel_profile": {k: {"launches": v[0], "ms": v[1], "tflops": v[2] / max(v[1], 1e-9) / 1e9}
                               for k, v in kprof.items()},
            "stage_ms": stages,
            "clocks": clocks,
            "device_memory": mem,
            "per_rank": per_rank,
            **({"text_side": text_side} if text_side else {}),
        }
        print(json.dumps(res))
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
