"""The ``kokoro synth`` pipeline over this engine: a file of utterances, one per line, written as one
WAV (or one WAV per line), resumable line by line. Mirrors src/cli.rs:

* ``read_input`` (src/cli.rs:216-257): UTF-8 with BOM stripped, CRLF accepted, trailing newline
  ignored, input sha256 of the raw bytes;
* per-line validation (src/cli.rs:480-520): blank lines (an error unless ``--blank-lines skip``),
  control characters other than TAB (``invalid``), chunks over 510 phoneme characters
  (``oversize``, never truncated);
* three pipelined stages (src/cli.rs:450-718): prepare (resume check + validation) -> GPU synthesis
  (lines collected in a window, then length-bucketed ``Engine.synth_batch`` calls with per-chunk seeds
  ``mix_seed(seed, line << 16 | chunk)``) -> writer threads (WAV encode, sha256, atomic write, JSON
  sidecar per line), bounded queues between them;
* ``resume_ok`` (src/cli.rs:267-277): a line is skipped when its sidecar has the same line, text
  sha256 and configuration and its WAV still has the recorded sha256;
* ``whole_file_output`` (src/cli.rs:818-925): the per-line WAVs assembled in line order into
  ``<stem>.wav`` (``kk_wav_assemble``: sha256-checked parts, atomic rename), reused when the
  assembly key and the file's sha256 are unchanged;
* exit status 0 (every line done), 1 (some line failed), 2 (job-level error).

Scope: the text frontend (graphemes -> phonemes) is not part of this build, so the input is
phoneme strings (``--input-format phonemes``, mapped to ids with the model's config.json
vocabulary); conversion with an external ffmpeg (``--encode``) and the benchmark / timeline options
are left out.

    python kokoro-rust_b200/cli.py synth --model-dir DIR --voice af_heart lines.txt --out-dir out
"""
from __future__ import annotations

import argparse
import json
import os
import queue
import sys
import threading
import time
import unicodedata
from dataclasses import dataclass, field
from typing import List, Optional

if __name__ == "__main__" and not __package__:
    # run as a file (the package directory's name is not a Python identifier): load the package
    # from this directory and run its copy of this module
    import importlib.util

    _here = os.path.dirname(os.path.abspath(__file__))
    _spec = importlib.util.spec_from_file_location("kokoro_rust_b200", os.path.join(_here, "__init__.py"),
                                                   submodule_search_locations=[_here])
    _pkg = importlib.util.module_from_spec(_spec)
    sys.modules["kokoro_rust_b200"] = _pkg
    _spec.loader.exec_module(_pkg)
    from kokoro_rust_b200 import cli as _cli

    sys.exit(_cli.main())

from . import wav  # noqa: E402
from .engine import MAX_PHONEMES, SAMPLE_RATE, BatchPolicy, mix_seed  # noqa: E402

ENGINE_VERSION = "kokoro-b200 0.1"


class JobError(RuntimeError):
    """A job-level failure (exit status 2)."""


@dataclass
class InputFile:
    display: str
    stem: str
    sha256: str
    lines: List[str]
    bom_stripped: bool
    crlf_lines: int


def read_input(path: str) -> InputFile:
    raw = sys.stdin.buffer.read() if path == "-" else open(path, "rb").read()
    sha = wav.sha256_hex(raw)
    bom = raw.startswith(b"\xef\xbb\xbf")
    body = raw[3:] if bom else raw
    try:
        text = body.decode("utf-8")
    except UnicodeDecodeError as e:
        off = e.start
        line = body[:off].count(b"\n") + 1
        col = off - (body[:off].rfind(b"\n") + 1)
        raise JobError(f"input is not valid UTF-8: line {line}, byte {col + 1} of the line "
                       f"(file byte {off + 3 * bom}); nothing synthesized")
    lines, crlf = [], 0
    for ln in text.split("\n"):
        if ln.endswith("\r"):
            crlf += 1
            ln = ln[:-1]
        lines.append(ln)
    if lines and lines[-1] == "":
        lines.pop()
    stem = "stdin" if path == "-" else (os.path.splitext(os.path.basename(path))[0] or "input")
    return InputFile(path, stem, sha, lines, bom, crlf)


def control_char(text: str):
    """(1-based column, char) of the first control character other than TAB (src/cli.rs:261-263)."""
    for i, c in enumerate(text):
        if c != "\t" and unicodedata.category(c) == "Cc":
            return i + 1, c
    return None


def sha256_file(path: str) -> str:
    with open(path, "rb") as f:
        return wav.sha256_hex(f.read())


def write_atomic_json(path: str, obj, fsync: bool):
    wav.write_atomic(path, json.dumps(obj, indent=2, ensure_ascii=False).encode("utf-8"), sync=fsync)


def resume_ok(json_path: str, wav_path: str, line: int, text_sha: str, cfg: dict) -> bool:
    try:
        with open(json_path, "r", encoding="utf-8") as f:
            sc = json.load(f)
    except (OSError, ValueError):
        return False
    if sc.get("line") != line or sc.get("text_sha256") != text_sha or sc.get("config") != cfg:
        return False
    if sc.get("status") != "ok" or not sc.get("audio_sha256"):
        return False  # blank / failed lines are always re-evaluated
    try:
        return sha256_file(wav_path) == sc["audio_sha256"]
    except OSError:
        return False


@dataclass
class Job:
    kind: str                  # "resumed" | "final" | "synth"
    line: int
    sidecar: dict = field(default_factory=dict)
    chunks: List[str] = field(default_factory=list)
    entry: Optional[dict] = None
    t0: float = 0.0


def whole_file_output(inp: InputFile, out_dir: str, state_dir: str, entries: list, lines_ok: bool, fmt: wav.Format,
                      force: bool, fsync: bool, notes: list):
    final_wav = os.path.join(out_dir, f"{inp.stem}.wav")
    record_path = os.path.join(state_dir, "output.json")
    try:
        with open(record_path, "r", encoding="utf-8") as f:
            previous = json.load(f)
    except (OSError, ValueError):
        previous = {}

    def not_written(reason: str) -> dict:
        out = {"wav": None, "reason": reason}
        if os.path.exists(final_wav):
            notes.append(f"{final_wav} was NOT updated: the file there is from an earlier run and does not reflect "
                         "this input")
            out["stale_wav"] = {"path": os.path.basename(final_wav), "sha256": sha256_file(final_wav),
                                "note": f"from an earlier run; not updated because {reason}"}
        else:
            notes.append(f"{final_wav} was not written")
        return out

    if not lines_ok:
        return not_written("lines failed"), False
    done = [e for e in entries if e["status"] == "ok"]
    if not done:
        notes.append(f"nothing to synthesize: {inp.display} has no lines with text")
        return not_written("the input has no lines with text"), False
    parts = [(os.path.join(state_dir, e["wav"]), e["audio_sha256"]) for e in done]
    key = wav.sha256_hex("".join(f"{e['line']}:{e['audio_sha256']}\n" for e in done).encode())
    key = f"{fmt.name}:{key}"
    current = sha256_file(final_wav) if os.path.exists(final_wav) else None
    reuse = (not force and current is not None and previous.get("assembly_key") == key
             and previous.get("sha256") == current)
    if reuse:
        print(f"{final_wav} is up to date", file=sys.stderr)
        sha, samples = current, int(previous.get("samples", 0))
    else:
        try:
            a = wav.assemble(parts, fmt, SAMPLE_RATE, final_wav, sync=fsync)
        except wav.WavError as e:
            notes.append(f"could not write {final_wav}: {e}")
            out = not_written("writing the new file failed")
            out["error"] = str(e)
            return out, False
        print(f"wrote {final_wav} ({len(parts)} lines)", file=sys.stderr)
        sha, samples = a.sha256, a.samples
    record = {"wav": os.path.basename(final_wav), "sha256": sha, "assembly_key": key, "samples": samples,
              "duration_s": samples / SAMPLE_RATE, "format": fmt.name, "encoded": None}
    write_atomic_json(record_path, record, fsync)
    out = dict(record)
    out.update(lines=len(parts), sample_rate=SAMPLE_RATE, resumed=reuse)
    del out["assembly_key"]
    return out, True


def synth(args, engine=None) -> int:
    """Run the pipeline; engine (an ``Engine``, or a ``multi.MultiEngine`` with ``--cuda-devices``)
    is created from ``args.model_dir`` when not given."""
    if args.input_format != "phonemes":
        raise JobError("--input-format text needs the text frontend, which is not part of this build "
                       "(use --input-format phonemes)")
    t_load = time.time()
    if engine is not None:
        return _synth(args, engine, t_load)
    d = args.model_dir
    weights = os.path.join(d, "kokoro-v1_0.pth")
    if not os.path.exists(weights):
        st = sorted(f for f in os.listdir(d) if f.endswith(".safetensors"))
        if not st:
            raise JobError(f"{d} has neither kokoro-v1_0.pth nor a .safetensors checkpoint")
        weights = os.path.join(d, st[0])
    devices = [int(x) for x in args.cuda_devices.split(",")] if args.cuda_devices else [args.cuda_device]
    if len(devices) > 1:
        from .multi import MultiEngine
        with MultiEngine(weights, devices, args.precision, model_dir=d) as eng:
            return _synth(args, eng, t_load)
    from .engine import Engine
    return _synth(args, Engine(weights, devices[0], args.precision, model_dir=d), t_load)


def _synth(args, engine, t_load: float) -> int:
    fmt = {"pcm16": wav.Format.Pcm16, "float32": wav.Format.Float32}[args.format]
    inp = read_input(args.input)
    os.makedirs(args.out_dir, exist_ok=True)
    voice_sha = engine.voice(args.voice).sha256
    load_s = time.time() - t_load
    cfg = {"engine": f"{ENGINE_VERSION} [{engine.identity()}]", "model_sha256": engine.model_sha256,
           "config_sha256": engine.config_sha256, "voice": args.voice, "voice_sha256": voice_sha,
           "speed": args.speed, "seed": args.seed, "format": fmt.name, "input_format": "Phonemes",
           "frontend": "none (phoneme input)", "sample_rate": SAMPLE_RATE}
    state_dir = os.path.join(args.out_dir, ".kokoro", inp.stem)
    os.makedirs(state_dir, exist_ok=True)
    wav_dir = args.out_dir if args.per_line else state_dir
    width = max(5, len(str(max(len(inp.lines), 1))))

    def name(line: int, ext: str) -> str:
        return f"{inp.stem}_{line:0{width}d}.{ext}"

    synthesis = {"batch_phonemes": args.batch_phonemes, "batch_items": args.batch_items,
                 "batch_window": args.batch_window, "batch_first_window": args.batch_first_window}

    def new_sidecar(line: int, text: str, text_sha: str) -> dict:
        return {"line": line, "input_file": inp.display, "input_sha256": inp.sha256, "text": text,
                "text_sha256": text_sha, "status": "ok", "error": None, "graphemes": [], "phonemes": [],
                "dropped_phoneme_chars": [], "config": cfg, "synthesis": synthesis, "wav": None,
                "audio_sha256": None, "samples": 0, "duration_s": 0.0, "clipped_samples": 0, "encoded": None,
                "encoded_sha256": None, "elapsed_s": 0.0}

    depth = 8
    prep_q: "queue.Queue" = queue.Queue(depth)
    out_q: "queue.Queue" = queue.Queue(depth)
    failures: list = []
    stop = threading.Event()

    def make_job(i: int, text: str) -> Job:
        line = i + 1
        wav_path, json_path = os.path.join(wav_dir, name(line, "wav")), os.path.join(state_dir, name(line, "json"))
        text_sha = wav.sha256_hex(text.encode("utf-8"))
        if not args.force and resume_ok(json_path, wav_path, line, text_sha, cfg):
            with open(json_path, "r", encoding="utf-8") as f:
                sc = json.load(f)
            entry = {"line": line, "status": sc["status"], "resumed": True, "wav": sc["wav"],
                     "text_sha256": sc["text_sha256"], "audio_sha256": sc["audio_sha256"],
                     "duration_s": sc["duration_s"]}
            return Job("resumed", line, entry=entry)
        sc = new_sidecar(line, text, text_sha)
        t0 = time.time()
        try:
            if not text.strip():
                sc["status"] = "blank"
                if args.blank_lines == "error":
                    raise ValueError("blank line (canonical input has none; use --blank-lines skip to allow)")
                return Job("final", line, sc, t0=t0)
            cc = control_char(text)
            if cc:
                sc["status"] = "invalid"
                raise ValueError(f"control character U+{ord(cc[1]):04X} at character {cc[0]}")
            chunks = [text]  # phoneme input: the line is its own chunk
            sc["phonemes"] = chunks
            over = [c for c in chunks if len(c) > MAX_PHONEMES]
            if over:
                sc["status"] = "oversize"
                raise ValueError(f"chunk of {len(over[0])} phoneme chars exceeds {MAX_PHONEMES}; refusing to truncate")
            return Job("synth", line, sc, chunks, t0=t0)
        except ValueError as e:
            if sc["status"] == "ok":
                sc["status"] = "error"
            sc["error"] = str(e)
            return Job("final", line, sc, t0=t0)

    def prepare():
        try:
            for i, text in enumerate(inp.lines):
                if stop.is_set():
                    break
                prep_q.put(make_job(i, text))
        except Exception as e:  # noqa: BLE001 - reported as a job-level error
            failures.append(e)
        finally:
            prep_q.put(None)

    counts = {"ok": 0, "skip": 0, "bad": 0}
    audio_total = [0.0]
    entries: list = []
    lock = threading.Lock()

    def write_one(job: Job, audio):
        sc, line = job.sidecar, job.line
        wav_path, json_path = os.path.join(wav_dir, name(line, "wav")), os.path.join(state_dir, name(line, "json"))
        if audio is not None:
            enc = wav.encode(audio, SAMPLE_RATE, fmt)
            wav.write_atomic(wav_path, enc.bytes, sync=args.fsync)
            sc.update(wav=name(line, "wav"), audio_sha256=wav.sha256_hex(enc.bytes), samples=int(len(audio)),
                      duration_s=len(audio) / SAMPLE_RATE, clipped_samples=enc.clipped)
        elif os.path.exists(wav_path):
            os.remove(wav_path)
        sc["elapsed_s"] = time.time() - job.t0
        done = sc["status"] == "ok" or (sc["status"] == "blank" and args.blank_lines == "skip")
        write_atomic_json(json_path, sc, args.fsync)
        with lock:
            if done:
                counts["ok"] += 1
            else:
                counts["bad"] += 1
                print(f"line {line}: {sc['status']} - {sc['error'] or ''}", file=sys.stderr)
            audio_total[0] += sc["duration_s"]
            entries.append({"line": line, "status": sc["status"], "resumed": False, "wav": sc["wav"],
                            "text_sha256": sc["text_sha256"], "audio_sha256": sc["audio_sha256"],
                            "duration_s": sc["duration_s"], "error": sc["error"]})

    def writer():
        while True:
            msg = out_q.get()
            if msg is None:
                return
            job, audio = msg
            try:
                if job.kind == "resumed":
                    with lock:
                        counts["skip"] += 1
                        audio_total[0] += job.entry["duration_s"]
                        entries.append(job.entry)
                else:
                    write_one(job, audio)
            except Exception as e:  # noqa: BLE001
                failures.append(e)
                stop.set()

    t_all = time.time()
    prep_t = threading.Thread(target=prepare, daemon=True)
    writers = [threading.Thread(target=writer, daemon=True) for _ in range(max(1, args.write_threads))]
    prep_t.start()
    for w in writers:
        w.start()
    policy = BatchPolicy(max_phonemes=args.batch_phonemes, max_items=max(1, args.batch_items))
    pending: List[Job] = []
    n_pending = 0
    flushed_once = False

    def flush():
        reqs = [(c, mix_seed(args.seed, (job.line << 16) | k)) for job in pending for k, c in enumerate(job.chunks)]
        res = iter(engine.synth_batch(reqs, args.voice, args.speed, policy))
        for job in pending:
            audio, err = [], None
            for _ in job.chunks:
                r = next(res)
                if isinstance(r, Exception):
                    err = err or str(r)
                elif err is None:
                    job.sidecar["dropped_phoneme_chars"].extend(r.dropped)
                    audio.append(r.audio)
            if err is None:
                import numpy as np
                out_q.put((job, np.concatenate(audio) if len(audio) > 1 else audio[0]))
            else:
                job.sidecar.update(status="error", error=err)
                out_q.put((job, None))
        pending.clear()

    prep_done = False
    try:
        while True:
            job = prep_q.get()
            if job is None:
                prep_done = True
                break
            if stop.is_set():
                break
            if job.kind != "synth":
                out_q.put((job, None))
                continue
            pending.append(job)
            n_pending += len(job.chunks)
            window = args.batch_window if (flushed_once or args.batch_first_window == 0) else \
                min(args.batch_first_window, args.batch_window)
            if n_pending >= window:
                n_pending, flushed_once = 0, True
                flush()
        if pending and not stop.is_set():
            flush()
    except Exception as e:  # noqa: BLE001 - a failure of the GPU stage ends the job
        failures.append(e)
        stop.set()
    finally:
        for _ in writers:
            out_q.put(None)
        for w in writers:
            w.join()
        while not prep_done:  # let a stopped prepare stage finish its last put
            prep_done = prep_q.get() is None
        prep_t.join()
    if failures:
        raise JobError(f"pipeline failed: {failures[0]}")
    wall = time.time() - t_all
    entries.sort(key=lambda e: e["line"])
    complete = counts["bad"] == 0
    notes: list = []
    output = None
    if not args.per_line:
        output, ok = whole_file_output(inp, args.out_dir, state_dir, entries, complete, fmt, args.force, args.fsync,
                                       notes)
        complete = complete and ok
    mpath = os.path.join(args.out_dir, f"{inp.stem}.manifest.json")
    if args.diagnostics:
        manifest = {"input_file": inp.display, "input_sha256": inp.sha256, "input_lines": len(inp.lines),
                    "bom_stripped": inp.bom_stripped, "crlf_lines": inp.crlf_lines,
                    "blank_lines_policy": args.blank_lines.capitalize(),
                    "mode": "per-line" if args.per_line else "single WAV", "output": output,
                    "line_audio_dir": "." if args.per_line else f".kokoro/{inp.stem}",
                    "naming": f"{inp.stem}_<1-based line, width {width}>.wav / .json", "config": cfg,
                    "complete": complete,
                    "counts": {"done": counts["ok"], "resumed": counts["skip"], "failed": counts["bad"]},
                    "audio_s": audio_total[0], "load_s": load_s, "synth_wall_s": wall, "lines": entries}
        write_atomic_json(mpath, manifest, args.fsync)
    elif os.path.exists(mpath):  # a manifest of an earlier --diagnostics run no longer describes the files
        try:
            with open(mpath, "r", encoding="utf-8") as f:
                old = json.load(f)
            if "stale" not in old:
                old["stale"] = {"note": "written by an earlier run; a later run without --diagnostics did not "
                                        "update it", "complete_then": old.get("complete")}
                old["complete"] = False
                write_atomic_json(mpath, old, args.fsync)
                notes.append(f"{mpath} is from an earlier run; it is now marked as out of date")
        except (OSError, ValueError):
            pass
    rtf = wall / audio_total[0] if audio_total[0] > 0 else 0.0
    print(f"{len(inp.lines)} lines: {counts['ok']} done, {counts['skip']} resumed/skipped, {counts['bad']} failed; "
          f"{audio_total[0]:.1f}s audio in {wall:.2f}s (RTF {rtf:.4f})", file=sys.stderr)
    for n in notes:
        print(n, file=sys.stderr)
    if not complete:
        if counts["bad"]:
            print(f"INCOMPLETE: {counts['bad']} line(s) failed (listed above)", file=sys.stderr)
        return 1
    return 0


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="kokoro", description=__doc__.split("\n\n")[0])
    sub = p.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("synth", help="write a file of utterances (one per line) as WAV")
    s.add_argument("input", help='UTF-8 file, one utterance per line ("-" reads standard input)')
    s.add_argument("--model-dir", default=os.environ.get("KOKORO_MODEL_DIR"), required="KOKORO_MODEL_DIR" not in os.environ)
    s.add_argument("--voice", default="af_heart")
    s.add_argument("--speed", type=float, default=1.0)
    s.add_argument("--cuda-device", type=int, default=0)
    s.add_argument("--cuda-devices", default=None,
                   help="comma-separated CUDA ordinals: one engine process per GPU, each batch window "
                        "spread over them (longest first to the least-loaded GPU), results in line order")
    s.add_argument("--precision", choices=["bf16", "fp32"], default="bf16")
    s.add_argument("--batch-phonemes", type=int, default=8000)
    s.add_argument("--batch-items", type=int, default=64)
    s.add_argument("--batch-window", type=int, default=256)
    s.add_argument("--batch-first-window", type=int, default=32)
    s.add_argument("--input-format", choices=["text", "phonemes"], default="phonemes")
    s.add_argument("--out-dir", default=".")
    s.add_argument("--per-line", action="store_true")
    s.add_argument("--diagnostics", action="store_true")
    s.add_argument("--format", choices=["pcm16", "float32"], default="pcm16")
    s.add_argument("--seed", type=int, default=0)
    s.add_argument("--force", action="store_true")
    s.add_argument("--blank-lines", choices=["error", "skip"], default="error")
    s.add_argument("--write-threads", type=int, default=4)
    s.add_argument("--fsync", action="store_true")
    return p


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    if args.batch_phonemes < 1:
        print("error: --batch-phonemes must be >= 1", file=sys.stderr)
        return 2
    try:
        return synth(args)
    except Exception as e:  # noqa: BLE001 - anything escaping the pipeline is a job-level error
        print(f"error: {e}", file=sys.stderr)
        return 2


if __name__ == "__main__":
    sys.exit(main())
