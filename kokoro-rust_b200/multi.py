"""Book-scale data parallelism on one host: one engine process per GPU behind the ``Engine``
interface, so the synth pipeline (or any caller of ``synth_batch``) spreads its batches over
several GPUs without a collective.

The reference is single-GPU (one engine per process, ``--cuda-device``, src/cli.rs:625). Across
GPUs the rules of its batching carry over (src/engine.rs:165-241): each ``synth_batch`` call is
split by longest-processing-time-first assignment of the requests (cost = phoneme characters) to
the live GPUs, every GPU runs its share through its own ``Engine.synth_batch`` (length-sorted
batches, OOM halving), and the results are merged back in request order on the host, a failed
request keeping its place as an exception.

Each worker is a separate process (``python multi.py --worker ...``) that sees only its own GPU
(``CUDA_VISIBLE_DEVICES``), so every engine has its own context, stream and memory; requests and
results travel as pickled plain data over the worker's stdin / stdout. A worker that exits (a
crashed process, a lost GPU) fails only the requests it held; later calls use the remaining
workers, and the call fails as a whole only when none is left.
"""
from __future__ import annotations

import os
import pickle
import subprocess
import sys
from typing import List, Optional, Sequence

if __name__ == "__main__" and not __package__:
    # run as a worker (the package directory's name is not a Python identifier): load the package
    # from this directory and run its copy of this module
    import importlib.util

    _here = os.path.dirname(os.path.abspath(__file__))
    _spec = importlib.util.spec_from_file_location("kokoro_rust_b200", os.path.join(_here, "__init__.py"),
                                                   submodule_search_locations=[_here])
    _pkg = importlib.util.module_from_spec(_spec)
    sys.modules["kokoro_rust_b200"] = _pkg
    _spec.loader.exec_module(_pkg)
    from kokoro_rust_b200 import multi as _multi

    sys.exit(_multi.worker_main(sys.argv[1:]))

from .engine import BatchPolicy, Synth, Voice  # noqa: E402
from .shard import LineError, assemble_in_order, shard_lpt  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


class WorkerLost(RuntimeError):
    """A worker process that exited or broke the protocol."""


class MultiEngine:
    """``Engine`` over several GPUs: ``synth_batch``, ``voice``, ``add_voice``, ``identity``,
    ``model_sha256`` and ``config_sha256`` as the single-GPU engine has them.

    devices: CUDA ordinals as the caller sees them (indices into its own ``CUDA_VISIBLE_DEVICES``
    when that is set). standin: a Python file whose ``make_engine(pkg, device)`` builds the
    worker's engine instead of ``Engine(weights, ...)`` (tests on hosts without a GPU)."""

    def __init__(self, weights_path: str, devices: Sequence[int], precision: str = "bf16",
                 model_dir: Optional[str] = None, standin: Optional[str] = None, start_timeout: float = 600.0):
        if not devices:
            raise ValueError("no devices")
        self.procs: List[Optional[subprocess.Popen]] = []
        if standin is None and os.environ.get("KK_NO_BUILD") != "1" and os.path.isdir(os.path.join(HERE, "csrc")):
            # bring the library up to date here, once, so the workers never compile concurrently
            from . import build as _build
            _build.build()
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        vis = [v.strip() for v in visible.split(",")] if visible else None
        self.devices = list(devices)
        for d in self.devices:
            env = dict(os.environ)
            if vis is not None:
                if not 0 <= d < len(vis):
                    self.close()
                    raise ValueError(f"device {d} is not among CUDA_VISIBLE_DEVICES={visible}")
                env["CUDA_VISIBLE_DEVICES"] = vis[d]
            else:
                env["CUDA_VISIBLE_DEVICES"] = str(d)
            cmd = [sys.executable, os.path.join(HERE, "multi.py"), "--worker", "--device", str(d), "--weights",
                   weights_path, "--precision", precision]
            if model_dir is not None:
                cmd += ["--model-dir", model_dir]
            if standin is not None:
                cmd += ["--standin", standin]
            self.procs.append(subprocess.Popen(cmd, stdin=subprocess.PIPE, stdout=subprocess.PIPE, env=env))
        infos = []
        for w in range(len(self.procs)):
            try:
                rep = self._recv(w, timeout=start_timeout)
            except WorkerLost as e:
                rep = ("fatal", str(e))
            infos.append(rep)
        bad = [(self.devices[w], r[1]) for w, r in enumerate(infos) if r[0] != "ready"]
        if bad:
            self.close()
            raise RuntimeError("; ".join(f"cuda device {d}: {m}" for d, m in bad))
        info = infos[0][1]
        self._identity = info["identity"]
        self.model_sha256, self.config_sha256 = info["model_sha256"], info["config_sha256"]
        self.voices = {}

    # -- protocol
    def _send(self, w: int, msg) -> None:
        p = self.procs[w]
        if p is None:
            raise WorkerLost(f"worker for cuda device {self.devices[w]} is gone")
        try:
            pickle.dump(msg, p.stdin, protocol=pickle.HIGHEST_PROTOCOL)
            p.stdin.flush()
        except (BrokenPipeError, OSError) as e:
            self._drop(w)
            raise WorkerLost(f"worker for cuda device {self.devices[w]} exited ({e})") from None

    def _recv(self, w: int, timeout: Optional[float] = None):
        p = self.procs[w]
        if p is None:
            raise WorkerLost(f"worker for cuda device {self.devices[w]} is gone")
        if timeout is not None:  # only before the first message, when nothing is buffered yet
            import select
            if not select.select([p.stdout], [], [], timeout)[0]:
                self._drop(w)
                raise WorkerLost(f"worker for cuda device {self.devices[w]} did not answer within {timeout:.0f} s")
        try:
            return pickle.load(p.stdout)
        except (EOFError, pickle.UnpicklingError, OSError) as e:
            self._drop(w)
            raise WorkerLost(f"worker for cuda device {self.devices[w]} exited ({type(e).__name__})") from None

    def _drop(self, w: int) -> None:
        p = self.procs[w]
        self.procs[w] = None
        if p is not None:
            try:
                p.kill()
                p.wait(timeout=10)
            except Exception:  # noqa: BLE001 - already gone
                pass

    def live(self) -> List[int]:
        return [w for w, p in enumerate(self.procs) if p is not None]

    def _ask_one(self, msg):
        """Send msg to the first live worker that answers; returns its reply."""
        for w in self.live():
            try:
                self._send(w, msg)
                return self._recv(w)
            except WorkerLost:
                continue
        raise RuntimeError("no GPU worker left")

    # -- the Engine interface
    def identity(self) -> str:
        return self._identity

    def voice(self, spec: str) -> Voice:
        if spec not in self.voices:
            rep = self._ask_one(("voice", spec))
            if rep[0] != "ok":
                raise ValueError(rep[1])
            self.voices[spec] = Voice(rep[1], rep[2])
        return self.voices[spec]

    def add_voice(self, name: str, pack) -> None:
        for w in self.live():
            try:
                self._send(w, ("add_voice", name, pack))
                self._recv(w)
            except WorkerLost:
                pass
        self.voices.pop(name, None)

    def synth_batch(self, reqs: Sequence[tuple], voice: str, speed: float = 1.0,
                    policy: BatchPolicy = BatchPolicy()) -> list:
        """Same contract as ``Engine.synth_batch``: per request a Synth or an Exception, in order."""
        live = self.live()
        if not live:
            raise RuntimeError("no GPU worker left")
        shards = shard_lpt([len(r[0]) for r in reqs], len(live)) if reqs else [[] for _ in live]
        sent = []
        for w, idx in zip(live, shards):
            if not idx:
                continue
            try:
                self._send(w, ("synth", [reqs[i] for i in idx], voice, float(speed), policy.max_phonemes,
                               policy.max_items))
                sent.append((w, idx))
            except WorkerLost as e:
                sent.append((w, idx, str(e)))
        per_rank = []
        for entry in sent:
            w, idx = entry[0], entry[1]
            part = {}
            if len(entry) == 3:
                rep = ("err", entry[2])
            else:
                try:
                    rep = self._recv(w)
                except WorkerLost as e:
                    rep = ("err", str(e))
            if rep[0] == "ok":
                for i, r in zip(idx, rep[1]):
                    part[i] = Synth(r[1], r[2], list(r[3])) if r[0] == "ok" else RuntimeError(r[1])
            else:
                for i in idx:
                    part[i] = LineError(rep[1])
            per_rank.append(part)
        return assemble_in_order(len(reqs), per_rank)

    def close(self) -> None:
        for w in range(len(self.procs)):
            p = self.procs[w]
            if p is None:
                continue
            try:
                pickle.dump(("quit",), p.stdin)
                p.stdin.flush()
                p.stdin.close()
                p.wait(timeout=30)
            except Exception:  # noqa: BLE001 - a worker that does not leave in time is ended
                p.kill()
                p.wait(timeout=10)
            self.procs[w] = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        if getattr(self, "procs", None):
            try:
                self.close()
            except Exception:  # noqa: BLE001
                pass


def worker_main(argv: List[str]) -> int:
    """One GPU's engine process: reads pickled requests from stdin, answers on stdout."""
    import argparse

    ap = argparse.ArgumentParser(prog="multi.py --worker")
    ap.add_argument("--worker", action="store_true")
    ap.add_argument("--device", type=int, required=True)
    ap.add_argument("--weights", required=True)
    ap.add_argument("--precision", default="bf16")
    ap.add_argument("--model-dir", default=None)
    ap.add_argument("--standin", default=None)
    args = ap.parse_args(argv)
    # the protocol owns the original stdout; anything else printed (Python or the library) goes
    # to stderr
    out = os.fdopen(os.dup(1), "wb")
    os.dup2(2, 1)
    inp = sys.stdin.buffer

    def send(msg):
        pickle.dump(msg, out, protocol=pickle.HIGHEST_PROTOCOL)
        out.flush()

    try:
        if args.standin:
            import importlib.util
            spec = importlib.util.spec_from_file_location("kk_standin", args.standin)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            eng = mod.make_engine(sys.modules["kokoro_rust_b200"], args.device)
        else:
            from .engine import Engine
            eng = Engine(args.weights, 0, args.precision, model_dir=args.model_dir)  # the one visible GPU
        send(("ready", {"identity": eng.identity(), "model_sha256": eng.model_sha256,
                        "config_sha256": eng.config_sha256}))
    except Exception as e:  # noqa: BLE001 - reported to the parent, which refuses to start
        send(("fatal", f"{type(e).__name__}: {e}"))
        return 1
    while True:
        try:
            msg = pickle.load(inp)
        except EOFError:
            return 0
        try:
            if msg[0] == "quit":
                return 0
            if msg[0] == "voice":
                v = eng.voice(msg[1])
                send(("ok", v.pack, v.sha256))
            elif msg[0] == "add_voice":
                eng.add_voice(msg[1], msg[2])
                send(("ok",))
            elif msg[0] == "synth":
                res = eng.synth_batch(msg[1], msg[2], msg[3], BatchPolicy(max_phonemes=msg[4], max_items=msg[5]))
                send(("ok", [("err", f"{type(r).__name__}: {r}") if isinstance(r, Exception) else
                             ("ok", r.audio, r.pred_dur, list(r.dropped)) for r in res]))
            else:
                send(("err", f"unknown request {msg[0]!r}"))
        except Exception as e:  # noqa: BLE001 - a failed request is answered, the worker stays
            send(("err", f"{type(e).__name__}: {e}"))
