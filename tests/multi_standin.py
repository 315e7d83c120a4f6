"""Stand-in engine for the multi-GPU host tests (loaded by path in each worker process): the
engine API over a deterministic fake GPU. Each item's audio depends only on the item (its ids and
seed), pred_dur carries the worker's device, and a request containing '!' ends the worker process
(a lost GPU)."""
import os

import numpy as np


class FakeGpu:
    identity = "fake"

    def __init__(self, kk, device):
        self.kk, self.device = kk, device

    def forward_batch(self, items):
        outs = []
        for it in items:
            if 99 in list(it.ids):
                os._exit(3)
            n = 600 * len(it.ids)
            t = np.arange(n, dtype=np.float64)
            a = (0.5 * np.sin(t * 0.01 * len(it.ids)) * (1 + (it.noise.seed % 7) * 0.01)).astype(np.float32)
            outs.append(self.kk.Output(a, np.full(len(it.ids), self.device, np.int64)))
        return outs


def make_engine(kk, device):
    e = kk.Engine.__new__(kk.Engine)
    e.gpu = FakeGpu(kk, device)
    e.model_dir, e.voices = "/nonexistent", {}
    e.vocab = {c: i + 1 for i, c in enumerate("abcdefghijklmnopərstuvwxyz ")}
    e.vocab["!"] = 99
    e.model_sha256, e.config_sha256 = "m" * 64, "c" * 64
    e.add_voice("af_heart", np.arange(510 * 256, dtype=np.float32).reshape(510, 256) / 1e5)
    return e
