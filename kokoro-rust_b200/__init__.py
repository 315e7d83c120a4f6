"""kokoro-b200: B200-native batched ragged Kokoro-82M forward behind a C ABI.

The compute lives in ``libkokoro_b200.so`` (CUDA for sm_100a, built from ``csrc/``); this package
holds the host-side mirror of the reference engine API (``engine``), WAV output (``wav``), the
checkpoint manifest and seeded random-init generator (``weights``) and the build step (``build``).
"""
from . import multi, pth, shard, wav, weights  # noqa: F401
from .engine import (BatchItem, BatchPolicy, Engine, GpuKokoro, ItemNoise, KokoroError, Output, Synth, Voice,
                     load_library, mix_seed, plan_batches)

__all__ = ["BatchItem", "BatchPolicy", "Engine", "GpuKokoro", "ItemNoise", "KokoroError", "Output", "Synth",
           "Voice", "load_library", "mix_seed", "plan_batches"]
