"""Data-parallel host path on CPU: 2 gloo ranks shard lines (LPT), "synthesise" them with a
deterministic stand-in for the per-GPU engine, gather and reassemble in line order."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import import_package


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def fake_synth(line_idx, toks):
    if line_idx == 13:  # a line that fails on its rank
        raise RuntimeError("synthetic failure on line 13")
    return np.full(600 * (len(toks) + 2), float(line_idx), np.float32)


def _worker(rank, world, port, lines, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    kk = import_package()
    mine = kk.shard.shard_lpt([len(t) for t in lines], world)[rank]
    out = {}
    for i in mine:
        try:
            out[i] = fake_synth(i, lines[i])
        except Exception as e:  # per-line failure travels back as data, never as a hang
            out[i] = e
    gathered = [None] * world
    dist.all_gather_object(gathered, out)
    if rank == 0:
        q.put(kk.shard.assemble_in_order(len(lines), gathered))
    dist.barrier()
    dist.destroy_process_group()


def test_lpt_balances_and_covers(kk):
    rng = np.random.default_rng(0)
    costs = list(rng.integers(8, 510, 2000))
    for world in (1, 2, 4, 8):
        shards = kk.shard.shard_lpt(costs, world)
        assert sorted(i for s in shards for i in s) == list(range(2000))
        loads = [sum(costs[i] for i in s) for s in shards]
        assert max(loads) - min(loads) <= max(costs)  # LPT bound


def test_assemble_reports_missing_and_duplicates(kk):
    res = kk.shard.assemble_in_order(3, [{0: "a"}, {2: "c"}])
    assert res[0] == "a" and res[2] == "c" and isinstance(res[1], kk.shard.LineError)
    with pytest.raises(ValueError):
        kk.shard.assemble_in_order(2, [{0: 1}, {0: 2}])


def test_two_rank_gloo_shard_and_reassemble():
    rng = np.random.default_rng(1)
    lines = [list(rng.integers(1, 178, n)) for n in rng.integers(8, 200, 40)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, lines, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(res) == 40
    for i, r in enumerate(res):
        if i == 13:
            assert isinstance(r, RuntimeError)
        else:
            assert r.shape == (600 * (len(lines[i]) + 2),) and r[0] == i
