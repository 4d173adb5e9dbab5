"""The sharded (N > 1) host path on CPU ranks (gloo, world_size 2): each rank builds and steps its own contiguous
range of seeded worlds with the parity oracle, the per-world statistics are all-gathered, and the result equals one
process stepping all the worlds; a rank that dies before the collective makes the other fail with an error (no
hang)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _stats_of(first, n, steps):
    import oracle_lib
    from goib2d import configs, shard
    from goib2d.world import map_state
    sc, model, host = configs.batch("c0", n, 0, first=first)
    st = oracle_lib.step(model, host, sc.settings, configs.DT, steps, threads=2)
    dev = map_state(lambda x: torch.from_numpy(np.array(x)), st)
    return shard.episode_stats(dev, 1)


def _worker(rank, world, port, n, steps, out, die):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root / "getting-over-it-rl_b200"), str(root / "tests")]
    import datetime
    from goib2d import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        first, cnt = shard.world_range(n, rank)
        stats = _stats_of(first, cnt, steps)
        if die and rank == 1:
            os._exit(3)  # a rank that leaves between steps, before the collective
        try:
            got = shard.gather_stats(stats)
            out[rank] = got.numpy().tobytes()
        except Exception as e:  # the surviving rank learns of the dead one through the collective's error
            out[rank] = b"error:" + str(e).encode()[:200]
    finally:
        if not (die and rank == 1):
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def test_sharded_stats_equal_single_process():
    port, n, steps = _free_port(), 3, 5
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(2, port, n, steps, out, False), nprocs=2, start_method="spawn", join=True)
    want = _stats_of(0, 2 * n, steps).numpy()
    for r in (0, 1):
        got = np.frombuffer(out[r], np.float32).reshape(want.shape)
        assert np.array_equal(got, want)
    assert not np.array_equal(want[0], want[n])  # the ranks' worlds really differ


def test_dead_rank_is_an_error_not_a_hang():
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    ctx = mp.start_processes(_worker, args=(2, port, 2, 2, out, True), nprocs=2, start_method="spawn", join=False)
    ctx.processes[0].join(120)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    assert not ctx.processes[0].is_alive()
    assert out.get(0, b"").startswith(b"error:")
