"""The N > 1 host path on CPU: two gloo ranks shard decisions, time with a
max over ranks, gather results; a rank that fails is reported, not waited on."""
import datetime
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist
    from laya_zig_b200 import shard, synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        sw = synth.sweep_decisions(600, seed=4)
        mine, loads = shard.shard(sw, world, rank, max_tokens=8192)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before its results are gathered")
        # stand-in for the per-decision forward: a value that depends only on the decision
        local = {i: int(sw[i].ids.astype(np.int64).sum() % 1000003) for b in mine for i in b}
        t = torch.tensor([float(len(local))])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res = shard.gather(local, len(sw))
        ok = res == [int(d.ids.astype(np.int64).sum() % 1000003) for d in sw]
        q.put((rank, "ok" if ok else "mismatch", float(t.item())))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error: %s" % type(e).__name__, 0.0))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(2):
        r, status, t = q.get(timeout=120)
        out[r] = status
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_two_ranks_shard_and_gather():
    out = _run("ok")
    assert out == {0: "ok", 1: "ok"}


def test_failed_rank_is_reported_not_hung():
    out = _run("fail")
    assert out[1].startswith("error")
    assert out[0].startswith("error")  # the surviving rank's collective fails instead of waiting forever
