"""Multi-rank host logic of the decode sharding on CPU (gloo, world size 2)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fasterkernels_b200 import shard
from fasterkernels_b200 import workloads as W


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        lens = W.config_lengths(5)
        sh = shard.shard_sequences(lens, world, rank)
        # stand-in for this rank's decode output: row b filled with its global index
        out = torch.stack([torch.full((4, 8), float(i)) for i in sh.indices])
        full = shard.gather_outputs(out, sh.indices, len(lens))
        ok = all(torch.all(full[b] == b) for b in range(len(lens)))
        # the max-over-ranks step timing the bench uses
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, ok, sh.kv_tokens, float(t)))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e), 0, 0.0))


def test_sequence_sharding_and_gather_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    res.sort()
    assert [r[1] for r in res] == [True, True], res
    tokens = [r[2] for r in res]
    assert sum(tokens) == sum(W.config_lengths(5))
    assert max(tokens) / (sum(tokens) / 2) < 1.001
    assert all(r[3] == 2.0 for r in res)


def test_kv_head_split_and_choice():
    assert shard.shard_kv_heads(8, 64, 4, 1) == ((2, 4), (16, 32))
    with pytest.raises(ValueError):
        shard.shard_kv_heads(8, 64, 3, 0)
    assert shard.choose_partition(4, 8, 4) == "kv_head"
    assert shard.choose_partition(128, 8, 8) == "sequence"
    sh = shard.shard_sequences([5, 4, 3, 2, 1], 2, 0)
    assert sh.indices == [0, 3, 4] and sh.kv_tokens == 8


def _failing_worker(rank, world, port, q, mode):
    """Rank 1 fails before the output gather: it raises and exits ("exit"), or
    stays alive without joining ("stall").  Rank 0 must get an error from the
    gather within the process group's timeout instead of hanging."""
    import datetime
    import time
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        lens = W.config_lengths(5)
        sh = shard.shard_sequences(lens, world, rank)
        out = torch.stack([torch.full((4, 8), float(i)) for i in sh.indices])
        if rank == 1:
            if mode == "stall":
                time.sleep(8)
                q.put((rank, "stalled", 0.0))
                return
            raise RuntimeError("simulated rank failure before the gather")
        t0 = time.time()
        try:
            shard.gather_outputs(out, sh.indices, len(lens))
            q.put((rank, "no error", time.time() - t0))
        except Exception as e:  # the expected path: the peer is gone or late
            q.put((rank, "error:" + type(e).__name__, time.time() - t0))
    except Exception as e:
        q.put((rank, "raised:" + str(e)[:60], 0.0))


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_gather_fails_fast_when_a_rank_dies(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r = q.get(timeout=120)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():  # pragma: no cover
            p.kill()
    assert res[0][1].startswith("error:"), res
    assert res[0][2] < 60.0, res  # bounded by the process-group timeout, not a hang
    assert res[1][1].startswith("raised:simulated") if mode == "exit" else res[1][1] == "stalled"
