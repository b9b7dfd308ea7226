"""Multi-rank host logic on CPU (gloo, world size 2 and 3): batch partition,
ordered gather of last-position logits, and a missing rank surfacing as an
error rather than a hang."""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, global_batch, V, q):
    sys.path.insert(0, ROOT)
    from mamba_integer_b200 import distributed as mdist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    mdist.init_from_env("gloo", timeout_s=30)
    lo, hi = mdist.shard_range(global_batch, world, rank)
    # each rank's "logits": row i of the global batch holds value i in every column
    local = torch.arange(lo, hi, dtype=torch.float32).unsqueeze(1).repeat(1, V)
    full = mdist.gather_last_logits(local, global_batch)
    # the reusable gather bench.py times: twice with the same buffers, fed a strided view
    # (the last position of [b, L, V] logits) as the prefill engine's output is
    g = mdist.LastLogitsGather(global_batch, V)
    seq = torch.zeros(hi - lo, 3, V)
    for step in range(2):
        seq[:, -1, :] = local + 1000 * step
        got = g(seq[:, -1, :])
        assert got.shape == (global_batch, V)
        assert got[:, 0].tolist() == [float(i + 1000 * step) for i in range(global_batch)]
    ids = mdist.gather_ids(torch.arange(lo, hi, dtype=torch.int64).unsqueeze(1).repeat(1, 2), global_batch)
    assert ids[:, 1].tolist() == list(range(global_batch))
    q.put((rank, (lo, hi), full[:, 0].tolist()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,global_batch", [(2, 64), (3, 64), (2, 5)])
def test_partition_and_ordered_gather(world, global_batch):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, global_batch, 4, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ranges = sorted(r[1] for r in res)
    assert ranges[0][0] == 0 and ranges[-1][1] == global_batch
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    for _, _, col in res:
        assert col == [float(i) for i in range(global_batch)]


def _lonely(port, q):
    sys.path.insert(0, ROOT)
    from mamba_integer_b200 import distributed as mdist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK="0", WORLD_SIZE="2")
    try:
        mdist.init_from_env("gloo", timeout_s=3)
        q.put("joined")
    except Exception as e:  # rendezvous times out: the peer never joined
        q.put(type(e).__name__)


def test_missing_rank_is_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_free_port(), q))
    p.start()
    msg = q.get(timeout=120)
    p.join(timeout=30)
    if p.is_alive():
        p.kill()
    assert msg != "joined"


def test_shard_counts():
    from mamba_integer_b200.distributed import shard_counts, shard_range

    assert shard_counts(64, 8) == [8] * 8
    assert shard_counts(5, 2) == [3, 2]
    assert shard_range(64, 4, 3) == (48, 64)
    with pytest.raises(ValueError):
        shard_counts(4, 0)
