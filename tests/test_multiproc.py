"""Multi-process host logic with world_size 2 over gloo (CPU): the sequence
partition every rank computes is identical, disjoint and balanced; each rank
plans its shard on its own dry-run pool; and a rank that fails before a
collective is detected by the other rank through the process group's timeout
(host-side failure detection, no GPU involved)."""
import os
import socket
from datetime import timedelta

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_worker(rank, world, port, q):
    import ctypes as C
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import numpy as np

    import krill_b200 as kb
    from krill_b200 import _lib as L
    from krill_b200.shard import lpt_partition
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    lengths = [int(x) for x in np.random.default_rng(1).integers(512, 8193, size=64)]
    parts = lpt_partition(lengths, world)
    mine = parts[rank]
    pool = kb.KVPool(32, 8, 32, 128, num_blocks=4000, device=-1)
    seqs = [pool.create_sequence() for _ in mine]
    for s, i in zip(seqs, mine):
        arr = (C.c_uint64 * 1)(s.handle)
        L.check(L.lib.krill_append_quantize(pool.handle, 1, arr, 0, 32, lengths[i], None, None, 1, None))
    arr = (C.c_uint64 * len(seqs))(*[s.handle for s in seqs])
    L.check(L.lib.krill_decode_attention(pool.handle, len(seqs), arr, 0, 32, None, 1, None, 2, 1.0, None))
    load = torch.tensor([sum(lengths[i] for i in mine)], dtype=torch.int64)
    gathered = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(gathered, load)
    idx = [torch.zeros(64, dtype=torch.int64) for _ in range(world)]
    mine_t = torch.full((64,), -1, dtype=torch.int64)
    mine_t[: len(mine)] = torch.tensor(mine)
    dist.all_gather(idx, mine_t)
    if rank == 0:
        all_idx = sorted(int(x) for t in idx for x in t.tolist() if x >= 0)
        q.put((all_idx, [int(t.item()) for t in gathered], sum(lengths), pool.last_plan()))
    dist.destroy_process_group()


def test_two_rank_partition_and_planning():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    all_idx, loads, total, plan = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all_idx == list(range(64))
    assert sum(loads) == total
    assert max(loads) - min(loads) <= 8192  # LPT: within one sequence
    assert plan[3] > 0


def _failing_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        # a rank that dies between steps, with no collective in flight
        os._exit(3)
    t = torch.ones(1)
    try:
        dist.all_reduce(t)
        q.put("no error")
    except Exception as e:  # the survivor learns of the failure on the host
        q.put(type(e).__name__)


def test_rank_failure_detected_by_survivor():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    result = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert result != "no error"
    assert procs[1].exitcode == 3
