"""Host-side multi-GPU logic on CPU with 2 gloo ranks: the LPT stream
partition is identical on every rank, disjoint, complete and balanced, and
the timing reductions give the max / sum over ranks."""
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


def _worker(rank, world, port, out_q):
    import datetime
    import sys
    from pathlib import Path

    import torch.distributed as dist
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import __graft_entry__ as ge
    ge.load_package()
    import importlib
    shard = importlib.import_module("qwenasr_cpp_b200.shard")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    rng = np.random.default_rng(5)
    prompts = rng.integers(65, 781, size=100)
    outs = rng.integers(32, 513, size=100)
    costs = [shard.stream_cost(int(p), int(n)) for p, n in zip(prompts, outs)]
    parts = shard.lpt_partition(costs, world)
    mine = parts[rank]
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    t_max = shard.reduce_max(dist, 1.0 + rank)
    t_sum = shard.reduce_sum(dist, float(len(mine)))
    dist.barrier()
    dist.destroy_process_group()
    out_q.put((rank, gathered, parts, costs, t_max, t_sum))


@pytest.mark.timeout(120)
def test_two_rank_partition_and_reductions():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=100) for _ in procs]
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    for rank, gathered, parts, costs, t_max, t_sum in res:
        assert gathered == parts                         # every rank computed the same split
        flat = sorted(i for part in parts for i in part)
        assert flat == list(range(100))                  # disjoint and complete
        loads = [sum(costs[i] for i in part) for part in parts]
        assert max(loads) - min(loads) <= max(costs)     # LPT balance bound
        assert t_max == 2.0 and t_sum == 100.0
