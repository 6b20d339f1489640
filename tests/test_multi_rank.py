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
    import bench
    box = bench.box_lengths(rank, world)                 # this rank's share of the whole-box bench workload
    box_all = [None] * world
    dist.all_gather_object(box_all, box.tolist())
    t_max = shard.reduce_max(dist, 1.0 + rank)
    t_sum = shard.reduce_sum(dist, float(len(mine)))
    dist.barrier()
    dist.destroy_process_group()
    out_q.put((rank, gathered, parts, costs, t_max, t_sum, box_all))


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
    import bench
    pool = np.concatenate([bench.stream_lengths(g) for g in range(2)])
    for rank, gathered, parts, costs, t_max, t_sum, box_all in res:
        assert gathered == parts                         # every rank computed the same split
        flat = sorted(i for part in parts for i in part)
        assert flat == list(range(100))                  # disjoint and complete
        loads = [sum(costs[i] for i in part) for part in parts]
        assert max(loads) - min(loads) <= max(costs)     # LPT balance bound
        assert t_max == 2.0 and t_sum == 100.0
        # whole-box bench workload: 256 streams per rank, together exactly the seeded pool
        assert [len(b) for b in box_all] == [256, 256]
        assert sorted(box_all[0] + box_all[1]) == sorted(pool.tolist())
        assert abs(sum(box_all[0]) - sum(box_all[1])) <= int(pool.max())


def test_lpt_cap_keeps_a_fixed_batch_per_rank():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import __graft_entry__ as ge
    ge.load_package()
    import importlib
    shard = importlib.import_module("qwenasr_cpp_b200.shard")
    rng = np.random.default_rng(3)
    costs = rng.integers(1, 5000, size=8 * 256)
    parts = shard.lpt_partition(costs, 8, cap=256)
    assert [len(p) for p in parts] == [256] * 8
    assert sorted(i for p in parts for i in p) == list(range(8 * 256))
    loads = [int(costs[p].sum()) for p in parts]
    assert max(loads) - min(loads) <= int(costs.max())
    with pytest.raises(ValueError):
        shard.lpt_partition(costs, 8, cap=255)
