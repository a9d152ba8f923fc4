"""Host-side multi-GPU logic on CPU: two gloo ranks (no GPU).

The encoder shards by image (one replica per GPU, no collective on the data
path); what runs across processes is the image split and the max-over-ranks
timing reduction that bench.py reports.  Both are exercised here exactly as
bench.py calls them, over a real two-process gloo group on 127.0.0.1.
"""
import importlib.util
import os
import socket
import subprocess
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _shard_mod():
    spec = importlib.util.spec_from_file_location("sam3_b200_shard", os.path.join(ROOT, "sam3.cpp_b200", "shard.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, out):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    shard = _shard_mod()
    mine = shard.image_shard(batch, rank, world)
    # per-rank "step time": rank-dependent so the max is known
    t = shard.max_over_ranks(10.0 + rank * 2.5 + len(mine) * 0.01, device=torch.device("cpu"))
    # every rank sees every other rank's shard: gather to check the partition
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    dist.barrier()
    dist.destroy_process_group()
    out.put((rank, mine, t, gathered))


@pytest.mark.parametrize("batch", [64, 7, 1])
def test_two_rank_shard_and_max(batch):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    shards = [r[1] for r in res]
    # disjoint, covering, balanced within one image
    flat = sorted(i for sh in shards for i in sh)
    assert flat == list(range(batch))
    assert max(map(len, shards)) - min(map(len, shards)) <= 1
    # both ranks report the same max-over-ranks time
    expect = max(10.0 + r * 2.5 + len(shards[r]) * 0.01 for r in range(world))
    assert all(abs(r[2] - expect) < 1e-12 for r in res)
    assert all(r[3] == shards for r in res)


def test_shard_rejects_bad_rank():
    shard = _shard_mod()
    with pytest.raises(ValueError):
        shard.image_shard(8, 2, 2)
    assert shard.max_over_ranks(3.5) == 3.5  # no process group: identity


def test_reference_arm_other_ranks_exit_quietly():
    """Under torchrun the reference arm's non-zero ranks do no work and print nothing."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference"], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0
    assert r.stdout.strip() == ""
