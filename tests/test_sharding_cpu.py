"""Host-side logic of the multi-GPU path, on CPU: the trace remap that gives
each rank its channels, the per-rank (sharded) timing semantics against the
unsharded run, and the all-gather + reorder of die activity that feeds the
replicated thermal step -- as world-size-2 gloo process groups."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import hbf_oracle as ho
from helpers import OracleRun, Setup
from hbfsim_b200 import sharding
from hbfsim_b200 import workloads as wl

STRIPE = 4096


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def setup_for(stacks, rank=0, world=1):
    p = wl.c0_profile()
    p["capacity_bytes"] = 64 * (1 << 30) * max(1, world)
    s = Setup(profile=p, model=3, stacks=stacks, stripe=STRIPE, shard_rank=rank,
              shard_count=world)
    s.ranges = [(wl.RANGE_BASE, 60 * (1 << 30) * max(1, world), 1, 3)]
    return s


def test_remap_keeps_each_access_on_the_rank_channels():
    world, stacks = 4, 2
    a = wl.c0_trace(20000, seed=3, range_length=60 << 30)
    base = setup_for(stacks)
    ob = OracleRun(base)
    d0 = ho.decode(ob.ranges, ob.count, ob.geometry, *a[:3])
    channels = stacks * base.profile["channels"]
    for rank in range(world):
        moved = sharding.remap_to_shard(a[0], rank, world, wl.RANGE_BASE, 60 << 30, channels,
                                        STRIPE)
        sh = setup_for(stacks * world, rank, world)
        osh = OracleRun(sh)
        d1 = ho.decode(osh.ranges, osh.count, osh.geometry, moved, a[1], a[2])
        # accesses inside one stripe unit (the remap moves stripe units)
        inside = (a[0] % STRIPE) + a[1] <= STRIPE
        timed = (d0["status"] == 1) & inside
        assert timed.sum() > 10000
        assert np.array_equal(d1["status"][timed], d0["status"][timed])
        assert np.array_equal(d1["channel"][timed] % world, np.full(timed.sum(), rank))
        assert np.array_equal(d1["channel"][timed] // world, d0["channel"][timed])
        assert np.array_equal(d1["die"][timed], d0["die"][timed])
        assert np.array_equal(d1["plane"][timed], d0["plane"][timed])


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        stacks = 2
        a = wl.c0_trace(30000, seed=9, range_length=60 << 30)
        # every rank times the whole trace with its shard geometry
        run = OracleRun(setup_for(stacks, rank, world))
        done, lat, status, _ = run.run(*a)
        results = [None] * world
        dist.all_gather_object(results, (done, lat, status))
        # activity of the rank's local dies, gathered and put in global order
        s = run.s
        dies = s.profile["dies_per_channel"]
        local = torch.arange(s.local_channels * dies, dtype=torch.int64) * 10 + rank
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        idx = torch.from_numpy(sharding.global_die_index(world, s.local_channels, dies,
                                                         s.channels_total))
        global_order = torch.cat(parts).index_select(0, idx).numpy()
        expect = sharding.global_die_order([p.numpy() for p in parts], world, dies,
                                           s.channels_total)
        if rank == 0:
            q.put((results, global_order, expect))
    finally:
        dist.destroy_process_group()


def test_sharded_ranks_reproduce_the_unsharded_run():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results, global_order, expect = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # the unsharded oracle on the same trace and channel count
    a = wl.c0_trace(30000, seed=9, range_length=60 << 30)
    s = setup_for(2)
    s.profile["capacity_bytes"] = 64 * (1 << 30) * world
    s.ranges = [(wl.RANGE_BASE, 60 * (1 << 30) * world, 1, 3)]
    want = OracleRun(s).run(*a)
    merged_done = np.zeros_like(want[0])
    merged_status = np.zeros_like(want[2])
    for done, lat, status in results:
        mine = status == 1
        merged_done[mine] = done[mine]
        merged_status[mine] = 1
    timed = want[2] == 1
    assert np.array_equal(merged_status == 1, timed)
    assert np.array_equal(merged_done[timed], want[0][timed])
    assert np.array_equal(global_order, expect)
