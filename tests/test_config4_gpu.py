"""Config 4 (the sharded mixed trace) against the oracle, on one GPU.

The trace generator of the config-4 bench (hbfsim_b200.workloads.C4Trace:
MoE expert reads and paged-KV reads / appends interleaved by arrival, on 16
stacks x 16 channels x 8 dies x 4 planes) at a reduced length, timed

  * unsharded: one context owns all 256 channels (the generic piece kernel:
    256 channels x 10 columns exceed the direct kernels' 512 column items);
  * sharded 8 ways: eight contexts on the one GPU, shard r owning channels
    g % 8 == r and timing only the accesses the generator kept for it (the
    direct kernels, 32 channels each), as the eight ranks of the bench do.

Every shard's ticks, latencies and statuses are bit-exact against the
oracle run of the same shard, and the shards together cover the trace.
"""
import os

import numpy as np
import pytest

from helpers import OracleRun, Setup, make_context
from hbfsim_b200 import workloads as wl

pytestmark = pytest.mark.gpu

N = 5 * 600_000 + 3        # global accesses (a ragged tail of 3)
SPAN = 3_000_000           # 3 ms of arrivals


def c4_setup(gen, rank, world):
    p = wl.c4_profile()
    unit = (p["page_bytes"] * p["channels"] * p["dies_per_channel"] * p["planes_per_die"] *
            p["pages_per_block"])
    p["capacity_bytes"] = -(-(wl.C4_MOE_LENGTH + gen.kv_length) // unit) * unit
    s = Setup(profile=p, model=3, stacks=wl.C4_STACKS, stripe=4096, shard_rank=rank,
              shard_count=world)
    s.ranges = [(wl.RANGE_BASE, wl.C4_MOE_LENGTH, 1, 1), (wl.C4_KV_BASE, gen.kv_length, 1, 3)]
    return s


def shard_trace(gen, rank, world):
    import torch

    def channel_of(a):
        kv = a >= wl.C4_KV_BASE
        media = torch.where(kv, a - wl.C4_KV_BASE + wl.C4_MOE_LENGTH, a - wl.RANGE_BASE)
        return (media >> 12) % 256

    parts = list(gen.chunks(channel_of, lambda g: g % world == rank, m=1 << 18))
    return [torch.cat([p[k] for p in parts]) for k in range(4)]


@pytest.mark.parametrize("world", [1, 8])
def test_config4_shards_match_oracle(tmp_path, world):
    import torch
    gen = wl.C4Trace("cuda", n=N, span_ns=SPAN)
    threads = os.cpu_count() or 1
    total = 0
    for rank in range(world):
        s = c4_setup(gen, rank, world)
        ctx = make_context(s, str(tmp_path / f"r{rank}"))
        dev = shard_trace(gen, rank, world)
        out = ctx.submit(*dev)
        torch.cuda.synchronize()
        host = (dev[0].cpu().numpy().view(np.uint64), dev[1].cpu().numpy().view(np.uint32),
                dev[2].cpu().numpy(), dev[3].cpu().numpy().view(np.uint64))
        want = OracleRun(s).run(*host, threads=threads)
        got = (out.done_ns.cpu().numpy().view(np.uint64),
               out.latency_ns.cpu().numpy().view(np.uint64), out.status.cpu().numpy())
        for g, w, name in zip(got, want[:3], ("done", "latency", "status")):
            bad = np.flatnonzero(g != w)
            assert bad.size == 0, f"rank {rank}: {name} differs at {bad[:5]}"
        assert (want[2] == 1).all(), "every access of the trace is timed on its shard"
        total += host[0].size
        ctx.close()
    assert total == N
