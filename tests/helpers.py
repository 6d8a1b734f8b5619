"""Shared test plumbing: run one trace through the CUDA path (C ABI via the
hbfsim_b200 host package) and through the CPU oracle, and compare."""
from __future__ import annotations

import ctypes
import tempfile
from dataclasses import dataclass, field

import numpy as np

import hbf_oracle as ho
from hbfsim_b200 import workloads as wl

ORDER_CODES = {"C": 0, "W": 1, "D": 2, "P": 3}


@dataclass
class Setup:
    profile: dict
    stacks: int = 1
    stripe: int = 4096
    shard_rank: int = 0
    shard_count: int = 1
    model: int = 3
    ranges: list = field(default_factory=list)  # (base, length, mode, perms)

    @property
    def channels_total(self):
        return self.stacks * self.profile["channels"]

    @property
    def local_channels(self):
        return 1 if self.model == 1 else -(-self.channels_total // self.shard_count)

    @property
    def k(self):
        return 1 if self.model == 1 else self.profile["dies_per_channel"] + 1


def oracle_ranges(setup: Setup):
    """Mirror of the context's range table: sorted, file offsets allocated in
    registration order by page-rounded extent (range_table.cpp:42-80)."""
    page = setup.profile["page_bytes"]
    rows, offset = [], 0
    for rid, (base, length, mode, perms) in enumerate(setup.ranges, start=1):
        rows.append((base, length, offset, rid, mode, perms, page))
        offset += -(-length // page) * page
    rows.sort(key=lambda r: r[0])
    return ho.make_ranges(rows), len(rows)


class OracleRun:
    """Oracle state across batches for one Setup."""

    def __init__(self, setup: Setup, refresh=None, throttle=None, admit=None):
        self.s = setup
        p = setup.profile
        self.ranges, self.count = oracle_ranges(setup)
        self.geometry = ho.make_geometry(setup.stacks, p["channels"], p["dies_per_channel"],
                                         p["planes_per_die"], setup.stripe, p["page_bytes"],
                                         p.get("plane_allocation_scheme", "CWDP"),
                                         setup.shard_rank, setup.shard_count)
        self.timing = ho.Timing(setup.model, p["time_scale"], p["read_latency_ns"],
                                p["program_latency_ns"], p["aggregate_bandwidth_bytes_per_s"],
                                p["page_bytes"])
        self.state = np.zeros(setup.local_channels * setup.k, np.uint64)
        self.set_factors(refresh, throttle, admit)

    def set_factors(self, refresh=None, throttle=None, admit=None):
        p, s = self.s.profile, self.s
        bw = p["channel_width_bits"] * p["channel_transfer_rate_mtps"] * 1_000_000 // 8
        r = np.zeros(s.local_channels, np.int64) if refresh is None else np.asarray(refresh)
        self.chan_bw = np.array([max(1, bw * (1000 - int(x)) // 1000) for x in r], np.uint64)
        t = np.full(s.stacks, 1000) if throttle is None else np.asarray(throttle)
        self.t_read = np.array([-(-p["read_latency_ns"] * int(x) // 1000) for x in t], np.uint64)
        self.t_prog = np.array([-(-p["program_latency_ns"] * int(x) // 1000) for x in t], np.uint64)
        self.admit = (np.zeros(s.stacks, np.uint64) if admit is None
                      else np.asarray(admit, np.uint64))

    def run(self, address, nbytes, op, arrival, threads=1):
        return ho.run_batch(self.ranges, self.count, self.geometry, self.timing,
                            self.chan_bw, self.t_read, self.t_prog, address, nbytes, op,
                            arrival, self.state, threads, self.admit)


def make_context(setup: Setup, tmpdir: str):
    import os
    from hbfsim_b200 import Context
    os.makedirs(tmpdir, exist_ok=True)
    wl.Workload("t", setup.profile, setup.stacks, setup.stripe, 0, 0).write_profile(tmpdir)
    path = f"{tmpdir}/{setup.profile['name']}.json"
    ctx = Context(path, report_dir=f"{tmpdir}/report", mode=setup.model)
    ctx.set_geometry(setup.stacks, setup.stripe, setup.shard_rank, setup.shard_count)
    for base, length, mode, perms in setup.ranges:
        ctx.register_device(base, length, mode, perms)
    return ctx


def to_device(arrays, device="cuda"):
    import torch
    a, b, o, t = arrays
    return (torch.from_numpy(a.view(np.int64)).to(device),
            torch.from_numpy(b.view(np.int32)).to(device),
            torch.from_numpy(o).to(device),
            torch.from_numpy(t.view(np.int64)).to(device))


def gpu_run(ctx, arrays):
    import torch
    dev = to_device(arrays)
    out = ctx.submit(*dev)
    torch.cuda.synchronize()
    return (out.done_ns.cpu().numpy().view(np.uint64), out.latency_ns.cpu().numpy().view(np.uint64),
            out.status.cpu().numpy())


def assert_same(gpu, oracle, what=""):
    gd, gl, gs = gpu
    od, ol, os_ = oracle[:3]
    assert gs.shape == os_.shape, what
    bad = np.flatnonzero(gs != os_)
    assert bad.size == 0, f"{what}: status differs at {bad[:5]} gpu={gs[bad[:5]]} oracle={os_[bad[:5]]}"
    bad = np.flatnonzero(gd != od)
    assert bad.size == 0, f"{what}: done differs at {bad[:5]} gpu={gd[bad[:5]]} oracle={od[bad[:5]]}"
    assert np.array_equal(gl, ol), what
