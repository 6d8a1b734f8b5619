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


# ---- stripe-decode goldens from the reference's UCIe layout functions ----
DECODE_DTYPE = np.dtype([("media_address", "<u8"), ("page", "<u8"), ("status", "<u4"),
                         ("range_index", "<u4"), ("stack", "<u4"), ("channel", "<u4"),
                         ("die", "<u4"), ("plane", "<u4")])


def layout_goldens(golden_dir):
    import json
    with open(golden_dir / "layout_goldens.json") as f:
        return json.load(f)


def bank_layout_cases(golden):
    """hbf_cold_read_bank goldens (bank_layout.cpp:59-72), grouped by layout,
    as decode cases: a module of `host_channels` channels, `ncdu` dies and
    `banks_per_die` banks is one stack whose planes are the banks, with 4 KiB
    stripes and pages and allocation order CPDW (channel fastest, then bank,
    then die) -- the order in which hbf_cold_read_bank splits an LPA.  Yields
    (Setup, address, bytes, op, expected channel, die, plane)."""
    groups = {}
    for hc, nd, nb, lpa, ch, die, bank in golden["bank"]:
        groups.setdefault((hc, nd, nb), []).append((lpa, ch, die, bank))
    for (hc, nd, nb), rows in sorted(groups.items()):
        p = wl.c0_profile()
        p.update(name=f"bank-{hc}-{nd}-{nb}", channels=hc, dies_per_channel=nd,
                 planes_per_die=nb, page_bytes=4096, plane_allocation_scheme="CPDW",
                 capacity_bytes=1 << 43)
        # the decode is the same for every timing model; the die model keeps
        # at most 15 dies per channel, so NCDU 16 decodes in a FAST context
        s = Setup(profile=p, model=3 if nd <= 15 else 1, stacks=1, stripe=4096)
        s.ranges = [(wl.RANGE_BASE, 1 << 42, 1, 3)]
        r = np.array(rows, np.uint64)
        lpa = r[:, 0]
        address = wl.RANGE_BASE + lpa * np.uint64(4096) + (lpa % np.uint64(32)) * np.uint64(128)
        n = lpa.size
        yield (s, address.astype(np.uint64), np.full(n, 128, np.uint32), np.zeros(n, np.uint8),
               r[:, 1], r[:, 2], r[:, 3])


def stripe_layout_cases(golden):
    """Page-striped placement goldens (stack_router.cpp:160-250, checked
    there by ContiguousStackMap::locate and inverse_page_striped) as decode
    cases: 4 stacks x 16 channels, 16 KiB stripes and pages, one die and
    plane, so a stripe unit's channel digit is the reference's
    (page + phase) % 64 when the striped range's media offset starts `phase`
    stripes in (a first range of phase * 16 KiB registered before it).
    Yields (Setup, address, bytes, op, phase, expected stack, module,
    module-local address)."""
    groups = {}
    for phase, offset, stack, module, local in golden["stripe"]:
        groups.setdefault(phase, []).append((offset, stack, module, local))
    for phase, rows in sorted(groups.items()):
        p = wl.c0_profile()
        p.update(name=f"stripe-{phase}", dies_per_channel=1, planes_per_die=1,
                 plane_allocation_scheme="CWDP", capacity_bytes=4 * 16 * (64 << 20))
        s = Setup(profile=p, model=3, stacks=4, stripe=16384)
        length = (64 * 1024 + 37) * 16384
        base = wl.RANGE_BASE + (1 << 40)
        s.ranges = ([(wl.RANGE_BASE, phase * 16384, 1, 3)] if phase else []) + \
            [(base, length, 1, 3)]
        r = np.array(rows, np.uint64)
        n = r.shape[0]
        yield (s, (base + r[:, 0]).astype(np.uint64), np.full(n, 128, np.uint32),
               np.zeros(n, np.uint8), phase, r[:, 1], r[:, 2], r[:, 3])


def check_layout_decode(got, case, kind):
    """Compare decoded records with a layout golden case (see the two
    generators above); `got` is a DECODE_DTYPE array."""
    assert (got["status"] == 1).all(), kind
    if kind == "bank":
        _, _, _, _, ch, die, bank = case
        assert np.array_equal(got["channel"], ch)
        assert np.array_equal(got["die"], die)
        assert np.array_equal(got["plane"], bank)
        assert (got["stack"] == 0).all()
    else:
        _, _, _, _, phase, stack, module, local = case
        assert np.array_equal(got["stack"], stack)
        assert np.array_equal(got["channel"] // 4, module)
        if phase == 0:
            # rows are counted from the media origin: with no phase the
            # page inside the plane is the module-local 16 KiB page
            assert np.array_equal(got["page"], local >> np.uint64(14))


def activity_of(setup, oracle, arrays, status):
    """Per local (channel, die) read bytes and write count of the modeled
    accesses, from the oracle's decode."""
    address, nbytes, op, _ = arrays
    dec = ho.decode(oracle.ranges, oracle.count, oracle.geometry, address, nbytes, op)
    m = status == 1
    dies = setup.profile["dies_per_channel"]
    idx = (dec["channel"][m] // setup.shard_count) * dies + dec["die"][m]
    size = setup.local_channels * dies
    rb = np.bincount(idx, weights=np.where(op[m] == 0, nbytes[m], 0), minlength=size)
    wr = np.bincount(idx, weights=(op[m] == 1), minlength=size)
    return rb.astype(np.uint64), wr.astype(np.uint64)


def oracle_linked(setup, oracle_run, arrays, profile: dict):
    """The die model (the oracle run `oracle_run` of `setup`) composed with
    each stack's UCIe link (the oracle's StreamingLink, or_link_run): per
    modeled access an AR at its arrival and an R at its die completion on
    its stack's link, in ready order (AR first at equal ticks, then batch
    order).  Returns (linked done, die done, status, AR delivery or -1)."""
    address, nbytes, op, arrival = arrays
    done, _, status, _ = oracle_run.run(*arrays, threads=8)
    dec = ho.decode(oracle_run.ranges, oracle_run.count, oracle_run.geometry, address, nbytes, op)
    modeled = np.flatnonzero(status == 1)
    linked = done.copy()
    ar = np.full(done.size, -1, np.int64)
    for stack in range(setup.stacks):
        idx = modeled[dec["stack"][modeled] == stack]
        if idx.size == 0:
            continue
        ready = np.concatenate([arrival[idx], done[idx]])
        kind = np.concatenate([np.zeros(idx.size, np.uint8), np.ones(idx.size, np.uint8)])
        who = np.concatenate([idx, idx])
        order = np.lexsort((who, kind, ready))
        delivered = ho.link_run(profile, kind[order], ready[order])[0]
        r = kind[order] == 1
        linked[who[order][r]] = delivered[r]
        ar[who[order][~r]] = delivered[~r].astype(np.int64)
    return linked, done, status, ar
