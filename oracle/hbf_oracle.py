"""ctypes wrapper around oracle/libhbf_oracle.so (the C restatement).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py as the checker.  The shipped package never
imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libhbf_oracle.so"

STATUS_MODELED = 1
STATUS_UNSUPPORTED = 6
STATUS_BYPASS = 8
STATUS_FOREIGN = 9
MODEL_FAST = 1
MODEL_DIE = 3
ORDER_LETTERS = {"C": 0, "W": 1, "D": 2, "P": 3}


class Range(ctypes.Structure):
    _fields_ = [("base", ctypes.c_uint64), ("length", ctypes.c_uint64),
                ("file_offset", ctypes.c_uint64), ("range_id", ctypes.c_uint32),
                ("mode", ctypes.c_uint32), ("permissions", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32), ("page_bytes", ctypes.c_uint64)]


class Geometry(ctypes.Structure):
    _fields_ = [("stacks", ctypes.c_uint32), ("channels_per_stack", ctypes.c_uint32),
                ("dies_per_channel", ctypes.c_uint32), ("planes_per_die", ctypes.c_uint32),
                ("stripe_bytes", ctypes.c_uint32), ("page_bytes", ctypes.c_uint32),
                ("order", ctypes.c_uint8 * 4), ("shard_rank", ctypes.c_uint32),
                ("shard_count", ctypes.c_uint32)]


class Timing(ctypes.Structure):
    _fields_ = [("model", ctypes.c_uint32), ("time_scale", ctypes.c_uint32),
                ("read_latency_ns", ctypes.c_uint64),
                ("program_latency_ns", ctypes.c_uint64),
                ("aggregate_bandwidth", ctypes.c_uint64),
                ("page_bytes", ctypes.c_uint64)]


class Decoded(ctypes.Structure):
    _fields_ = [("media_address", ctypes.c_uint64), ("page", ctypes.c_uint64),
                ("status", ctypes.c_uint32), ("range_index", ctypes.c_uint32),
                ("stack", ctypes.c_uint32), ("channel", ctypes.c_uint32),
                ("die", ctypes.c_uint32), ("plane", ctypes.c_uint32)]


class Stats(ctypes.Structure):
    _fields_ = [("modeled", ctypes.c_uint64), ("bypass", ctypes.c_uint64),
                ("unsupported", ctypes.c_uint64), ("foreign", ctypes.c_uint64),
                ("fast_modeled_ns", ctypes.c_uint64), ("latency_sum", ctypes.c_uint64),
                ("max_done", ctypes.c_uint64)]


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        subprocess.run(["make", "-C", str(HERE), "libhbf_oracle.so"], check=True,
                       capture_output=True)
    lib = ctypes.CDLL(str(LIB_PATH))
    u64, u32, p = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_void_p
    lib.or_saturating_add.restype = u64
    lib.or_saturating_add.argtypes = [u64, u64]
    lib.or_saturating_multiply.restype = u64
    lib.or_saturating_multiply.argtypes = [u64, u32]
    lib.or_fast_transfer_ns.restype = u64
    lib.or_fast_transfer_ns.argtypes = [u32, u64]
    lib.or_fast_service_ns.restype = u64
    lib.or_fast_service_ns.argtypes = [u64, u32, u64]
    lib.or_find_range_index.restype = u32
    lib.or_find_range_index.argtypes = [p, u32, u64]
    lib.or_access_supported.restype = ctypes.c_int
    lib.or_access_supported.argtypes = [p, u64, u32, u32]
    lib.or_range_overlaps.restype = ctypes.c_int
    lib.or_range_overlaps.argtypes = [p, u64, u32]
    lib.or_media_descriptor.restype = ctypes.c_int
    lib.or_media_descriptor.argtypes = [p, u64, u32, u32, p, p]
    lib.or_sample_threshold.restype = u64
    lib.or_sample_threshold.argtypes = [ctypes.c_double]
    lib.or_hybrid_reference_sample.restype = ctypes.c_int
    lib.or_hybrid_reference_sample.argtypes = [u64, u32, u64, u64]
    lib.or_decode_batch.restype = None
    lib.or_decode_batch.argtypes = [p, u32, p, p, p, p, u64, p]
    lib.or_run_batch_threads.restype = ctypes.c_int
    lib.or_run_batch_threads.argtypes = [p, u32, p, p, p, p, p, p, p, p, p, p,
                                         u64, p, p, p, p, p, ctypes.c_int]
    lib.or_clock_new.restype = ctypes.c_void_p
    lib.or_clock_new.argtypes = [u64]
    lib.or_clock_free.restype = None
    lib.or_clock_free.argtypes = [p]
    lib.or_clock_run.restype = None
    lib.or_clock_run.argtypes = [p, p, p, u64, p, p, p]
    lib.or_capacity_timing.restype = None
    lib.or_capacity_timing.argtypes = [p, p, p, p, p, p, p, p, p, p, p, p, u64, u32, p, p, p]
    lib.or_lru_run.restype = None
    lib.or_lru_run.argtypes = [p, p, u64, u64, p, p, p]
    lib.or_empirical_cumulative_ns.restype = u64
    lib.or_empirical_cumulative_ns.argtypes = [p, p, u32, u32]
    lib.or_empirical_service_ns.restype = u64
    lib.or_empirical_service_ns.argtypes = [p, p, u32, u32]
    lib.or_update_empirical_burst.restype = ctypes.c_int
    lib.or_update_empirical_burst.argtypes = [u64, u64, u32, p, p]
    lib.or_empirical_control_valid.restype = ctypes.c_int
    lib.or_empirical_control_valid.argtypes = [p]
    lib.or_empirical_request_service.restype = ctypes.c_int
    lib.or_empirical_request_service.argtypes = [p, u64, u64, u32, p, p, p]
    lib.or_link_run.restype = ctypes.c_int
    lib.or_link_run.argtypes = [p, p, p, u64, p, p]
    lib.or_prefetch_run.restype = ctypes.c_int
    lib.or_prefetch_run.argtypes = [p, u64, p, p]
    lib.or_run_empirical_batch.restype = ctypes.c_int
    lib.or_run_empirical_batch.argtypes = [p, u32, p, u32, u64, p, p, p, p, u64, p, p, p, p,
                                           p]
    return lib


LIB = _load()


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def make_ranges(rows) -> ctypes.Array:
    """rows: iterable of (base, length, file_offset, range_id, mode, perms, page)."""
    rows = list(rows)
    arr = (Range * max(1, len(rows)))()
    for k, r in enumerate(rows):
        arr[k] = Range(int(r[0]), int(r[1]), int(r[2]), int(r[3]), int(r[4]),
                       int(r[5]), 0, int(r[6]))
    return arr


def make_geometry(stacks, channels, dies, planes, stripe, page, order="CWDP",
                  shard_rank=0, shard_count=1) -> Geometry:
    g = Geometry()
    g.stacks, g.channels_per_stack = stacks, channels
    g.dies_per_channel, g.planes_per_die = dies, planes
    g.stripe_bytes, g.page_bytes = stripe, page
    for k, ch in enumerate(order):
        g.order[k] = ORDER_LETTERS[ch]
    g.shard_rank, g.shard_count = shard_rank, shard_count
    return g


def decode(ranges, count, geometry, address, nbytes, op) -> np.ndarray:
    n = address.size
    out = (Decoded * max(1, n))()
    LIB.or_decode_batch(ctypes.cast(ranges, ctypes.c_void_p), count,
                        ctypes.byref(geometry), _ptr(address), _ptr(nbytes),
                        _ptr(op), n, ctypes.cast(out, ctypes.c_void_p))
    dt = np.dtype([("media_address", "<u8"), ("page", "<u8"), ("status", "<u4"),
                   ("range_index", "<u4"), ("stack", "<u4"), ("channel", "<u4"),
                   ("die", "<u4"), ("plane", "<u4")])
    return np.frombuffer(bytes(out), dtype=dt)[:n].copy()


def run_batch(ranges, count, geometry, timing, chan_bw, t_read, t_prog, address,
              nbytes, op, arrival, state, threads=1, admit=None):
    """Returns (done, latency, status, stats dict); updates `state` in place."""
    n = address.size
    done = np.zeros(n, np.uint64)
    latency = np.zeros(n, np.uint64)
    status = np.zeros(n, np.uint8)
    stats = Stats()
    rc = LIB.or_run_batch_threads(
        ctypes.cast(ranges, ctypes.c_void_p), count, ctypes.byref(geometry),
        ctypes.byref(timing), _ptr(chan_bw), _ptr(t_read), _ptr(t_prog),
        None if admit is None else _ptr(admit), _ptr(address), _ptr(nbytes), _ptr(op), _ptr(arrival), n, _ptr(state),
        _ptr(done), _ptr(latency), _ptr(status), ctypes.byref(stats), threads)
    if rc != 0:
        raise MemoryError("oracle allocation failed")
    return done, latency, status, {f: getattr(stats, f) for f, _ in Stats._fields_}


def lru(pages: np.ndarray, writes: np.ndarray, frames: int):
    n = pages.size
    hit = np.zeros(n, np.uint8)
    victim = np.zeros(n, np.uint64)
    vdirty = np.zeros(n, np.uint8)
    LIB.or_lru_run(_ptr(pages), _ptr(writes), n, frames, _ptr(hit), _ptr(victim),
                   _ptr(vdirty))
    return hit, victim, vdirty


class Clock:
    """Second-chance CLOCK state across batches (the reference runtime's
    capacity policy)."""

    def __init__(self, frames: int):
        self.handle = LIB.or_clock_new(frames)
        if not self.handle:
            raise MemoryError("oracle allocation failed")

    def run(self, pages: np.ndarray, writes: np.ndarray):
        n = pages.size
        pages = np.ascontiguousarray(pages, np.uint64)
        writes = np.ascontiguousarray(writes, np.uint8)
        hit = np.zeros(n, np.uint8)
        victim = np.zeros(n, np.uint64)
        vdirty = np.zeros(n, np.uint8)
        LIB.or_clock_run(self.handle, _ptr(pages), _ptr(writes), n, _ptr(hit), _ptr(victim),
                         _ptr(vdirty))
        return hit, victim, vdirty

    def __del__(self):
        if getattr(self, "handle", None):
            LIB.or_clock_free(self.handle)
            self.handle = None


def capacity_timing(geometry, timing, chan_bw, t_read, t_prog, admit, status, hit, page,
                    victim, victim_dirty, arrival, page_shift, state):
    """Completion and latency of every access of a capacity batch; updates
    `state` (die model words) in place."""
    n = arrival.size
    done = np.zeros(n, np.uint64)
    latency = np.zeros(n, np.uint64)
    LIB.or_capacity_timing(ctypes.byref(geometry), ctypes.byref(timing), _ptr(chan_bw),
                           _ptr(t_read), _ptr(t_prog), None if admit is None else _ptr(admit),
                           _ptr(status), _ptr(hit), _ptr(page), _ptr(victim),
                           _ptr(victim_dirty), _ptr(arrival), n, page_shift, _ptr(state),
                           _ptr(done), _ptr(latency))
    return done, latency


class Empirical(ctypes.Structure):
    _fields_ = [("flags", ctypes.c_uint32), ("count", ctypes.c_uint32),
                ("program_latency_ns", ctypes.c_uint64),
                ("pages", ctypes.c_uint32 * 6), ("cumulative_ns", ctypes.c_uint64 * 6)]


def make_empirical(pages, cumulative, program_latency_ns, flags=1, count=6) -> Empirical:
    e = Empirical()
    e.flags, e.count, e.program_latency_ns = flags, count, program_latency_ns
    for k in range(6):
        e.pages[k] = int(pages[k]) if k < len(pages) else 0
        e.cumulative_ns[k] = int(cumulative[k]) if k < len(cumulative) else 0
    return e


def empirical_cumulative(pages, cumulative, count, run) -> int:
    pa = np.ascontiguousarray(pages, np.uint32)
    ca = np.ascontiguousarray(cumulative, np.uint64)
    return int(LIB.or_empirical_cumulative_ns(_ptr(pa), _ptr(ca), count, run))


def empirical_service(pages, cumulative, count, run) -> int:
    pa = np.ascontiguousarray(pages, np.uint32)
    ca = np.ascontiguousarray(cumulative, np.uint64)
    return int(LIB.or_empirical_service_ns(_ptr(pa), _ptr(ca), count, run))


def update_burst(previous, page, op):
    """(packed, run_pages, valid) of hbf_device.cuh update_empirical_burst."""
    packed, run = ctypes.c_uint64(), ctypes.c_uint32()
    ok = LIB.or_update_empirical_burst(previous, page, op, ctypes.byref(packed),
                                       ctypes.byref(run))
    return packed.value, run.value, bool(ok)


def empirical_control_valid(e: Empirical) -> bool:
    return bool(LIB.or_empirical_control_valid(ctypes.byref(e)))


def empirical_request(e: Empirical, previous, page, op):
    """(service_ns, packed, run_pages, valid) of empirical_request_service."""
    svc, packed, run = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint32()
    ok = LIB.or_empirical_request_service(ctypes.byref(e), previous, page, op,
                                          ctypes.byref(svc), ctypes.byref(packed),
                                          ctypes.byref(run))
    return svc.value, packed.value, run.value, bool(ok)


def run_empirical(ranges, count, e: Empirical, time_scale, request_timeout_ns, address,
                  nbytes, op, arrival, state):
    """One batch of the empirical FAST model; state = [tail, packed burst]
    (uint64[2]) updated in place.  Returns (done, latency, status, stats)."""
    n = address.size
    done = np.zeros(n, np.uint64)
    latency = np.zeros(n, np.uint64)
    status = np.zeros(n, np.uint8)
    stats = Stats()
    rc = LIB.or_run_empirical_batch(
        ctypes.cast(ranges, ctypes.c_void_p), count, ctypes.byref(e), time_scale,
        request_timeout_ns, _ptr(address), _ptr(nbytes), _ptr(op), _ptr(arrival), n,
        _ptr(state), _ptr(done), _ptr(latency), _ptr(status), ctypes.byref(stats))
    if rc != 0:
        raise MemoryError("oracle allocation failed")
    return done, latency, status, {f: getattr(stats, f) for f, _ in Stats._fields_}


class PrefetchCell(ctypes.Structure):
    _fields_ = [("policy", ctypes.c_uint32), ("lead_distance", ctypes.c_uint32),
                ("accuracy", ctypes.c_double), ("buffer_pages", ctypes.c_uint32),
                ("max_in_flight", ctypes.c_uint32), ("read_latency_ns", ctypes.c_uint64),
                ("compute_ns_per_access", ctypes.c_uint64), ("seed", ctypes.c_uint64)]


PREFETCH_STATS = ("total_ns", "stall_ns", "demand_accesses", "demand_misses",
                  "prefetch_hits", "prefetch_issued", "prefetch_wasted")


def prefetch_run(pages: np.ndarray, cell: dict) -> tuple:
    """The prefetch model on one cell; returns the 7 stats in PREFETCH_STATS
    order."""
    c = PrefetchCell(cell["policy"], cell["lead"], cell["accuracy"], cell["buffer"],
                     cell["in_flight"], cell["read_ns"], cell["compute_ns"], cell["seed"])
    out = (ctypes.c_uint64 * 7)()
    pages = np.ascontiguousarray(pages, np.uint64)
    if LIB.or_prefetch_run(_ptr(pages), pages.size, ctypes.byref(c), out) != 0:
        raise MemoryError("oracle allocation failed")
    return tuple(int(v) for v in out)


class LinkProfile(ctypes.Structure):
    _fields_ = [("gt_per_second", ctypes.c_uint32), ("initial_ar_granules", ctypes.c_uint32),
                ("initial_r_granules", ctypes.c_uint32), ("max_accepted", ctypes.c_uint32),
                ("propagation_ns", ctypes.c_uint64), ("consume_ns", ctypes.c_uint64 * 2)]


class LinkResult(ctypes.Structure):
    _fields_ = [("counters", (ctypes.c_uint64 * 8) * 2), ("now", ctypes.c_uint64),
                ("ar_credits", ctypes.c_uint32), ("r_credits", ctypes.c_uint32),
                ("heap_peak", ctypes.c_uint64)]


def link_run(profile: dict, direction: np.ndarray, ready: np.ndarray):
    """The UCIe streaming link under the batch driver; returns (delivered
    ticks, counters [2][8], now, ar_credits, r_credits)."""
    p = LinkProfile(profile["gt"], profile["ar"], profile["r"], profile["accepted"],
                    profile["prop"], (ctypes.c_uint64 * 2)(*profile["consume"]))
    direction = np.ascontiguousarray(direction, np.uint8)
    ready = np.ascontiguousarray(ready, np.uint64)
    delivered = np.zeros(ready.size, np.uint64)
    out = LinkResult()
    if LIB.or_link_run(ctypes.byref(p), _ptr(direction), _ptr(ready), ready.size,
                       _ptr(delivered), ctypes.byref(out)) != 0:
        raise ValueError("link overflow")
    counters = np.array([[out.counters[d][k] for k in range(8)] for d in range(2)], np.uint64)
    link_run.heap_peak = out.heap_peak
    return delivered, counters, out.now, out.ar_credits, out.r_credits


def cores() -> int:
    return os.cpu_count() or 1
