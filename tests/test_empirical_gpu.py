"""GPU parity of the FAST model with an empirical burst-curve profile
(reference: the empirical branch of resolve_fast_or_hybrid,
src/cuda_runtime/device/hbf_device.cu:797-838, with hbf_device.cuh:959-1140).

Completion ticks, latencies, statuses, the carried state (channel tail and
packed burst state) and the counters are compared bit for bit with the oracle
(oracle/hbf_oracle.c or_run_empirical_batch), itself pinned to the
reference's functions by tests/golden/device_goldens.jsonl; the reference's
own fast-path traces are replayed through the CUDA path directly.
"""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

import hbf_oracle as ho
from helpers import Setup, make_context, oracle_ranges, to_device
from hbfsim_b200 import _lib
from hbfsim_b200 import workloads as wl

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "device_goldens.jsonl"
RANGE = 15 * wl.GIB
U64MAX = (1 << 64) - 1


def setup_for(profile, ranges=None):
    s = Setup(profile=profile, model=1, stacks=1, stripe=4096)
    s.ranges = ranges or [(wl.RANGE_BASE, RANGE, 1, 3)]
    return s


class EmpiricalOracle:
    """Oracle state across batches for one empirical Setup."""

    def __init__(self, setup, request_timeout_ns=1_000_000_000):
        p = setup.profile
        curve = p["empirical_vmem"]["read_curve"]
        self.e = ho.make_empirical([c["pages"] for c in curve],
                                   [c["cumulative_ns"] for c in curve],
                                   p["program_latency_ns"])
        self.ranges, self.count = oracle_ranges(setup)
        self.scale = p["time_scale"]
        self.timeout = request_timeout_ns
        self.state = np.zeros(2, np.uint64)
        self.stats = {}

    def run(self, address, nbytes, op, arrival):
        out = ho.run_empirical(self.ranges, self.count, self.e, self.scale, self.timeout,
                               address, nbytes, op, arrival, self.state)
        for k, v in out[3].items():
            self.stats[k] = (self.stats.get(k, 0) + v) % (1 << 64) if k != "max_done" \
                else max(self.stats.get(k, 0), v)
        return out


def submit(ctx, arrays):
    import torch
    out = ctx.submit(*to_device(arrays))
    torch.cuda.synchronize()
    return (out.done_ns.cpu().numpy().view(np.uint64),
            out.latency_ns.cpu().numpy().view(np.uint64), out.status.cpu().numpy())


def same(got, want, what):
    gd, gl, gs = got
    wd, wl_, ws = want[:3]
    bad = np.flatnonzero(gs != ws)
    assert bad.size == 0, f"{what}: status at {bad[:5]}: {gs[bad[:5]]} vs {ws[bad[:5]]}"
    bad = np.flatnonzero(gd != wd)
    assert bad.size == 0, f"{what}: done at {bad[:5]}: {gd[bad[:5]]} vs {wd[bad[:5]]}"
    assert np.array_equal(gl, wl_), what


def test_reference_fast_path_traces(tmp_path):
    """The reference's empirical fast path, computed by its own helpers
    (golden traces), replayed through the CUDA kernels: a sequential-heavy
    trace on the cd8p curve, a random curve with time_scale 7, one whose tail
    and arrivals saturate at 2^64 - 1 (the exact fallback kernel) and a curve
    ending at 1023 pages."""
    traces = [json.loads(l) for l in GOLDEN.read_text().splitlines() if '"emp_trace"' in l]
    assert len(traces) == 4
    for k, rec in enumerate(traces):
        profile = wl.vmem_profile(rec["pages"], rec["cum"], rec["program"], rec["scale"])
        ctx = make_context(setup_for(profile, [(wl.RANGE_BASE, wl.GIB, 1, 3)]),
                           str(tmp_path / f"t{k}"))
        assert ctx.state_words() == 2
        ctx.set_state(np.array([rec["tail0"], 0], np.uint64))
        steps = rec["steps"]
        page = np.array([s[1] for s in steps], np.uint64)
        arrays = ((wl.RANGE_BASE + page * 4096).astype(np.uint64),
                  np.full(page.size, 256, np.uint32),
                  np.array([s[2] for s in steps], np.uint8),
                  np.array([s[0] for s in steps], np.uint64))
        done, latency, status = submit(ctx, arrays)
        assert np.all(status == 1), f"trace {k}"
        assert done.tolist() == [s[4] for s in steps], f"trace {k}"
        assert np.array_equal(latency, done - arrays[3])
        stats = ctx.batch_stats()
        assert stats["fast_modeled_ns"] == sum(s[5] for s in steps) % (1 << 64)
        assert ctx.get_stats()["fast_requests"] == len(steps)
        ctx.close()


def mixed(arrays, rng, frac=0.02):
    """Adds bypass (outside every range), zero-byte and page-straddling
    accesses to a trace."""
    address, nbytes, op, arrival = (a.copy() for a in arrays)
    n = address.size
    pick = rng.random(n)
    byp = pick < frac
    address[byp] = wl.HBM_BASE + rng.integers(0, 1 << 30, int(byp.sum())).astype(np.uint64)
    zero = (pick >= frac) & (pick < 1.5 * frac)
    nbytes[zero] = 0
    cross = (pick >= 1.5 * frac) & (pick < 2 * frac)
    address[cross] = address[cross] - address[cross] % 4096 + 4032
    nbytes[cross] = 128
    return address, nbytes, op, arrival


@pytest.mark.parametrize("n,batches,mean_run", [(20_000, 1, 1.5), (300_000, 3, 48.0),
                                                (2_000_000, 2, 700.0)])
def test_batches_match_oracle(tmp_path, n, batches, mean_run):
    rng = np.random.default_rng(n + batches)
    profile = wl.vmem_profile()
    setup = setup_for(profile)
    arrays = mixed(wl.vmem_trace(n, seed=batches, mean_run=mean_run), rng)
    ctx = make_context(setup, str(tmp_path))
    oracle = EmpiricalOracle(setup)
    cuts = np.sort(rng.choice(np.arange(1, n), batches - 1, replace=False))
    for k, (lo, hi) in enumerate(zip(np.r_[0, cuts], np.r_[cuts, n])):
        part = tuple(a[lo:hi] for a in arrays)
        same(submit(ctx, part), oracle.run(*part), f"batch {k}")
        assert np.array_equal(ctx.get_state(), oracle.state), f"batch {k}: state"
    stats = ctx.batch_stats()
    for key, okey in (("modeled", "modeled"), ("bypass", "bypass"),
                      ("unsupported", "unsupported"), ("fast_modeled_ns", "fast_modeled_ns"),
                      ("max_done_ns", "max_done"), ("latency_sum_ns", "latency_sum")):
        assert stats[key] == oracle.stats[okey], key
    assert stats["batches"] == batches and stats["device_errors"] == 0
    ctx.close()


def test_long_streaks_cross_tiles_and_ctas(tmp_path):
    """Runs longer than the 1023-page cap, across many tiles and CTA ranges,
    with an operation switch at the same next page (a new run) and a state
    carried into a second batch in the middle of a streak."""
    n = 3_000_000
    page = np.arange(n, dtype=np.uint64) + 17
    page[1_500_000:] += 5  # one break
    op = np.zeros(n, np.uint8)
    op[2_000_000:2_000_100] = 1
    arrival = np.cumsum(np.random.default_rng(2).integers(0, 4, n)).astype(np.uint64)
    arrays = ((wl.RANGE_BASE + page * 4096).astype(np.uint64), np.full(n, 4096, np.uint32),
              op, arrival)
    setup = setup_for(wl.vmem_profile())
    ctx = make_context(setup, str(tmp_path))
    oracle = EmpiricalOracle(setup)
    for lo, hi in ((0, 1_234_567), (1_234_567, n)):
        part = tuple(a[lo:hi] for a in arrays)
        same(submit(ctx, part), oracle.run(*part), f"[{lo}, {hi})")
        assert np.array_equal(ctx.get_state(), oracle.state)
    assert int(oracle.state[1]) & 1023 == 1023
    ctx.close()


def test_invalid_control_header_is_unsupported(tmp_path):
    """A curve that passes profile validation but not the device control
    check (first breakpoint 0 pages): every timed access is Unsupported, as
    in the reference (hbf_device.cu:773-777); bypass stays bypass."""
    profile = wl.vmem_profile(pages=(0, 4, 16, 64, 256, 512))
    setup = setup_for(profile)
    rng = np.random.default_rng(3)
    arrays = mixed(wl.vmem_trace(50_000, seed=3), rng, frac=0.1)
    ctx = make_context(setup, str(tmp_path))
    oracle = EmpiricalOracle(setup)
    want = oracle.run(*arrays)
    assert set(np.unique(want[2]).tolist()) == {6, 8}
    same(submit(ctx, arrays), want, "invalid header")
    ctx.close()


def test_saturating_batch_takes_the_exact_kernel(tmp_path):
    """time_scale near 2^32: the host's bound fails, the single-thread kernel
    times the batch with saturating arithmetic (ticks reach 2^64 - 1)."""
    setup = setup_for(wl.vmem_profile(time_scale=4_000_000_000))
    arrays = wl.vmem_trace(20_000, seed=4, write_p=0.8)
    ctx = make_context(setup, str(tmp_path))
    oracle = EmpiricalOracle(setup)
    want = oracle.run(*arrays)
    assert int(want[0].max()) == U64MAX
    same(submit(ctx, arrays), want, "saturating")
    assert np.array_equal(ctx.get_state(), oracle.state)
    ctx.close()


def test_out_of_order_batch_is_refused(tmp_path):
    """A batch whose arrivals go backwards is refused on the device: the
    state and counters stay as they were, the refusal is counted."""
    setup = setup_for(wl.vmem_profile())
    ctx = make_context(setup, str(tmp_path))
    first = wl.vmem_trace(40_000, seed=5)
    submit(ctx, first)
    before = ctx.get_state().copy()
    bad = wl.vmem_trace(40_000, seed=6)
    arrival = bad[3].copy()
    arrival[20_000:] = arrival[20_000:] // 2
    submit(ctx, (bad[0], bad[1], bad[2], arrival))
    assert np.array_equal(ctx.get_state(), before)
    stats = ctx.batch_stats()
    assert stats["device_errors"] == 1 and stats["modeled"] == 40_000
    with pytest.raises(Exception):
        ctx.flush()  # the refusal is reported once
    ctx.flush()
    ctx.close()


def test_static_entry_point_matches(tmp_path):
    """The no-allocation entry point runs the same kernels for an empirical
    context (scratch allocated with the context)."""
    import torch
    setup = setup_for(wl.vmem_profile())
    arrays = mixed(wl.vmem_trace(200_000, seed=7), np.random.default_rng(7))
    ctx = make_context(setup, str(tmp_path))
    oracle = EmpiricalOracle(setup)
    lib = _lib.load()
    dev = to_device(arrays)
    n = arrays[0].size
    out = [torch.empty(n, dtype=torch.int64, device="cuda"),
           torch.empty(n, dtype=torch.int64, device="cuda"),
           torch.empty(n, dtype=torch.uint8, device="cuda")]
    batch = _lib.AccessBatchV1(ctypes.sizeof(_lib.AccessBatchV1), 1, n,
                               dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(),
                               dev[3].data_ptr(), out[0].data_ptr(), out[1].data_ptr(),
                               out[2].data_ptr())
    stream = torch.cuda.current_stream().cuda_stream or 1
    assert lib.hbfsim_submit_access_batch_static_v1(ctx.handle, ctypes.byref(batch),
                                                    ctypes.c_void_p(stream)) == 0
    torch.cuda.synchronize()
    got = (out[0].cpu().numpy().view(np.uint64), out[1].cpu().numpy().view(np.uint64),
           out[2].cpu().numpy())
    same(got, oracle.run(*arrays), "static entry")
    ctx.close()


def test_element_offset_buffers(tmp_path):
    """Inputs starting one element into their arrays (8-, 4- and 1-byte
    offsets from the allocation): the same results as the oracle."""
    import torch
    setup = setup_for(wl.vmem_profile())
    arrays = mixed(wl.vmem_trace(70_001, seed=12), np.random.default_rng(12))
    ctx = make_context(setup, str(tmp_path))
    dev = tuple(t[1:] for t in to_device(arrays))
    out = ctx.submit(*dev)
    torch.cuda.synchronize()
    got = (out.done_ns.cpu().numpy().view(np.uint64), out.latency_ns.cpu().numpy().view(np.uint64),
           out.status.cpu().numpy())
    same(got, EmpiricalOracle(setup).run(*(a[1:] for a in arrays)), "offset buffers")
    ctx.close()
