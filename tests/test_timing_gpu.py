"""Parity of the CUDA timing path with the CPU oracle (bit-exact).

Every test runs the same seeded trace through libhbfsim_b200.so (C ABI) and
through oracle/libhbf_oracle.so and requires identical completion ticks,
latencies, statuses, carried state and counters.
"""
import numpy as np
import pytest

import hbf_oracle as ho
from helpers import OracleRun, Setup, assert_same, gpu_run, make_context, to_device
from hbfsim_b200 import workloads as wl

pytestmark = pytest.mark.gpu
GIB = 1 << 30


@pytest.fixture
def tmp(tmp_path):
    return str(tmp_path)


def c0_setup(model=3, **kw):
    s = Setup(profile=wl.c0_profile(), model=model, **kw)
    s.ranges = [(wl.RANGE_BASE, 64 * GIB, 1, 3)]
    return s


@pytest.mark.parametrize("model", [1, 3])
@pytest.mark.parametrize("n", [1, 31, 2048, 2049, 70001])
def test_c0_small_batches(tmp, model, n):
    s = c0_setup(model)
    ctx = make_context(s, tmp)
    arrays = wl.c0_trace(n, seed=n)
    ora = OracleRun(s)
    want = ora.run(*arrays)
    assert_same(gpu_run(ctx, arrays), want, f"model {model} n {n}")
    assert np.array_equal(ctx.get_state(), ora.state)
    st = ctx.batch_stats()
    assert st["modeled"] == want[3]["modeled"]
    assert st["max_done_ns"] == want[3]["max_done"]
    assert st["latency_sum_ns"] == want[3]["latency_sum"]
    if model == 1:
        assert ctx.get_stats()["fast_modeled_ns"] == want[3]["fast_modeled_ns"]
    ctx.close()


@pytest.mark.parametrize("model", [1, 3])
def test_c0_full_config(tmp, model):
    """BASELINE config 0 at its full size: 1,048,576 accesses."""
    s = c0_setup(model)
    ctx = make_context(s, tmp)
    arrays = wl.c0_trace(1 << 20, seed=0)
    ora = OracleRun(s)
    want = ora.run(*arrays, threads=8)
    assert_same(gpu_run(ctx, arrays), want, "c0 full")
    assert np.array_equal(ctx.get_state(), ora.state)
    assert ctx.simulated_time() == want[3]["max_done"]
    ctx.close()


def test_batches_carry_state(tmp):
    """Splitting a trace into ragged batches gives the single-batch result."""
    s = c0_setup(3)
    ctx = make_context(s, tmp)
    arrays = wl.c0_trace(50000, seed=5)
    ora = OracleRun(s)
    want = ora.run(*arrays)
    got = []
    for lo, hi in [(0, 1), (1, 4097), (4097, 4100), (4100, 33333), (33333, 50000)]:
        got.append(gpu_run(ctx, tuple(a[lo:hi] for a in arrays)))
    cat = tuple(np.concatenate([g[k] for g in got]) for k in range(3))
    assert_same(cat, want, "batched")
    assert np.array_equal(ctx.get_state(), ora.state)


def test_statuses_multi_range(tmp):
    """Bypass, straddle, cross-page, permission, bad op, zero bytes and a
    capacity-mode range, across several ranges with gaps."""
    s = Setup(profile=wl.c0_profile(), model=3, stacks=2, stripe=8192)
    page = 16384
    base = 1 << 40
    s.ranges = [(base, 5 * page + 100, 1, 3), (base + 8 * page, 3 * page, 1, 1),
                (base + 16 * page, 2 * page, 2, 3), (base + 20 * page, 40 * page, 1, 2)]
    ctx = make_context(s, tmp)
    rng = np.random.default_rng(11)
    n = 20000
    addr = base - page + rng.integers(0, 64 * page, n).astype(np.uint64)
    nbytes = rng.choice(np.array([0, 1, 8, 128, 4096, 9000], np.uint32), n)
    op = rng.choice(np.array([0, 1, 2], np.uint8), n, p=[0.6, 0.35, 0.05])
    arrival = np.cumsum(rng.integers(0, 50, n)).astype(np.uint64)
    ora = OracleRun(s)
    want = ora.run(addr, nbytes, op, arrival)
    got = gpu_run(ctx, (addr, nbytes, op, arrival))
    assert_same(got, want, "statuses")
    kinds = set(np.unique(got[2]).tolist())
    assert {1, 6, 8} <= kinds


def test_misaligned_buffers(tmp):
    s = c0_setup(3)
    ctx = make_context(s, tmp)
    import torch
    arrays = wl.c0_trace(9000, seed=3)
    dev = to_device(arrays)
    sl = tuple(t[1:] for t in dev)  # 8/4/1-byte offsets: scalar path
    out = ctx.submit(*sl)
    torch.cuda.synchronize()
    ora = OracleRun(s)
    want = ora.run(*(a[1:] for a in arrays))
    got = (out.done_ns.cpu().numpy().view(np.uint64), out.latency_ns.cpu().numpy().view(np.uint64),
           out.status.cpu().numpy())
    assert_same(got, want, "misaligned")


def test_unsorted_batch_refused(tmp):
    s = c0_setup(3)
    ctx = make_context(s, tmp)
    arrays = wl.c0_trace(5000, seed=1)
    gpu_run(ctx, arrays)
    before = ctx.get_state()
    bad = list(arrays)
    bad[3] = bad[3].copy()
    bad[3][100], bad[3][101] = bad[3][101] + 5, bad[3][100]
    gpu_run(ctx, tuple(bad))
    from hbfsim_b200 import HbfsimError
    with pytest.raises(HbfsimError):
        ctx.flush()
    assert np.array_equal(ctx.get_state(), before)
    assert ctx.batch_stats()["device_errors"] == 1
    # a batch that goes back in time relative to the previous batch
    gpu_run(ctx, tuple(a[:10] for a in arrays))
    with pytest.raises(HbfsimError):
        ctx.flush()


@pytest.mark.parametrize("model", [1, 3])
def test_saturating_sequential_path(tmp, model):
    """Arrivals near 2^64 take the exact saturating kernel."""
    s = c0_setup(model)
    ctx = make_context(s, tmp)
    addr, nbytes, op, _ = wl.c0_trace(3000, seed=9)
    arrival = (np.uint64(2**64 - 400_000) +
               np.cumsum(np.full(3000, 100, np.uint64))).astype(np.uint64)
    op[-100:] = 1  # writes: a + tPROG passes 2^64 and saturates
    ora = OracleRun(s)
    want = ora.run(addr, nbytes, op, arrival)
    assert_same(gpu_run(ctx, (addr, nbytes, op, arrival)), want, "saturating")
    assert (want[0] == np.uint64(2**64 - 1)).any()
    assert np.array_equal(ctx.get_state(), ora.state)


def test_deep_backlog_and_long_gaps(tmp):
    """The chains replay a channel's accesses in 32-bit words relative to a
    base while every word of the tile stays within 2^31 of it, else in 64
    bits.  Three phases in one batch: 800,000 accesses (90 % writes) at one
    arrival, whose die queues run seconds ahead of the arrivals (the unit
    step once the queue is 2^30 past the arrivals); arrivals with a 3e9-tick
    gap every 300 accesses (tiles span more than 2^31, and the arrivals
    overtake the queue inside a segment); then the usual gaps."""
    s = c0_setup(3, stacks=1)
    ctx = make_context(s, tmp)
    deep, gapped = 800_000, 150_000
    n = deep + 2 * gapped
    addr, nbytes, op, _ = wl.c0_trace(n, seed=21)
    rng = np.random.default_rng(22)
    op[:deep] = (rng.random(deep) < 0.9).astype(np.uint8)
    gaps = np.zeros(n, np.uint64)
    gaps[0] = 1000
    gaps[deep:deep + gapped:300] = 3_000_000_000
    gaps[deep + gapped:] = np.rint(rng.exponential(2.0, gapped)).astype(np.uint64)
    arrival = np.cumsum(gaps, dtype=np.uint64)
    ora = OracleRun(s)
    want = ora.run(addr, nbytes, op, arrival, threads=4)
    assert want[1][:deep].max() > (1 << 31)  # the queues outgrew the 32-bit window
    assert_same(gpu_run(ctx, (addr, nbytes, op, arrival)), want, "backlog and gaps")
    assert np.array_equal(ctx.get_state(), ora.state)
    # the same accesses again, the carried state far ahead of the new arrivals
    arrival2 = arrival + arrival[-1] + np.uint64(1)
    want2 = ora.run(addr, nbytes, op, arrival2, threads=4)
    assert_same(gpu_run(ctx, (addr, nbytes, op, arrival2)), want2, "second batch")
    assert np.array_equal(ctx.get_state(), ora.state)
    ctx.close()


def test_chain_window_boundaries(tmp):
    """Carried states placed around the edges of the 32-bit chain window:
    channel c starts with its queue at first arrival + delta[c], deltas from
    far below the arrivals to 2^32 above them, around 2^30 (where the
    arrivals stop counting unless they overtake the queue) and 2^31 (where
    the window ends).  Arrival jumps of 1.5e9 and 3e9 ticks inside tiles let
    arrivals overtake the queues mid-segment.  Every channel's result must
    equal the oracle's, whichever replay each segment takes."""
    s = c0_setup(3, stacks=1)
    ctx = make_context(s, tmp)
    C, K = s.local_channels, s.k
    a0 = 10**12
    deltas = [-(2**31) - 5, -(2**30), -5, 0, 1, 2**20, 2**30 - 2, 2**30 - 1, 2**30, 2**30 + 1,
              2**30 + 2**29, 2**31 - 2**25, 2**31 - 1, 2**31, 2**31 + 7, 2**32]
    assert len(deltas) == C
    state = np.zeros(C * K, np.uint64)
    for c, dl in enumerate(deltas):
        chan = a0 + dl
        state[c * K] = chan
        for j in range(1, K):
            state[c * K + j] = max(0, chan + 1000 * j - 2000)
    n = 20_000
    addr, nbytes, op, _ = wl.c0_trace(n, seed=31)
    arrival = a0 + np.arange(n, dtype=np.uint64)
    arrival[5000:] += np.uint64(1_500_000_000)
    arrival[12_000:] += np.uint64(3_000_000_000)
    ctx.set_state(state)
    ora = OracleRun(s)
    ora.state[:] = state
    want = ora.run(addr, nbytes, op, arrival)
    assert_same(gpu_run(ctx, (addr, nbytes, op, arrival)), want, "window boundaries")
    assert np.array_equal(ctx.get_state(), ora.state)
    ctx.close()


def test_refresh_throttle_admit_factors(tmp):
    s = c0_setup(3, stacks=2)
    ctx = make_context(s, tmp)
    rng = np.random.default_rng(4)
    refresh = rng.integers(0, 400, s.local_channels).astype(np.uint32)
    throttle = np.array([1000, 1750], np.uint32)
    admit = np.array([0, 150_000], np.uint64)
    ctx.set_channel_factors(refresh, throttle, admit)
    arrays = wl.c0_trace(40000, seed=8)
    ora = OracleRun(s, refresh, throttle, admit)
    assert_same(gpu_run(ctx, arrays), ora.run(*arrays), "factors")
    r, t, a = ctx.channel_factors(s.local_channels, s.stacks)
    assert np.array_equal(r, refresh) and np.array_equal(t, throttle) and np.array_equal(a, admit)


def test_transfer_quotients_every_size_and_rate(tmp):
    """ceil(bytes * 1e9 / bw) for channel rates that are not 1e9 * 2^k: the
    quotient is estimated with the channel's fp64 reciprocal and settled with
    the remainder.  Every access size from 1 byte to a whole page on channels
    whose refresh shares (0..900 permille) leave odd rates (refresh 0 keeps
    the shift path), against the oracle's integer division."""
    s = c0_setup(3, stacks=2)
    ctx = make_context(s, tmp)
    rng = np.random.default_rng(77)
    refresh = rng.integers(0, 901, s.local_channels).astype(np.uint32)
    refresh[:4] = [0, 1, 500, 900]
    ctx.set_channel_factors(refresh, None, None)
    page = s.profile["page_bytes"]
    n = 60_000
    size = np.concatenate([np.arange(1, page + 1), rng.integers(1, page + 1, n - page)])
    size = size[:n].astype(np.uint32)
    pages = rng.integers(0, (64 * GIB) // page, n, dtype=np.int64)
    address = (wl.RANGE_BASE + pages * page).astype(np.uint64)
    op = (rng.random(n) < 0.1).astype(np.uint8)
    arrival = np.cumsum(rng.integers(0, 40, n)).astype(np.uint64)
    arrays = (address, size, op, arrival)
    ora = OracleRun(s, refresh, None, None)
    want = ora.run(*arrays)
    assert (want[2] == 1).all()
    assert_same(gpu_run(ctx, arrays), want, "transfer quotients")
    ctx.close()


def test_channel_shards_partition_the_trace(tmp):
    """Each shard times only its channels; the union equals the unsharded run."""
    arrays = wl.c0_trace(30000, seed=12)
    full = OracleRun(c0_setup(3, stacks=4)).run(*arrays)
    merged_done = np.zeros_like(full[0])
    seen = np.zeros(full[0].size, bool)
    for rank in range(3):
        s = c0_setup(3, stacks=4, shard_rank=rank, shard_count=3)
        ctx = make_context(s, f"{tmp}/r{rank}")
        got = gpu_run(ctx, arrays)
        assert_same(got, OracleRun(s).run(*arrays), f"shard {rank}")
        mine = got[2] == 1
        merged_done[mine] = got[0][mine]
        assert not (seen & mine).any()
        seen |= mine
        ctx.close()
    modeled = full[2] == 1
    assert np.array_equal(seen, modeled)
    assert np.array_equal(merged_done[modeled], full[0][modeled])


@pytest.mark.parametrize("order,stacks,stripe", [("CWDP", 1, 4096), ("DPCW", 4, 512),
                                                 ("PCDW", 2, 16384), ("WDCP", 3, 2048)])
def test_decode_matches_oracle(tmp, order, stacks, stripe):
    import torch
    p = wl.c0_profile()
    p["plane_allocation_scheme"] = order
    s = Setup(profile=p, model=3, stacks=stacks, stripe=stripe)
    s.ranges = [(wl.RANGE_BASE, 60 * GIB, 1, 3), (wl.RANGE_BASE + 80 * GIB, GIB, 1, 1)]
    ctx = make_context(s, tmp)
    rng = np.random.default_rng(2)
    n = 50000
    addr = (wl.RANGE_BASE + rng.integers(0, 82 * GIB, n)).astype(np.uint64)
    nbytes = rng.choice(np.array([1, 128, 4096], np.uint32), n)
    op = rng.integers(0, 2, n).astype(np.uint8)
    dev = to_device((addr, nbytes, op, np.zeros(n, np.uint64)))
    raw = ctx.decode(dev[0], dev[1], dev[2])
    torch.cuda.synchronize()
    dt = np.dtype([("media_address", "<u8"), ("page", "<u8"), ("status", "<u4"),
                   ("range_index", "<u4"), ("stack", "<u4"), ("channel", "<u4"),
                   ("die", "<u4"), ("plane", "<u4")])
    got = np.frombuffer(raw.cpu().numpy().tobytes(), dtype=dt)
    ora = OracleRun(s)
    want = ho.decode(ora.ranges, ora.count, ora.geometry, addr, nbytes, op)
    for f in ("status", "media_address"):
        assert np.array_equal(got[f], want[f]), f
    m = want["status"] == 1
    for f in ("range_index", "stack", "channel", "die", "plane", "page"):
        assert np.array_equal(got[f][m], want[f][m]), f


@pytest.mark.parametrize("kind", ["bank", "stripe"])
def test_decode_against_reference_layout(tmp, golden_dir, kind):
    """The device decode (hbfsim_decode_batch_v1) against goldens from the
    reference's own UCIe layout functions (bank_layout.cpp
    hbf_cold_read_bank, stack_router.cpp page-striped placement)."""
    import torch
    from helpers import (DECODE_DTYPE, bank_layout_cases, check_layout_decode,
                         layout_goldens, stripe_layout_cases)
    golden = layout_goldens(golden_dir)
    gen = bank_layout_cases if kind == "bank" else stripe_layout_cases
    for k, case in enumerate(gen(golden)):
        ctx = make_context(case[0], f"{tmp}/{k}")
        dev = to_device((*case[1:4], np.zeros(case[1].size, np.uint64)))
        raw = ctx.decode(dev[0], dev[1], dev[2])
        torch.cuda.synchronize()
        got = np.frombuffer(raw.cpu().numpy().tobytes(), dtype=DECODE_DTYPE)
        check_layout_decode(got, case, kind)
        ctx.close()


def test_c1_slice_parity(tmp):
    """A slice of the MoE decode trace (config 1 shape, 4 stacks)."""
    s = Setup(profile=wl.c0_profile(), model=3, stacks=4, stripe=4096)
    s.ranges = [(wl.RANGE_BASE, 60 * GIB, 1, 1)]
    ctx = make_context(s, tmp)
    bases, counts = wl.c1_segments(seed=1, steps=1, layers=3)
    arrays = wl.expand_segments(bases, counts)
    want = OracleRun(s).run(*arrays, threads=8)
    got = gpu_run(ctx, arrays)
    assert_same(got, want, "c1 slice")
    assert (got[2] == 8).sum() == 3 * 16384  # attention weights bypass to HBM


def test_checkpoint_resume_bit_exact(tmp):
    s = c0_setup(3)
    arrays = wl.c0_trace(20000, seed=21)
    first = tuple(a[:9000] for a in arrays)
    second = tuple(a[9000:] for a in arrays)
    ctx = make_context(s, tmp)
    gpu_run(ctx, first)
    saved = ctx.get_state()
    r1 = gpu_run(ctx, second)
    ctx2 = make_context(s, f"{tmp}/b")
    ctx2.set_state(saved)
    # the resumed context must also know the last arrival ordering
    r2 = gpu_run(ctx2, second)
    assert_same(r2, (r1[0], r1[1], r1[2]), "resume")


def test_host_buffer_path_matches_device_path(tmp):
    import torch
    s = c0_setup(3)
    arrays = wl.c0_trace(300000, seed=30)
    ctx = make_context(s, tmp)
    want = OracleRun(s).run(*arrays)
    pinned = [torch.from_numpy(a.view({8: np.int64, 4: np.int32, 1: np.uint8}[a.itemsize]))
              .pin_memory() for a in arrays]
    out = ctx.submit_host(*pinned)
    assert_same((out.done_ns, out.latency_ns, out.status), want, "host path")


@pytest.mark.parametrize("dies,stacks,channels", [(1, 1, 16), (2, 2, 16), (3, 1, 16), (8, 1, 16),
                                                  (4, 16, 16), (8, 4, 16), (8, 1, 8),
                                                  (4, 1, 4)])
def test_kernel_variants(tmp, dies, stacks, channels):
    """Direct (register) kernels for D in {1,2,4,8} with few channels, piece
    kernels for other D or many channels: all bit-exact.  With one tile per
    CTA and 2 C (D + 2) <= 256 (D = 8 on 8 channels, D = 4 on 4, D = 1 and 2
    on 16) each tile's halves are timed as two ranges."""
    p = wl.c0_profile()
    p["dies_per_channel"] = dies
    p["channels"] = channels
    p["capacity_bytes"] = p["page_bytes"] * channels * dies * 4 * 256 * 64
    s = Setup(profile=p, model=3, stacks=stacks, stripe=4096)
    s.ranges = [(wl.RANGE_BASE, p["capacity_bytes"] - (1 << 20), 1, 3)]
    ctx = make_context(s, tmp)
    arrays = wl.c0_trace(60000, seed=dies * 10 + stacks + channels,
                         range_length=p["capacity_bytes"] - (1 << 20))
    ora = OracleRun(s)
    assert_same(gpu_run(ctx, arrays), ora.run(*arrays, threads=4), f"D={dies} S={stacks}")
    assert np.array_equal(ctx.get_state(), ora.state)


def test_hybrid_sampler_bits(tmp):
    """A7: the sampler bit of every timed access, numbered across batches,
    against the reference predicate (hbf_device.cuh:738-744) restated in the
    oracle and applied in batch order."""
    import torch
    p = wl.c0_profile()
    p["reference_sample_rate"] = 0.3
    p["reference_warmup_requests"] = 700
    s = Setup(profile=p, model=3, stacks=2, stripe=4096)
    s.ranges = [(wl.RANGE_BASE, 8 << 30, 1, 3), (wl.RANGE_BASE + (16 << 30), 4 << 30, 1, 1)]
    ctx = make_context(s, tmp)
    oracle = OracleRun(s)
    thr = ho.LIB.or_sample_threshold(0.3)
    seq = 0
    for k, n in enumerate((5000, 12345)):
        arrays = wl.c0_trace(n, seed=40 + k, range_length=24 << 30)
        dev = to_device(arrays)
        got = ctx.sample(dev[0], dev[1], dev[2]).cpu().numpy()
        torch.cuda.synchronize()
        dec = ho.decode(oracle.ranges, oracle.count, oracle.geometry, *arrays[:3])
        want = np.zeros(n, np.uint8)
        for i in np.flatnonzero(dec["status"] == 1):
            rid = oracle.ranges[int(dec["range_index"][i])].range_id
            key = int(dec["media_address"][i]) ^ (rid << 32) ^ int(arrays[2][i])
            want[i] = ho.LIB.or_hybrid_reference_sample(seq, 700, thr, key)
            seq += 1
        assert np.array_equal(got, want), f"batch {k}"
        assert 0 < want.sum() < (dec["status"] == 1).sum()
    ctx.close()


@pytest.mark.parametrize("rank,shards", [(0, 8), (5, 8), (1, 2)])
def test_config4_shard(tmp, rank, shards):
    """Config-4 geometry (16 stacks x 16 channels x 8 dies x 4 planes) as one
    rank of an N-GPU run: a mixed trace of the config-1 (expert streaming)
    and config-2 (paged KV) patterns interleaved by arrival; the rank times
    its channels bit-exactly and marks the others' accesses foreign."""
    p = wl.c4_profile()
    s = Setup(profile=p, model=3, stacks=16, stripe=4096, shard_rank=rank, shard_count=shards)
    s.ranges = [(wl.RANGE_BASE, 120 << 30, 1, 3)]
    rng = np.random.default_rng(rank + 10 * shards)
    bases, counts = wl.c1_segments(seed=rank, steps=1, layers=2)
    moe = wl.expand_segments(bases, counts)
    lengths = wl.c2_lengths(seed=rank, seqs=32, lmin=512, lmax=2048)
    kv_addr, kv_bytes, kv_op = wl.c2_step(lengths, 0, 4, layers=2, base=wl.RANGE_BASE + (64 << 30))
    n1, n2 = moe[0].size, kv_addr.size
    # interleave by arrival: 60 % expert reads, 40 % KV page accesses
    take = min(n1, int(n2 * 1.5))
    order = np.argsort(np.r_[np.arange(take) / 0.6, np.arange(int(take / 1.5)) / 0.4],
                       kind="stable")
    address = np.r_[moe[0][:take], kv_addr[:int(take / 1.5)]][order]
    nbytes = np.r_[moe[1][:take], kv_bytes[:int(take / 1.5)]][order]
    op = np.r_[moe[2][:take], kv_op[:int(take / 1.5)]][order]
    arrival = np.arange(address.size, dtype=np.uint64)
    arrays = (address.astype(np.uint64), nbytes.astype(np.uint32), op.astype(np.uint8), arrival)
    ctx = make_context(s, tmp)
    ora = OracleRun(s)
    got = gpu_run(ctx, arrays)
    want = ora.run(*arrays, threads=8)
    assert_same(got, want, f"c4 rank {rank}/{shards}")
    assert (want[2] == 9).sum() > 0 and (want[2] == 1).sum() > 0
    assert np.array_equal(ctx.get_state(), ora.state)
