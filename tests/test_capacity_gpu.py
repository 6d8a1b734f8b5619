"""GPU parity of Capacity mode (A4): exact-LRU hit / victim / victim-dirty
decisions of the batch-parallel kernels against the oracle's sequential LRU
(oracle/hbf_oracle.c or_lru_run, itself pinned to the reference LruCache by
tests/golden/lru_goldens.json), bit for bit, across batches that carry the
resident list."""
import json
from pathlib import Path

import numpy as np
import pytest

import hbf_oracle as ho
from helpers import Setup, make_context
from hbfsim_b200 import workloads as wl

pytestmark = pytest.mark.gpu

PAGE = 4096
GOLDEN = Path(__file__).resolve().parent / "golden" / "lru_goldens.json"
NONE = (1 << 64) - 1


def capacity_context(tmp, frames, capacity_gib=64):
    p = wl.c0_profile()
    p["capacity_bytes"] = capacity_gib << 30
    s = Setup(profile=p, model=3, stacks=1, stripe=4096)
    s.ranges = [(wl.RANGE_BASE, (capacity_gib - 1) << 30, 2, 3)]
    ctx = make_context(s, tmp)
    ctx.capacity_configure(frames, PAGE)
    return ctx


def to_accesses(pages, writes, rng):
    off = rng.integers(0, PAGE // 128, pages.size) * 128
    address = (wl.RANGE_BASE + pages.astype(np.uint64) * PAGE + off.astype(np.uint64))
    nbytes = np.minimum(rng.choice([128, 512, 4096], pages.size), PAGE - off).astype(np.uint32)
    return address.astype(np.uint64), nbytes, writes.astype(np.uint8)


def run_gpu(ctx, address, nbytes, op):
    import torch
    dev = [torch.from_numpy(address.view(np.int64)).cuda(),
           torch.from_numpy(nbytes.view(np.int32)).cuda(), torch.from_numpy(op).cuda()]
    hit, victim, dirty, status = ctx.submit_capacity(*dev)
    return (hit.cpu().numpy(), victim.cpu().numpy().view(np.uint64), dirty.cpu().numpy(),
            status.cpu().numpy())


def check(got, want, what):
    hit, victim, dirty, status = got
    assert np.all(status == 1), what
    bad = np.flatnonzero(hit != want[0])
    assert bad.size == 0, f"{what}: hit differs at {bad[:5]}"
    bad = np.flatnonzero(victim != want[1])
    assert bad.size == 0, f"{what}: victim differs at {bad[:5]}: {victim[bad[:5]]} vs {want[1][bad[:5]]}"
    bad = np.flatnonzero(dirty != want[2])
    assert bad.size == 0, f"{what}: dirty differs at {bad[:5]}"


def test_reference_lru_goldens(tmp_path):
    rng = np.random.default_rng(0)
    for k, case in enumerate(json.loads(GOLDEN.read_text())):
        ctx = capacity_context(str(tmp_path / f"c{k}"), case["frames"])
        pages = np.array(case["keys"], np.uint64)
        got = run_gpu(ctx, *to_accesses(pages, np.zeros(pages.size, np.uint8), rng))
        assert got[0].tolist() == case["hits"], f"case {k}"
        victims = [NONE if v < 0 else v for v in case["victims"]]
        assert [int(v) for v in got[1]] == victims, f"case {k}"
        ctx.close()


def trace(rng, n, universe, locality):
    pages = np.empty(n, np.uint64)
    hot = rng.integers(0, universe, 64)
    for i in range(n):
        r = rng.random()
        if r < locality and i:
            pages[i] = pages[i - 1 - rng.integers(0, min(i, 48))]
        elif r < locality + 0.2:
            pages[i] = hot[rng.integers(0, hot.size)]
        else:
            pages[i] = rng.integers(0, universe)
    return pages


@pytest.mark.parametrize("frames,universe,n,batches", [(1, 5, 3000, 3), (7, 40, 20000, 4),
                                                      (300, 2000, 60000, 5),
                                                      (5000, 4000, 40000, 2),
                                                      (2048, 1 << 20, 200000, 3)])
def test_lru_matches_oracle_across_batches(tmp_path, frames, universe, n, batches):
    rng = np.random.default_rng(frames + n)
    pages = trace(rng, n, universe, 0.4) if n <= 60000 else \
        np.where(rng.random(n) < 0.5, rng.integers(0, 4096, n), rng.integers(0, universe, n)).astype(np.uint64)
    writes = (rng.random(n) < 0.2).astype(np.uint8)
    want = ho.lru(pages, writes, frames)
    ctx = capacity_context(str(tmp_path), frames)
    cuts = np.sort(rng.choice(np.arange(1, n), batches - 1, replace=False))
    for k, (lo, hi) in enumerate(zip(np.r_[0, cuts], np.r_[cuts, n])):
        got = run_gpu(ctx, *to_accesses(pages[lo:hi], writes[lo:hi], rng))
        check(got, tuple(w[lo:hi] for w in want), f"batch {k}")
    resident, _ = ctx.capacity_state()
    assert resident.size == min(frames, np.unique(pages).size)
    ctx.close()


def test_cyclic_scan_larger_than_the_cache(tmp_path):
    """Config-2 shape, reduced: every step reads all KV pages in the same
    order (a scan larger than HBM: exact LRU misses every time) and appends."""
    rng = np.random.default_rng(4)
    blocks = rng.integers(64, 512, 16)
    steps, frames = 4, int(blocks.sum() * 0.2)
    pages, writes = [], []
    base = np.cumsum(np.r_[0, blocks[:-1] + steps])
    for t in range(steps):
        for s_, (b0, nb) in enumerate(zip(base, blocks)):
            pages.append(np.arange(b0, b0 + nb + t, dtype=np.uint64))
            w = np.zeros(nb + t, np.uint8)
            w[-1] = 1  # the appended token's page is written
            writes.append(w)
    pages = np.concatenate(pages)
    writes = np.concatenate(writes)
    want = ho.lru(pages, writes, frames)
    ctx = capacity_context(str(tmp_path), frames)
    got = run_gpu(ctx, *to_accesses(pages, writes, rng))
    check(got, want, "scan")
    assert want[0].sum() < pages.size * 0.05
    ctx.close()


def test_statuses_and_page_numbering(tmp_path):
    """Accesses outside capacity ranges are not cached; LRU pages count from
    each range's file offset; an access crossing an LRU page is refused."""
    p = wl.c0_profile()
    s = Setup(profile=p, model=3, stacks=1, stripe=4096)
    s.ranges = [(wl.RANGE_BASE, 1 << 30, 1, 3), (wl.RANGE_BASE + (4 << 30), 1 << 30, 2, 3)]
    ctx = make_context(s, str(tmp_path))
    ctx.capacity_configure(4, PAGE)
    cap = wl.RANGE_BASE + (4 << 30)
    address = np.array([wl.RANGE_BASE + 100, cap + 5 * PAGE, cap + 5 * PAGE + 8, cap + PAGE - 64,
                        wl.HBM_BASE, cap + 7 * PAGE], np.uint64)
    nbytes = np.array([128, 128, 128, 128, 128, 256], np.uint32)
    op = np.array([0, 1, 0, 0, 0, 0], np.uint8)
    hit, victim, dirty, status = run_gpu(ctx, address, nbytes, op)
    assert status.tolist() == [6, 1, 1, 6, 8, 1]
    assert hit.tolist() == [0, 0, 1, 0, 0, 0]
    first_page = (1 << 30) // PAGE  # the capacity range's file offset in pages
    pages, dirty_bits = ctx.capacity_state()
    assert pages.tolist() == [first_page + 5, first_page + 7]
    assert dirty_bits.tolist() == [1, 0]
    ctx.close()


@pytest.mark.parametrize("frames,write_p,n", [(256, 0.02, 60000), (64, 0.5, 30000)])
def test_media_action_timing_matches_oracle(tmp_path, frames, write_p, n):
    """Misses become media actions timed with the die model: the program of
    a dirty victim, then the chained read.  All actions of a batch are timed
    in parallel rounds that raise the chained reads to their programs'
    completions until none moves, or else in pieces that start at the
    chained reads."""
    import torch
    from helpers import OracleRun
    rng = np.random.default_rng(frames)
    pages = np.where(rng.random(n) < 0.6, rng.integers(0, 2 * frames, n),
                     rng.integers(0, 1 << 18, n)).astype(np.uint64)
    writes = (rng.random(n) < write_p).astype(np.uint8)
    address, nbytes, op = to_accesses(pages, writes, rng)
    arrival = np.cumsum(rng.exponential(20.0, n).astype(np.uint64) + 1).astype(np.uint64)
    hit_w, victim_w, dirty_w = ho.lru(pages, writes, frames)
    p = wl.c0_profile()
    p["capacity_bytes"] = 64 << 30
    s = Setup(profile=p, model=3, stacks=1, stripe=4096)
    s.ranges = [(wl.RANGE_BASE, 63 << 30, 2, 3)]
    oracle = OracleRun(s)
    ctx = capacity_context(str(tmp_path), frames)
    cut = n // 3
    for k, (lo, hi) in enumerate(((0, cut), (cut, n))):
        dev = [torch.from_numpy(address[lo:hi].view(np.int64)).cuda(),
               torch.from_numpy(nbytes[lo:hi].view(np.int32)).cuda(),
               torch.from_numpy(op[lo:hi]).cuda(),
               torch.from_numpy(arrival[lo:hi].view(np.int64)).cuda()]
        hit, victim, dirty, status, done, latency = ctx.submit_capacity(*dev, timed=True)
        done = done.cpu().numpy().view(np.uint64)
        latency = latency.cpu().numpy().view(np.uint64)
        assert np.array_equal(hit.cpu().numpy(), hit_w[lo:hi])
        want_done, want_lat = ho.capacity_timing(
            oracle.geometry, oracle.timing, oracle.chan_bw, oracle.t_read, oracle.t_prog,
            oracle.admit, np.ones(hi - lo, np.uint8), hit_w[lo:hi], pages[lo:hi],
            victim_w[lo:hi], dirty_w[lo:hi], arrival[lo:hi], 12, oracle.state)
        bad = np.flatnonzero(done != want_done)
        assert bad.size == 0, f"batch {k}: done differs at {bad[:5]}: {done[bad[:5]]} vs {want_done[bad[:5]]}"
        assert np.array_equal(latency, want_lat)
        chained = int((dirty_w[lo:hi] == 1).sum())
        assert chained > 0
        rounds, pieces, walked = ctx.capacity_rounds()
        assert rounds >= 2 and not walked
    assert np.array_equal(ctx.get_state(), oracle.state)
    ctx.close()


def test_config2_timed_steps_full_size(tmp_path):
    """Config 2 at full size: decode steps 0 and 1 of the Llama-3-8B-shaped
    paged-KV trace (about 3.5e7 page references each; HBM holds 20 % of the
    KV pages) through exact LRU with their media actions timed, bit-exact
    against the oracle (LRU decisions, then every access's completion)."""
    import torch
    from helpers import OracleRun
    lengths = wl.c2_lengths(0)
    frames = wl.c2_frames(lengths)
    p = wl.c0_profile()
    p["capacity_bytes"] = 160 << 30
    s = Setup(profile=p, model=3, stacks=1, stripe=4096)
    s.ranges = [(wl.RANGE_BASE, 150 << 30, 2, 3)]
    ctx = make_context(s, str(tmp_path))
    ctx.capacity_configure(frames, PAGE)
    oracle = OracleRun(s)
    steps = [wl.c2_step(lengths, t, 256) for t in range(2)]
    pages = [((a - np.uint64(wl.RANGE_BASE)) >> np.uint64(12)).astype(np.uint64)
             for a, _, _ in steps]
    ops = [o for _, _, o in steps]
    want_all = ho.lru(np.concatenate(pages), np.concatenate(ops), frames)
    start = 0
    t0 = 0
    for t, (address, nbytes, op) in enumerate(steps):
        n = address.size
        arrival = (np.uint64(t0) + np.arange(n, dtype=np.uint64)).astype(np.uint64)
        t0 += n
        want = tuple(w[start:start + n] for w in want_all)
        start += n
        dev = [torch.from_numpy(address.view(np.int64)).cuda(),
               torch.from_numpy(nbytes.view(np.int32)).cuda(), torch.from_numpy(op).cuda(),
               torch.from_numpy(arrival.view(np.int64)).cuda()]
        hit, victim, dirty, status, done, latency = ctx.submit_capacity(*dev, timed=True)
        check((hit.cpu().numpy(), victim.cpu().numpy().view(np.uint64), dirty.cpu().numpy(),
               status.cpu().numpy()), want, f"step {t}")
        want_done, want_lat = ho.capacity_timing(
            oracle.geometry, oracle.timing, oracle.chan_bw, oracle.t_read, oracle.t_prog,
            oracle.admit, np.ones(n, np.uint8), want[0], pages[t], want[1], want[2], arrival,
            12, oracle.state)
        got = done.cpu().numpy().view(np.uint64)
        bad = np.flatnonzero(got != want_done)
        assert bad.size == 0, f"step {t}: done differs at {bad[:5]}"
        assert np.array_equal(latency.cpu().numpy().view(np.uint64), want_lat)
        del dev, hit, victim, dirty, status, done, latency
    assert int(want_all[2].sum()) > 0, "the steps evict dirty pages (chained reads)"
    assert np.array_equal(ctx.get_state(), oracle.state)
    ctx.close()


# ---- CLOCK (the reference runtime's second-chance policy) ----
CLOCK_GOLDEN = Path(__file__).resolve().parent / "golden" / "clock_goldens.json"


def clock_context(tmp, frames):
    ctx = capacity_context(tmp, frames)
    ctx.capacity_configure(frames, PAGE, policy="clock")
    return ctx


def test_clock_reference_goldens(tmp_path):
    """GPU CLOCK decisions against the reference HbmCache
    (tests/golden/clock_goldens.json), each case over three batches."""
    rng = np.random.default_rng(1)
    for k, case in enumerate(json.loads(CLOCK_GOLDEN.read_text())):
        ctx = clock_context(str(tmp_path / f"c{k}"), case["frames"])
        pages = np.array(case["pages"], np.uint64)
        ops = np.array(case["ops"], np.uint8)
        n = pages.size
        parts = []
        for lo, hi in ((0, n // 3), (n // 3, 2 * n // 3), (2 * n // 3, n)):
            parts.append(run_gpu(ctx, *to_accesses(pages[lo:hi], ops[lo:hi], rng)))
        got = tuple(np.concatenate([p[j] for p in parts]) for j in range(4))
        want = (np.array(case["hit"], np.uint8), np.array(case["victim"], np.uint64),
                np.array(case["victim_dirty"], np.uint8))
        check(got, want, f"clock case {k} ({case['kind']}, {case['frames']} frames)")
        resident, _ = ctx.capacity_state()
        assert resident.size == min(case["frames"], np.unique(pages).size)
        ctx.close()


@pytest.mark.parametrize("frames,universe,n", [(1, 4, 2000), (31, 90, 20000),
                                               (64, 500, 50000), (3000, 9000, 120000)])
def test_clock_matches_oracle_with_media_timing(tmp_path, frames, universe, n):
    """CLOCK decisions and the timed media actions of the misses against the
    oracle (CLOCK pinned to the reference by the goldens above), over
    batches that carry the frames, bits and hand."""
    import torch
    from helpers import OracleRun
    rng = np.random.default_rng(frames + n)
    pages = trace(rng, n, universe, 0.3) if n <= 50000 else \
        np.where(rng.random(n) < 0.7, rng.integers(0, frames, n),
                 rng.integers(0, universe, n)).astype(np.uint64)
    writes = (rng.random(n) < 0.25).astype(np.uint8)
    address, nbytes, op = to_accesses(pages, writes, rng)
    arrival = np.cumsum(rng.exponential(20.0, n).astype(np.uint64) + 1).astype(np.uint64)
    clock = ho.Clock(frames)
    p = wl.c0_profile()
    p["capacity_bytes"] = 64 << 30
    s = Setup(profile=p, model=3, stacks=1, stripe=4096)
    s.ranges = [(wl.RANGE_BASE, 63 << 30, 2, 3)]
    oracle = OracleRun(s)
    ctx = clock_context(str(tmp_path), frames)
    cuts = [0, n // 5, n // 2, n]
    for k, (lo, hi) in enumerate(zip(cuts[:-1], cuts[1:])):
        hit_w, victim_w, dirty_w = clock.run(pages[lo:hi], writes[lo:hi])
        dev = [torch.from_numpy(address[lo:hi].view(np.int64)).cuda(),
               torch.from_numpy(nbytes[lo:hi].view(np.int32)).cuda(),
               torch.from_numpy(op[lo:hi]).cuda(),
               torch.from_numpy(arrival[lo:hi].view(np.int64)).cuda()]
        hit, victim, dirty, status, done, latency = ctx.submit_capacity(*dev, timed=True)
        check((hit.cpu().numpy(), victim.cpu().numpy().view(np.uint64), dirty.cpu().numpy(),
               status.cpu().numpy()), (hit_w, victim_w, dirty_w), f"batch {k}")
        want_done, want_lat = ho.capacity_timing(
            oracle.geometry, oracle.timing, oracle.chan_bw, oracle.t_read, oracle.t_prog,
            oracle.admit, np.ones(hi - lo, np.uint8), hit_w, pages[lo:hi], victim_w, dirty_w,
            arrival[lo:hi], 12, oracle.state)
        got_done = done.cpu().numpy().view(np.uint64)
        bad = np.flatnonzero(got_done != want_done)
        assert bad.size == 0, f"batch {k}: done differs at {bad[:5]}"
        assert np.array_equal(latency.cpu().numpy().view(np.uint64), want_lat)
    assert np.array_equal(ctx.get_state(), oracle.state)
    stats = ctx.capacity_stats()
    assert stats["service_resident_hits"] + stats["service_misses"] == n
    ctx.close()
