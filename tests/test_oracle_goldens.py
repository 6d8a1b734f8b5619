"""Pin the CPU oracle to the reference before trusting it as the checker.

Every golden here was produced by the reference's own code (see
tests/golden/make_goldens.py): hbf_device.cuh / calibrator.cpp compiled from
source, tools/eq3_layered_export.py + ThermalModel, and the offline LruCache.
"""
import ctypes
import json

import numpy as np
import pytest

import hbf_oracle as ho
from thermal_oracle import ThermalGrid


def _device_records(golden_dir):
    with open(golden_dir / "device_goldens.jsonl") as f:
        return [json.loads(line) for line in f]


def test_range_lookup_and_media_descriptor(golden_dir):
    table = None
    count = 0
    checked = 0
    for rec in _device_records(golden_dir):
        if rec["kind"] == "ranges":
            table = ho.make_ranges(rec["ranges"])
            count = len(rec["ranges"])
            continue
        if rec["kind"] != "probe":
            continue
        a, b, op = rec["a"], rec["bytes"], rec["op"]
        tp = ctypes.cast(table, ctypes.c_void_p)
        index = ho.LIB.or_find_range_index(tp, count, a)
        assert index == rec["index"]
        if index != count:
            rp = ctypes.cast(ctypes.byref(table[index]), ctypes.c_void_p)
            assert ho.LIB.or_access_supported(rp, a, b, op) == rec["supported"]
            logical = ctypes.c_uint64(0)
            mbytes = ctypes.c_uint32(0)
            valid = ho.LIB.or_media_descriptor(rp, a, b, op, ctypes.addressof(logical),
                                               ctypes.addressof(mbytes))
            assert valid == rec["media_valid"]
            if valid:
                assert logical.value == rec["logical"]
                assert mbytes.value == rec["media_bytes"]
        successor = 0 if index == count else index + 1
        if successor < count:
            sp_ = ctypes.cast(ctypes.byref(table[successor]), ctypes.c_void_p)
            assert ho.LIB.or_range_overlaps(sp_, a, b) == rec["succ_overlap"]
        checked += 1
    assert checked > 1000


def test_classification_matches_reference_predicates(golden_dir):
    """The oracle's per-access status follows the resolve order of checks:
    bytes==0 -> unsupported; outside a range -> unsupported if the span
    touches the successor range, else bypass; inside -> media descriptor."""
    table = None
    rows = []
    geometry = ho.make_geometry(1, 1, 1, 1, 4096, 4096)
    for rec in _device_records(golden_dir):
        if rec["kind"] == "ranges":
            table, rows = ho.make_ranges(rec["ranges"]), rec["ranges"]
            continue
        if rec["kind"] != "probe" or rec["op"] > 1:
            continue
        d = ho.decode(table, len(rows), geometry, np.array([rec["a"]], np.uint64),
                      np.array([rec["bytes"]], np.uint32),
                      np.array([rec["op"]], np.uint8))[0]
        count = len(rows)
        inside = rec["index"] != count and rec["a"] - rows[rec["index"]][0] < rows[rec["index"]][1]
        if rec["bytes"] == 0:
            expect = ho.STATUS_UNSUPPORTED
        elif not inside:
            expect = ho.STATUS_UNSUPPORTED if rec["succ_overlap"] == 1 else ho.STATUS_BYPASS
        elif rec["media_valid"] != 1:
            expect = ho.STATUS_UNSUPPORTED
        else:
            mode = rows[rec["index"]][4]
            expect = ho.STATUS_MODELED if mode == 1 else ho.STATUS_UNSUPPORTED
        assert d["status"] == expect, rec
        if expect == ho.STATUS_MODELED:
            assert d["media_address"] == rec["logical"]


def test_transfer_service_and_saturating(golden_dir):
    n = 0
    for rec in _device_records(golden_dir):
        if rec["kind"] == "transfer":
            assert ho.LIB.or_fast_transfer_ns(rec["bytes"], rec["bw"]) == rec["transfer"]
            assert ho.LIB.or_fast_service_ns(10000, rec["bytes"], rec["bw"]) == rec["service"]
            # calibrator.cpp returns 0 for a zero-byte request while the device
            # helper returns the base latency; the reference pins the two only
            # for bytes >= 1 (tests/cpu/calibrator_test.cpp:42-75).
            if rec["bytes"] > 0 and rec["bw"] > 0:
                assert rec["service"] == rec["host_service"]
            n += 1
        elif rec["kind"] == "sat":
            assert ho.LIB.or_saturating_add(rec["a"], rec["b"]) == rec["add"]
            assert ho.LIB.or_saturating_multiply(rec["a"], rec["b"] & 0xFFFFFFFF) == rec["mul"]
            n += 1
        elif rec["kind"] == "hybrid":
            assert ho.LIB.or_hybrid_reference_sample(
                rec["seq"], rec["warmup"], rec["threshold"], rec["key"]) == rec["sample"]
            n += 1
    assert n > 200


def test_fast_model_traces(golden_dir):
    """The oracle's FAST model reproduces the reference tail recurrence
    (hbf_device.cu:883-910) step for step, saturation included."""
    traces = [r for r in _device_records(golden_dir) if r["kind"] == "fast_trace"]
    assert len(traces) == 3
    for tr in traces:
        steps = np.array(tr["steps"], dtype=object)
        n = len(steps)
        page = tr["page"]
        base = 1 << 40
        ranges = ho.make_ranges([(base, 1 << 36, 0, 1, 1, 3, page)])
        g = ho.make_geometry(1, 1, 1, 1, page, page)
        t = ho.Timing(ho.MODEL_FAST, tr["scale"], tr["read_lat"], tr["prog_lat"],
                      tr["bw"], page)
        arrival = np.array([int(s[0]) for s in steps], np.uint64)
        op = np.array([int(s[1]) for s in steps], np.uint8)
        addr = np.full(n, base, np.uint64)
        nbytes = np.full(n, 64, np.uint32)
        state = np.array([tr["tail0"]], np.uint64)
        zeros = np.zeros(1, np.uint64)
        done, lat, status, stats = ho.run_batch(ranges, 1, g, t, zeros, zeros, zeros,
                                                addr, nbytes, op, arrival, state)
        assert (status == ho.STATUS_MODELED).all()
        assert [int(x) for x in done] == [int(s[2]) for s in steps]
        assert stats["fast_modeled_ns"] == sum(int(s[3]) for s in steps) % (1 << 64)


def test_thermal_oracle_against_reference_model(golden_dir):
    cases = json.loads((golden_dir / "thermal_goldens.json").read_text())
    for case in cases:
        grid = ThermalGrid(case["stack"])
        out = np.array(grid.run(case["power_w"], case["dt"]))
        ref = np.array(case["temperature_k"])
        assert np.max(np.abs(out - ref) / ref) < 1e-12


def test_lru_oracle_against_reference_policy(golden_dir):
    for case in json.loads((golden_dir / "lru_goldens.json").read_text()):
        keys = np.array(case["keys"], np.uint64)
        writes = np.zeros(keys.size, np.uint8)
        hit, victim, _ = ho.lru(keys, writes, case["frames"])
        assert hit.tolist() == case["hits"]
        expect = [(1 << 64) - 1 if v < 0 else v for v in case["victims"]]
        assert [int(v) for v in victim] == expect


def test_lru_dirty_tracking():
    # capacity 2: write A, read B, read C evicts A (dirty), read A evicts B (clean)
    keys = np.array([10, 11, 12, 10], np.uint64)
    writes = np.array([1, 0, 0, 0], np.uint8)
    hit, victim, vdirty = ho.lru(keys, writes, 2)
    assert hit.tolist() == [0, 0, 0, 0]
    assert victim.tolist()[2:] == [10, 11]
    assert vdirty.tolist()[2:] == [1, 0]


@pytest.mark.parametrize("threads", [1, 3])
def test_die_model_threads_agree(threads):
    rng = np.random.default_rng(3)
    n = 5000
    ranges = ho.make_ranges([(1 << 30, 1 << 28, 0, 1, 1, 3, 16384)])
    g = ho.make_geometry(2, 4, 4, 2, 4096, 16384)
    t = ho.Timing(ho.MODEL_DIE, 1, 3000, 200000, 0, 16384)
    addr = (1 << 30) + rng.integers(0, (1 << 28) - 4096, n, dtype=np.uint64) // 128 * 128
    nbytes = np.where(rng.random(n) < 0.8, 128, 512).astype(np.uint32)
    op = (rng.random(n) < 0.1).astype(np.uint8)
    arrival = np.cumsum(rng.integers(0, 5, n)).astype(np.uint64)
    bw = np.full(8, 8_000_000_000, np.uint64)
    tr = np.full(2, 3000, np.uint64)
    tp = np.full(2, 200000, np.uint64)
    s1 = np.zeros(8 * 5, np.uint64)
    s2 = np.zeros(8 * 5, np.uint64)
    d1, l1, st1, _ = ho.run_batch(ranges, 1, g, t, bw, tr, tp, addr, nbytes, op, arrival, s1, 1)
    d2, l2, st2, _ = ho.run_batch(ranges, 1, g, t, bw, tr, tp, addr, nbytes, op, arrival, s2, threads)
    assert (d1 == d2).all() and (l1 == l2).all() and (s1 == s2).all()


# ---- empirical burst-curve profile (hbf_device.cuh:959-1140) ----

def test_empirical_curve_lookup(golden_dir):
    curves = [r for r in _device_records(golden_dir) if r["kind"] == "emp_curve"]
    assert len(curves) >= 8
    for rec in curves:
        pages = rec["pages"] + [0] * (6 - len(rec["pages"]))
        cum = rec["cum"] + [0] * (6 - len(rec["cum"]))
        for run, want_c, want_s in zip(rec["runs"], rec["cumulative"], rec["service"]):
            assert ho.empirical_cumulative(pages, cum, rec["count"], run) == want_c, run
            assert ho.empirical_service(pages, cum, rec["count"], run) == want_s, run


def test_empirical_reference_kats():
    """The reference's own known answers (tests/cpu/device_helper_abi_test.cpp)."""
    pages = [1, 4, 16, 64, 256, 512]
    cum = [11133, 41495, 168606, 2824351, 10767793, 20254374]
    assert ho.empirical_cumulative(pages, cum, 6, 0) == 0
    assert ho.empirical_cumulative(pages, cum, 6, 1) == 11133
    assert ho.empirical_cumulative(pages, cum, 6, 3) == 31375
    assert ho.empirical_cumulative(pages, cum, 6, 4) == 41495
    assert ho.empirical_cumulative(pages, cum, 6, 512) == 20254374
    assert ho.empirical_cumulative(pages, cum, 6, 513) == 20291431
    packed, run, ok = ho.update_burst(0, 100, 0)
    assert ok and run == 1
    packed, run, ok = ho.update_burst(packed, 101, 0)
    assert ok and run == 2
    assert ho.update_burst(packed, 103, 0)[1] == 1
    assert ho.update_burst(packed, 101, 0)[1] == 1
    assert ho.update_burst(packed, 102, 1)[1] == 1
    e = ho.make_empirical(pages, cum, 408305)
    total, state = 0, 0
    for page in range(4):
        svc, state, _, ok = ho.empirical_request(e, state, page, 0)
        assert ok
        total += svc
    assert total == 41495
    svc, state, run, ok = ho.empirical_request(e, state, 99, 0)
    assert ok and run == 1 and svc == 11133
    svc, state, run, ok = ho.empirical_request(e, state, 100, 1)
    assert ok and run == 1 and svc == 408305


def test_empirical_burst_state(golden_dir):
    chains = [r for r in _device_records(golden_dir) if r["kind"] == "emp_burst"]
    assert len(chains) == 4
    steps = 0
    for rec in chains:
        for prev, page, op, packed, run, valid in rec["steps"]:
            assert ho.update_burst(prev, page, op) == (packed, run, bool(valid))
            steps += 1
    assert steps >= 3000


def test_empirical_control_header(golden_dir):
    recs = [r for r in _device_records(golden_dir) if r["kind"] == "emp_control"]
    assert len(recs) == 40 and {r["valid"] for r in recs} == {0, 1}
    for rec in recs:
        e = ho.make_empirical(rec["pages"], rec["cum"], rec["program"], rec["flags"],
                              rec["count"])
        assert ho.empirical_control_valid(e) == bool(rec["valid"])
        svc, _, _, ok = ho.empirical_request(e, 0, 5, 0)
        assert (svc if ok else 0) == rec["service"]


def test_empirical_fast_path_traces(golden_dir):
    """The empirical branch of resolve_fast_or_hybrid (hbf_device.cu:797-838)
    as the reference's helpers compute it, against the oracle's batch runner:
    one timing range of 4 KiB pages, every access one page."""
    traces = [r for r in _device_records(golden_dir) if r["kind"] == "emp_trace"]
    assert len(traces) == 4
    base = 1 << 40
    for rec in traces:
        steps = rec["steps"]
        e = ho.make_empirical(rec["pages"], rec["cum"], rec["program"])
        ranges = ho.make_ranges([(base, 1 << 34, 0, 1, 1, 3, 4096)])
        page = np.array([s[1] for s in steps], np.uint64)
        address = (base + page * 4096).astype(np.uint64)
        nbytes = np.full(page.size, 64, np.uint32)
        op = np.array([s[2] for s in steps], np.uint8)
        arrival = np.array([s[0] for s in steps], np.uint64)
        state = np.array([rec["tail0"], 0], np.uint64)
        done, _, status, stats = ho.run_empirical(ranges, 1, e, rec["scale"], 10**9,
                                                  address, nbytes, op, arrival, state)
        assert np.all(status == 1)
        assert done.tolist() == [s[4] for s in steps]
        assert stats["fast_modeled_ns"] == sum(s[5] for s in steps) % (1 << 64)


# ---- per-block retention ledger (experiments/eq3_system_thermal/reliability.py) ----

def replay_retention(case):
    """Replays one golden scenario through the oracle ledger; yields
    (step, ledger, due blocks, due bits) after every epoch."""
    import retention_oracle as ro
    led = ro.Ledger(case["dies"], case["blocks_per_die"], case["ea_ev"], case["initial_age_ns"],
                    case["initial_wall_age_ns"], case["epoch_ns"], case["refresh_trigger"],
                    case["initial_temperature_k"])
    for step in case["steps"]:
        led.advance(step["end_ns"], step["temps"], midpoint=True)
        led.program(step["programs"])
        led.erase(step["erases"])
        blocks, bits = led.due(step["end_ns"])
        led.refresh(step["refresh"])
        yield step, led, blocks, bits


def test_retention_oracle_against_reference_ledger(golden_dir):
    cases = json.loads((golden_dir / "retention_goldens.json").read_text())
    assert len(cases) == 3
    for case in cases:
        n = case["dies"] * case["blocks_per_die"]
        for step, led, blocks, bits in replay_retention(case):
            want = np.zeros(n, np.uint8)
            want[blocks] = bits
            assert want.tolist() == step["due"]
            assert led.age.tolist() == step["age"]          # bit-exact: same float steps
            assert led.next_due.tolist() == step["next_due"]
            assert [-1 if v == (1 << 64) - 1 else int(v) for v in led.last_commit] == \
                step["last_commit"]
            assert led.counts.tolist() == step["counts"]


# ---- prefetch model (src/prefetch/prefetch_model.cpp) ----

PREFETCH_KEYS = ("policy", "accuracy", "lead", "buffer", "in_flight", "read_ns", "compute_ns",
                 "seed")


def test_prefetch_oracle_against_reference_model(golden_dir):
    """The oracle's restatement (Mersenne Twister predictor draws, FIFO
    staging buffer, min-heap media servers) against the reference model
    compiled from its own source, cell for cell."""
    streams = json.loads((golden_dir / "prefetch_goldens.json").read_text())
    assert [s["stream"] for s in streams] == ["sequential", "random", "moe", "loop"]
    cells = 0
    for s in streams:
        pages = np.array(s["pages"], np.uint64)
        for row in s["cells"]:
            got = ho.prefetch_run(pages, dict(zip(PREFETCH_KEYS, row[:8])))
            assert list(got) == row[8:], (s["stream"], row[:8])
            cells += 1
    assert cells == 340


# ---- UCIe streaming link (src/ucie/link.cpp) ----

def test_link_oracle_against_reference_link(golden_dir):
    """The oracle's restatement of the streaming link (event order, flit
    packing, credit reservation and legal grants, retries) under the batch
    driver, against the reference class compiled from its own source."""
    cases = json.loads((golden_dir / "link_goldens.json").read_text())
    assert len(cases) == 30
    for k, c in enumerate(cases):
        delivered, counters, now, ar, r = ho.link_run(c["profile"], np.array(c["direction"]),
                                                      np.array(c["ready"]))
        assert delivered.tolist() == c["delivered"], k
        assert counters.tolist() == c["counters"], k
        assert [ar, r, now] == c["tail"], k


def test_stripe_decode_against_reference_layout(golden_dir):
    """A2 pinned: the oracle's mixed-radix decode reproduces the reference's
    hbf_cold_read_bank (LPA -> channel, die, bank) and its page-striped
    stack/module placement, in the geometries where the two describe the
    same mapping (helpers.bank_layout_cases, helpers.stripe_layout_cases)."""
    from helpers import (OracleRun, bank_layout_cases, check_layout_decode, layout_goldens,
                         stripe_layout_cases)
    golden = layout_goldens(golden_dir)
    cases = 0
    for kind, gen in (("bank", bank_layout_cases), ("stripe", stripe_layout_cases)):
        for case in gen(golden):
            ora = OracleRun(case[0])
            got = ho.decode(ora.ranges, ora.count, ora.geometry, *case[1:4])
            check_layout_decode(got, case, kind)
            cases += case[1].size
    assert cases == len(golden["bank"]) + len(golden["stripe"])


def test_clock_oracle_against_reference_cache(golden_dir):
    """The oracle's CLOCK (or_clock_run) against the reference HbmCache's
    second-chance decisions, each case split over three calls (the state
    carries across calls)."""
    with open(golden_dir / "clock_goldens.json") as f:
        cases = json.load(f)
    for case in cases:
        pages = np.array(case["pages"], np.uint64)
        ops = np.array(case["ops"], np.uint8)
        clock = ho.Clock(case["frames"])
        cuts = [0, len(pages) // 3, 2 * len(pages) // 3, len(pages)]
        got = [clock.run(pages[a:b], ops[a:b]) for a, b in zip(cuts[:-1], cuts[1:])]
        hit = np.concatenate([g[0] for g in got])
        victim = np.concatenate([g[1] for g in got])
        dirty = np.concatenate([g[2] for g in got])
        assert np.array_equal(hit, np.array(case["hit"], np.uint8)), case["kind"]
        assert np.array_equal(victim, np.array(case["victim"], np.uint64)), case["kind"]
        assert np.array_equal(dirty, np.array(case["victim_dirty"], np.uint8)), case["kind"]


def test_linked_stage_oracle_against_reference_link(golden_dir):
    """The die model followed by each stack's UCIe link, composed with the
    oracle's link (or_link_run) the way tests/golden/linked_goldens.json
    composes the reference StreamingLink: every access's R and AR delivery."""
    from helpers import OracleRun, Setup, oracle_linked
    from hbfsim_b200 import workloads as wl
    with open(golden_dir / "linked_goldens.json") as f:
        g = json.load(f)
    p = wl.c0_profile()
    s = Setup(profile=p, model=3, stacks=g["stacks"], stripe=4096)
    s.ranges = [(wl.RANGE_BASE, p["capacity_bytes"] - (1 << 20), 1, 3)]
    arrays = wl.c0_trace(g["n"], seed=g["seed"], range_length=p["capacity_bytes"] - (1 << 20))
    linked, done, status, ar = oracle_linked(s, OracleRun(s), arrays, g["profile"])
    assert done.tolist() == g["die_done"]
    assert status.tolist() == g["status"]
    assert linked.tolist() == g["linked_done"]
    assert ar.tolist() == g["ar_delivered"]
