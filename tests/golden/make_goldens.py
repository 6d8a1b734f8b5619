"""Regenerate the golden fixtures in this directory from the HBFSim reference.

Run where the HBFSim source tree is available; its location comes from the
HBFSIM_REFERENCE environment variable, which must be set:

    make -C oracle REF=$HBFSIM_REFERENCE   # golden generators from reference sources
    HBFSIM_REFERENCE=<tree> python tests/golden/make_goldens.py

Fixtures written:
  device_goldens.jsonl   range lookup / access_supported / media_descriptor,
                         fast_transfer_ns, fast_service_ns (device and host),
                         saturating arithmetic, hybrid sampler bit and
                         fast-model traces, all computed by the reference's own
                         functions (src/cuda_runtime/device/hbf_device.cuh,
                         src/hybrid/calibrator.cpp).
  layout_goldens.json    the reference's stripe decode of the UCIe stack path:
                         hbf_cold_read_bank / hbf_media_lpa
                         (src/ucie/bank_layout.cpp) and the page-striped
                         placement checked by ContiguousStackMap::locate and
                         inverse_page_striped (src/ucie/stack_router.cpp).
  clock_goldens.json     hit / victim / victim-dirty decisions of the reference
                         second-chance CLOCK HBM cache
                         (src/cuda_runtime/hbm_cache.cpp, compiled from
                         source) driven as the capacity service resolves
                         page references.
  linked_goldens.json    the die model composed with each stack's UCIe link:
                         AR at the arrival and R at the die completion of
                         every access of a seeded trace, through the
                         reference StreamingLink (src/ucie/link.cpp).
  link_goldens.json      delivery ticks, counters and credits of the reference
                         UCIe streaming link (src/ucie/link.cpp, compiled
                         from source) on message batches.
  prefetch_goldens.json  statistics of the reference prefetch model
                         (src/prefetch/prefetch_model.cpp, compiled from
                         source) for sweep cells on four page streams.
  retention_goldens.json per-block retention ages, due reasons, refreshes and
                         program / erase counts from the reference
                         ReliabilityLedger (experiments/eq3_system_thermal/
                         reliability.py).
  thermal_goldens.json   layered RC grids built by the reference exporter
                         (tools/eq3_layered_export.py discretize()/network())
                         and advanced by the reference ThermalModel
                         (src/eq3_thermal/thermal.cpp, backward Euler with
                         dense Cholesky).

Nothing at test time reads the reference tree: the tests read only these
fixtures.
"""
from __future__ import annotations

import importlib.util
import json
import os
import random
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
if not os.environ.get("HBFSIM_REFERENCE"):
    sys.exit("make_goldens.py: set HBFSIM_REFERENCE to the HBFSim source tree")
REF = Path(os.environ["HBFSIM_REFERENCE"])
REF_BIN = REPO / "oracle" / "_ref" / "ref_goldens"
REF_PREFETCH = REPO / "oracle" / "_ref" / "ref_prefetch"
REF_LINK = REPO / "oracle" / "_ref" / "ref_link"
REF_LAYOUT = REPO / "oracle" / "_ref" / "ref_layout"
REF_CLOCK = REPO / "oracle" / "_ref" / "ref_clock"


def load_exporter():
    path = REF / "tools" / "eq3_layered_export.py"
    spec = importlib.util.spec_from_file_location("eq3_layered_export", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def device_goldens() -> None:
    out = subprocess.run([str(REF_BIN), "device"], check=True,
                         capture_output=True, text=True).stdout
    (HERE / "device_goldens.jsonl").write_text(out)


def layered_ir(stack: dict) -> dict:
    """The layer-stack description used by this build, written as the
    exporter's package IR: one full-footprint component per layer."""
    nx, ny, cell = stack["nx"], stack["ny"], stack["cell_m"]
    z = 0.0
    components, materials = [], {}
    for index, layer in enumerate(stack["layers"]):
        name = f"mat{index}"
        materials[name] = {"cv_j_m3_k": layer["cv_j_m3_k"],
                           "k_xyz_w_m_k": layer["k_xyz_w_m_k"]}
        components.append({"id": f"layer{index:02d}", "material": name,
                           "xyz_m": [0.0, 0.0, z],
                           "size_m": [nx * cell, ny * cell, layer["thickness_m"]],
                           "powered": True, "physical_type": "HBF"})
        z += layer["thickness_m"]
    return {"package_size_m": [nx * cell, ny * cell, z],
            "components": components, "materials": materials,
            "boundaries": {"bottom": stack["bottom"], "top": stack["top"],
                           "initial_temperature_k": stack["initial_k"]}}


def thermal_case(exporter, stack: dict, steps: int, dt: float, seed: int) -> dict:
    ir = layered_ir(stack)
    grid = exporter.discretize(ir, stack["cell_m"])
    edges, boundaries = exporter.network(ir, grid)
    cells = grid["cells"]
    rng = random.Random(seed)
    n = len(cells)
    powers = []
    for _ in range(steps):
        row = [0.0] * n
        for i in range(n):
            if rng.random() < 0.4:
                row[i] = rng.uniform(0.0, 0.05)
        powers.append(row)
    lines = [f"nodes {n}"]
    for c, (g, t) in zip(cells, boundaries):
        lines.append(f"{c['capacity_j_k']!r} {g!r} {t!r} {stack['initial_k']!r} 0")
    lines.append(f"edges {len(edges)}")
    lines += [f"{i} {j} {g!r}" for i, j, g in edges]
    lines.append(f"steps {steps} {dt!r}")
    lines += [" ".join(repr(p) for p in row) for row in powers]
    with tempfile.NamedTemporaryFile("w", suffix=".net", delete=False) as f:
        f.write("\n".join(lines) + "\n")
        path = f.name
    try:
        out = subprocess.run([str(REF_BIN), "thermal", path], check=True,
                             capture_output=True, text=True).stdout
    finally:
        os.unlink(path)
    temps = [[float(v) for v in line.split()[2:]] for line in out.splitlines()]
    return {"stack": stack, "dt": dt, "steps": steps, "power_w": powers,
            "temperature_k": temps, "shape": grid["shape"],
            "edge_count": len(edges)}


def thermal_goldens() -> None:
    exporter = load_exporter()
    silicon = {"cv_j_m3_k": 1.66e6, "k_xyz_w_m_k": [148.0, 148.0, 148.0]}
    nand = {"cv_j_m3_k": 1.75e6, "k_xyz_w_m_k": [110.0, 110.0, 35.0]}
    cases = []
    stack_a = {"nx": 6, "ny": 5, "cell_m": 1.0e-3, "initial_k": 318.15,
               "layers": [dict(silicon, thickness_m=100e-6),
                          dict(nand, thickness_m=50e-6),
                          dict(nand, thickness_m=50e-6)],
               "bottom": {"h_w_m2_k": 0.0, "ambient_k": 318.15},
               "top": {"h_w_m2_k": 2.0e4, "ambient_k": 318.15}}
    cases.append(thermal_case(exporter, stack_a, steps=6, dt=1e-3, seed=1))
    stack_b = {"nx": 8, "ny": 8, "cell_m": 0.5e-3, "initial_k": 330.0,
               "layers": [dict(silicon, thickness_m=80e-6)] +
                         [dict(nand, thickness_m=40e-6) for _ in range(4)],
               "bottom": {"h_w_m2_k": 500.0, "ambient_k": 310.0},
               "top": {"h_w_m2_k": 1.5e4, "ambient_k": 318.15}}
    cases.append(thermal_case(exporter, stack_b, steps=5, dt=2e-3, seed=2))
    (HERE / "thermal_goldens.json").write_text(json.dumps(cases))


def lru_goldens() -> None:
    """Exact-LRU victims from the reference's offline policy
    (adapters/vllm_capacity/placement_policy.py LruCache)."""
    sys.path.insert(0, str(REF / "adapters" / "vllm_capacity"))
    from placement_policy import LruCache  # noqa: E402  (reference code)
    rng = random.Random(7)
    cases = []
    for frames, universe, length in ((0, 5, 40), (1, 4, 60), (2, 3, 50),
                                     (16, 40, 3000), (100, 150, 6000),
                                     (64, 1000, 4000)):
        keys = []
        for _ in range(length):
            if rng.random() < 0.5 and keys:
                keys.append(keys[-1 - rng.randrange(min(len(keys), 32))])
            else:
                keys.append(rng.randrange(universe))
        cache = LruCache(frames)
        hits, victims = [], []
        for position, key in enumerate(keys):
            result = cache.access((0, key), position)
            hits.append(1 if result.hit else 0)
            victims.append(-1 if result.evicted is None else result.evicted[1])
        cases.append({"frames": frames, "keys": keys, "hits": hits,
                      "victims": victims})
    (HERE / "lru_goldens.json").write_text(json.dumps(cases))


def retention_goldens() -> None:
    """Per-block ages, due reasons, committed refreshes and program / erase
    counts from the reference ReliabilityLedger
    (experiments/eq3_system_thermal/reliability.py), driven as
    run_maintenance_point.py:189, 225-234 drives it: one cohort per die per
    epoch at the midpoint of the die's previous and current temperature."""
    sys.path.insert(0, str(REF / "experiments" / "eq3_system_thermal"))
    from reliability import DAY_NS, ReliabilityLedger  # noqa: E402  (reference code)
    hour = 3_600_000_000_000
    rng = random.Random(11)
    cases = []
    for ea, trigger, age0, wall0, epoch0 in ((1.04, "wall_only", DAY_NS * 9, 0, 0),
                                             (1.08, "equivalent_age_or_wall",
                                              DAY_NS - hour, 0, 5_000),
                                             (1.01, "equivalent_age_or_wall", 0,
                                              DAY_NS // 2, 0)):
        dies, per_die, t_init = 3, 4, 330.0
        names = [f"d{d}/b{b}" for d in range(dies) for b in range(per_die)]
        ledger = ReliabilityLedger({"ea_ev": ea, "refresh_trigger": trigger,
                                    "initial_equivalent_age_ns": age0,
                                    "initial_wall_age_ns": wall0,
                                    "maintenance_epoch_ns": epoch0})
        prev = [t_init] * dies
        now = epoch0
        steps = []
        for epoch in range(14):
            length = rng.choice([1_000_000, hour, 7 * hour, 123_456_789])
            temps = [rng.uniform(300.0, 410.0) for _ in range(dies)]
            for d in range(dies):
                midpoint = (prev[d] + temps[d]) / 2
                ledger.advance_temperature_many(names[d * per_die:(d + 1) * per_die], now,
                                                now + length, midpoint)
                prev[d] = temps[d]
            now += length
            programs = [rng.randrange(len(names)) for _ in range(rng.randrange(4))]
            for b in programs:
                ledger.record_program(names[b], now, True, f"p{epoch}.{b}")
            erases = [rng.randrange(len(names)) for _ in range(rng.randrange(3))]
            for b in erases:
                ledger.record_erase(names[b], now, True, f"e{epoch}.{b}")
            due = []
            for n in names:
                reasons = ledger.due_reasons(n, now)
                due.append((1 if "WALL_24H_SCENARIO_CADENCE" in reasons else 0) |
                           (2 if "EQUIVALENT_AGE_24H_CONSERVATIVE_POLICY" in reasons else 0))
            refresh = [i for i in range(len(names)) if due[i] and rng.random() < 0.6]
            for i in refresh:
                ledger.record_refresh_terminal(names[i], now, True, f"m{epoch}.{i}")
            blocks = ledger.snapshot()["blocks"]
            rows = [blocks[n] for n in names]
            steps.append({
                "end_ns": now, "temps": temps, "programs": programs, "erases": erases,
                "due": due, "refresh": refresh,
                "age": [r["equivalent_age_ns"] for r in rows],
                "next_due": [r["next_wall_due_ns"] for r in rows],
                "last_commit": [-1 if r["last_refresh_commit_ns"] is None
                                else r["last_refresh_commit_ns"] for r in rows],
                "counts": [[r["program_phase_started_count"] for r in rows],
                           [r["program_completed_count"] for r in rows],
                           [r["erase_phase_started_count"] for r in rows],
                           [r["erase_completed_count"] for r in rows]]})
        cases.append({"ea_ev": ea, "refresh_trigger": trigger, "initial_age_ns": age0,
                      "initial_wall_age_ns": wall0, "epoch_ns": epoch0, "dies": dies,
                      "blocks_per_die": per_die, "initial_temperature_k": t_init,
                      "steps": steps})
    (HERE / "retention_goldens.json").write_text(json.dumps(cases))


def prefetch_streams() -> dict:
    """Page streams for the prefetch goldens: sequential, uniform random,
    MoE-like (per token and layer, 4 of 16 experts, 2 pages each, shuffled)
    and a small looping working set with noise."""
    rng = random.Random(21)
    streams = {"sequential": list(range(3000)),
               "random": [rng.randrange(24000) for _ in range(3000)]}
    moe = []
    for _token in range(60):
        for layer in range(6):
            experts = list(range(16))
            rng.shuffle(experts)
            for e in experts[:4]:
                base = (layer * 16 + e) * 2
                moe += [base, base + 1]
    streams["moe"] = moe
    streams["loop"] = [(k % 50) if rng.random() < 0.85 else rng.randrange(10_000)
                       for k in range(3000)]
    return streams


def prefetch_goldens() -> None:
    """Statistics of the reference prefetch model
    (src/prefetch/prefetch_model.cpp, compiled from source into
    oracle/_ref/ref_prefetch) for cells across every policy and parameter,
    on the streams above."""
    rng = random.Random(5)
    out = []
    for name, pages in prefetch_streams().items():
        cells = [(0, 1.0, 1, 64, 32, 10_000, 0, 1), (1, 1.0, 1, 64, 32, 10_000, 4_000, 1),
                 (1, 1.0, 0, 64, 32, 10_000, 4_000, 1), (2, 0.5, 0, 64, 32, 5_000, 100, 3)]
        if name == "sequential":  # the reference sweep's grid
            for read in (1_000, 2_000, 4_000, 5_000, 10_000, 20_000):
                cells.append((0, 0.0, 8, 64, 32, read, 4_000, 7))
                cells.append((1, 0.0, 8, 64, 32, read, 4_000, 7))
                for acc in (0.0, 0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9, 0.95, 1.0):
                    cells.append((2, acc, 8, 64, 32, read, 4_000, 7))
        for _ in range(60):
            cells.append((rng.choice((0, 1, 2, 2, 2)), rng.choice((0.0, 0.3, 0.7, 0.95, 1.0)),
                          rng.choice((1, 2, 8, 40, 500)), rng.choice((1, 3, 8, 64, 200)),
                          rng.choice((1, 4, 32, 300)), rng.choice((700, 10_000, 20_000)),
                          rng.choice((0, 50, 4_000)), rng.randrange(1 << 40)))
        with tempfile.TemporaryDirectory() as tmp:
            stream_path = Path(tmp) / "stream.bin"
            stream_path.write_bytes(b"".join(int(p).to_bytes(8, "little") for p in pages))
            cell_path = Path(tmp) / "cells.txt"
            cell_path.write_text("".join(f"{c[0]} {c[1]!r} {c[2]} {c[3]} {c[4]} {c[5]} {c[6]} "
                                         f"{c[7]}\n" for c in cells))
            res = subprocess.run([str(REF_PREFETCH), str(stream_path), str(cell_path)],
                                 check=True, capture_output=True, text=True).stdout
        rows = [list(c) + [int(v) for v in line.split()]
                for c, line in zip(cells, res.splitlines())]
        assert len(rows) == len(cells)
        out.append({"stream": name, "pages": pages, "cells": rows})
    (HERE / "prefetch_goldens.json").write_text(json.dumps(out))


def link_goldens() -> None:
    """Delivery ticks, byte and flit counters, credits and final tick of the
    reference UCIe streaming link (src/ucie/link.cpp, compiled from source
    into oracle/_ref/ref_link) under the batch driver, for profiles from the
    reference's own link test (128 credits each, the minimum 3 / 14, a slow
    consumer) and random ones, on message batches of mixed directions."""
    rng = random.Random(31)
    profiles = [dict(gt=16, ar=128, r=128, accepted=128, prop=0, consume=[0, 0]),
                dict(gt=16, ar=3, r=14, accepted=4, prop=0, consume=[0, 0]),
                dict(gt=16, ar=12, r=56, accepted=2, prop=0, consume=[0, 98]),
                dict(gt=8, ar=12, r=56, accepted=4, prop=5, consume=[3, 40]),
                dict(gt=32, ar=40, r=200, accepted=16, prop=1, consume=[0, 0])]
    for _ in range(25):
        profiles.append(dict(gt=rng.choice([8, 16, 32]), ar=rng.choice([3, 4, 12, 40, 128]),
                             r=rng.choice([14, 20, 56, 200]),
                             accepted=rng.choice([1, 2, 4, 16, 128]),
                             prop=rng.choice([0, 1, 7, 100]),
                             consume=[rng.choice([0, 0, 3, 50]), rng.choice([0, 2, 100, 1000])]))
    cases = []
    for k, prof in enumerate(profiles):
        m = 17 if k == 0 else rng.randrange(1, 300)
        share = rng.random()
        direction = [0 if k == 0 else (1 if rng.random() < share else 0) for _ in range(m)]
        ready, t = [], 0
        for _ in range(m):
            t += 0 if (k == 0 or rng.random() < 0.5) else rng.randrange(40)
            ready.append(t)
        text = (f"{prof['gt']} {prof['ar']} {prof['r']} {prof['accepted']} {prof['prop']} "
                f"{prof['consume'][0]} {prof['consume'][1]} {m}\n" +
                "".join(f"{d} {r}\n" for d, r in zip(direction, ready)))
        out = subprocess.run([str(REF_LINK)], input=text, check=True, capture_output=True,
                             text=True).stdout.split("\n")
        cases.append({"profile": prof, "direction": direction, "ready": ready,
                      "delivered": [int(v) for v in out[:m]],
                      "counters": [[int(v) for v in out[m].split()],
                                   [int(v) for v in out[m + 1].split()]],
                      "tail": [int(v) for v in out[m + 2].split()]})
    (HERE / "link_goldens.json").write_text(json.dumps(cases))


def layout_goldens() -> None:
    """Stripe-decode goldens from the reference's UCIe layout functions
    (oracle/ref_layout.cpp over src/ucie/bank_layout.cpp and
    src/ucie/stack_router.cpp): per-LPA host channel / core die / bank, and
    per logical offset of a page-striped parent its stack, module and
    module-local address."""
    out = subprocess.run([str(REF_LAYOUT)], check=True, capture_output=True,
                         text=True).stdout.split("\n")
    bank, stripe = [], []
    for line in out:
        f = line.split()
        if not f:
            continue
        (bank if f[0] == "bank" else stripe).append([int(v) for v in f[1:]])
    (HERE / "layout_goldens.json").write_text(json.dumps({
        "bank_fields": ["host_channels", "ncdu", "banks_per_die", "lpa", "host_channel",
                        "core_die", "bank"],
        "bank": bank,
        "stripe_fields": ["phase", "logical_offset", "stack", "module", "module_local"],
        "stripe": stripe}))


def clock_goldens() -> None:
    """Second-chance CLOCK decisions of the reference HBM cache
    (oracle/ref_clock.cpp over src/cuda_runtime/hbm_cache.cpp) on random and
    cyclic page traces: hit, victim page and victim dirty bit per access."""
    rng = random.Random(77)
    cases = []
    shapes = [(1, 3, 60, 0.5, "random"), (2, 5, 200, 0.3, "random"),
              (7, 30, 2000, 0.3, "random"), (64, 300, 4000, 0.2, "random"),
              (100, 140, 2000, 0.1, "cyclic"), (33, 1000, 3000, 0.05, "zipf"),
              (500, 800, 6000, 0.25, "random")]
    for frames, npages, n, wfrac, kind in shapes:
        if kind == "cyclic":
            pages = [k % npages for k in range(n)]
        elif kind == "zipf":
            weights = [1.0 / (k + 1) ** 1.1 for k in range(npages)]
            pages = rng.choices(range(npages), weights=weights, k=n)
        else:
            pages = [rng.randrange(npages) for _ in range(n)]
        ops = [1 if rng.random() < wfrac else 0 for _ in range(n)]
        text = f"{frames} {n}\n" + "".join(f"{p} {o}\n" for p, o in zip(pages, ops))
        out = subprocess.run([str(REF_CLOCK)], input=text, check=True, capture_output=True,
                             text=True).stdout.split()
        vals = [int(v) for v in out]
        cases.append({"frames": frames, "kind": kind, "pages": pages, "ops": ops,
                      "hit": vals[0::3], "victim": vals[1::3], "victim_dirty": vals[2::3]})
    (HERE / "clock_goldens.json").write_text(json.dumps(cases))


LINKED = {"n": 4000, "seed": 31, "stacks": 2,
          "profile": {"gt": 16, "ar": 12, "r": 56, "accepted": 4, "prop": 7,
                      "consume": [2, 3]}}


def linked_messages(stack, arrival, done, modeled):
    """Per stack, AR at the arrival and R at the die completion of every
    modeled access, in ready order (AR first at equal ticks, then batch
    order): [(direction, ready, access, kind)] per stack."""
    out = {}
    for i in range(len(stack)):
        if not modeled[i]:
            continue
        out.setdefault(int(stack[i]), []).append((int(arrival[i]), 0, i))
    for i in range(len(stack)):
        if modeled[i]:
            out[int(stack[i])].append((int(done[i]), 1, i))
    return {k: sorted(v, key=lambda m: (m[0], m[1], m[2])) for k, v in out.items()}


def linked_goldens() -> None:
    """The die model followed by each stack's UCIe link: the oracle's die
    completions of a seeded config-0-shaped trace on 2 stacks, then the
    reference StreamingLink (oracle/_ref/ref_link, src/ucie/link.cpp
    compiled from source) carrying per access an AR at its arrival and an R
    at its die completion; the fixture holds every access's R and AR
    delivery ticks."""
    import numpy as np
    sys.path.insert(0, str(REPO / "oracle"))
    sys.path.insert(0, str(REPO))
    import hbf_oracle as ho
    from hbfsim_b200 import workloads as wl
    cfg = LINKED
    prof = wl.c0_profile()
    length = prof["capacity_bytes"] - (1 << 20)
    a, b, o, t = wl.c0_trace(cfg["n"], seed=cfg["seed"], range_length=length)
    ranges = ho.make_ranges([(wl.RANGE_BASE, length, 0, 1, 1, 3, prof["page_bytes"])])
    geom = ho.make_geometry(cfg["stacks"], prof["channels"], prof["dies_per_channel"],
                            prof["planes_per_die"], 4096, prof["page_bytes"])
    timing = ho.Timing(3, 1, prof["read_latency_ns"], prof["program_latency_ns"],
                       prof["aggregate_bandwidth_bytes_per_s"], prof["page_bytes"])
    chans = cfg["stacks"] * prof["channels"]
    bw = prof["channel_width_bits"] * prof["channel_transfer_rate_mtps"] * 1_000_000 // 8
    state = np.zeros(chans * (prof["dies_per_channel"] + 1), np.uint64)
    done, _, status, _ = ho.run_batch(ranges, 1, geom, timing, np.full(chans, bw, np.uint64),
                                      np.full(cfg["stacks"], prof["read_latency_ns"], np.uint64),
                                      np.full(cfg["stacks"], prof["program_latency_ns"],
                                              np.uint64), a, b, o, t, state)
    dec = ho.decode(ranges, 1, geom, a, b, o)
    msgs = linked_messages(dec["stack"], t, done, status == 1)
    p = cfg["profile"]
    linked = [int(x) for x in done]
    ar = [-1] * cfg["n"]
    for stack, m in sorted(msgs.items()):
        text = (f"{p['gt']} {p['ar']} {p['r']} {p['accepted']} {p['prop']} "
                f"{p['consume'][0]} {p['consume'][1]} {len(m)}\n" +
                "".join(f"{d} {r}\n" for r, d, _ in m))
        out = subprocess.run([str(REF_LINK)], input=text, check=True, capture_output=True,
                             text=True).stdout.split("\n")
        for (ready, d, i), tick in zip(m, out[:len(m)]):
            if d == 1:
                linked[i] = int(tick)
            else:
                ar[i] = int(tick)
    (HERE / "linked_goldens.json").write_text(json.dumps(
        dict(cfg, die_done=[int(x) for x in done], status=[int(x) for x in status],
             linked_done=linked, ar_delivered=ar)))


GENERATORS = {"device": device_goldens, "thermal": thermal_goldens, "lru": lru_goldens,
              "retention": retention_goldens, "prefetch": prefetch_goldens,
              "link": link_goldens, "layout": layout_goldens, "clock": clock_goldens,
              "linked": linked_goldens}


def main() -> int:
    """All fixtures, or the ones named on the command line."""
    if not REF_BIN.exists():
        print("build oracle/_ref/ref_goldens first (make -C oracle REF=...)", file=sys.stderr)
        return 2
    for name in sys.argv[1:] or list(GENERATORS):
        GENERATORS[name]()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
