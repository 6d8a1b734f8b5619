"""GPU parity of the per-block retention-age ledger (reference:
experiments/eq3_system_thermal/reliability.py ReliabilityLedger, driven as
run_maintenance_point.py:189, 225-234 drives it).

Ages are fp64 sums of (end - start) * exp(Ea/kB (1/Tref - 1/T)); CUDA's exp
and the host's may differ in the last bit, so ages are compared within 1e-12
relative.  Due reasons, refresh bookkeeping and program / erase counts are
compared exactly.  The oracle (oracle/retention_oracle.py) is pinned to the
reference class by tests/golden/retention_goldens.json.
"""
import json
from pathlib import Path

import numpy as np
import pytest

import hbf_oracle as ho
import retention_oracle as ro
from helpers import OracleRun, Setup, make_context, to_device
from hbfsim_b200 import workloads as wl

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "retention_goldens.json"
REL = 1e-12


def setup_c0():
    p = wl.c0_profile()
    s = Setup(profile=p, model=3, stacks=1, stripe=4096)
    s.ranges = [(wl.RANGE_BASE, p["capacity_bytes"] - (1 << 20), 1, 3)]
    return s


def close(got, want):
    scale = np.maximum(np.abs(want), 1.0)
    return np.max(np.abs(got - want) / scale) <= REL


def device_u32(values):
    import torch
    return torch.tensor(np.asarray(values, np.int64), dtype=torch.int32, device="cuda")


def compare(ctx, led, what):
    st = ctx.retention_state()
    assert close(st["age_ns"], led.age), what
    assert np.array_equal(st["next_wall_due_ns"], led.next_due), what
    assert np.array_equal(st["last_refresh_commit_ns"], led.last_commit), what
    got = np.stack([st["program_started"], st["program_completed"], st["erase_started"],
                    st["erase_completed"]])
    assert np.array_equal(got, led.counts), what
    assert st["frontier_ns"] == led.frontier


def test_reference_scenarios(tmp_path):
    """The golden scenarios of the reference ledger (3 dies x 4 blocks each,
    midpoint temperatures, refreshes, programs, erases) on the device ledger
    of a config-0 context: golden die d is local die d, golden block k of it
    is the die's block k.  Every other block follows the oracle."""
    import torch
    cases = json.loads(GOLDEN.read_text())
    for k, case in enumerate(cases):
        setup = setup_c0()
        ctx = make_context(setup, str(tmp_path / f"c{k}"))
        n = ctx.retention_configure(case["ea_ev"], case["initial_temperature_k"],
                                    case["initial_age_ns"], case["initial_wall_age_ns"],
                                    case["epoch_ns"], case["refresh_trigger"])
        dies = setup.local_channels * setup.profile["dies_per_channel"]
        per_die = n // dies
        assert n == 16384 and per_die == 256
        led = ro.Ledger(dies, per_die, case["ea_ev"], case["initial_age_ns"],
                        case["initial_wall_age_ns"], case["epoch_ns"], case["refresh_trigger"],
                        case["initial_temperature_k"])
        gd, gb = case["dies"], case["blocks_per_die"]
        mapped = np.array([d * per_die + b for d in range(gd) for b in range(gb)])
        prev = [case["initial_temperature_k"]] * dies
        for e, step in enumerate(case["steps"]):
            cur = list(step["temps"]) + [330.0 + 0.25 * d for d in range(gd, dies)]
            mid = [(prev[d] + cur[d]) / 2 for d in range(dies)]  # the driver's midpoint
            prev = cur
            ctx.retention_advance(step["end_ns"], torch.tensor(mid, dtype=torch.float64,
                                                                device="cuda"))
            led.advance(step["end_ns"], mid, midpoint=False)
            if step["erases"]:
                ctx.retention_record_erase(device_u32(mapped[step["erases"]]))
                led.erase(mapped[step["erases"]])
            blocks, bits = ctx.retention_due(step["end_ns"])
            want_blocks, want_bits = led.due(step["end_ns"])
            assert np.array_equal(blocks, want_blocks) and np.array_equal(bits, want_bits), e
            golden_bits = np.zeros(gd * gb, np.uint8)
            sel = np.isin(blocks, mapped)
            golden_bits[np.searchsorted(mapped, blocks[sel])] = bits[sel]
            assert golden_bits.tolist() == step["due"], f"case {k} epoch {e}"
            if step["refresh"]:
                ctx.retention_refresh(device_u32(mapped[step["refresh"]]))
                led.refresh(mapped[step["refresh"]])
            st = ctx.retention_state()
            assert close(st["age_ns"][mapped], np.array(step["age"])), f"case {k} epoch {e}"
            assert st["next_wall_due_ns"][mapped].tolist() == step["next_due"]
            # programs come from access batches on the device (tested below):
            # only the erase counts are compared with the golden here
            assert st["erase_started"][mapped].tolist() == step["counts"][2]
            assert st["erase_completed"][mapped].tolist() == step["counts"][3]
            compare(ctx, led, f"case {k} epoch {e}")
        ctx.close()


def test_thermal_driven_epochs(tmp_path):
    """Epochs of the thermal grid: the ledger ages every block at the
    midpoint of its die's previous and current mean temperature."""
    from test_thermal_gpu import POWER, REFRESH, floorplan, stack_desc
    import torch
    setup = setup_c0()
    dies_per_channel = setup.profile["dies_per_channel"]
    channels = setup.profile["channels"]
    n_dies = channels * dies_per_channel
    ctx = make_context(setup, str(tmp_path))
    desc = stack_desc(16, 16, dies_per_channel)
    throttle = {"light_k": 500.0, "severe_k": 510.0, "shutdown_k": 520.0, "hysteresis_k": 1.0,
                "light_permille": 1250, "severe_permille": 2000}
    ctx.thermal_configure(desc, floorplan(1, channels, dies_per_channel, 16), POWER, REFRESH,
                          throttle)
    n = ctx.retention_configure(1.08, desc["initial_k"], refresh_trigger="equivalent_age_or_wall")
    led = ro.Ledger(n_dies, n // n_dies, 1.08, refresh_trigger="equivalent_age_or_wall",
                    initial_temperature_k=desc["initial_k"])
    rng = np.random.default_rng(1)
    epoch_ns = 3_600_000_000_000  # one hour of retention per 5 ms thermal epoch
    for k in range(8):
        rb = torch.from_numpy(rng.integers(0, 1 << 24, n_dies).astype(np.int64)).cuda()
        wr = torch.from_numpy(rng.integers(0, 400_000, n_dies).astype(np.int64)).cuda()
        ctx.advance_epoch_global(5e-3, rb, wr)
        ctx.retention_advance((k + 1) * epoch_ns)
        led.advance((k + 1) * epoch_ns, ctx.die_temperatures(n_dies), midpoint=True)
        blocks, bits = ctx.retention_due((k + 1) * epoch_ns)
        want = led.due((k + 1) * epoch_ns)
        assert np.array_equal(blocks, want[0]) and np.array_equal(bits, want[1]), k
        if k == 5 and blocks.size:
            ctx.retention_refresh(device_u32(blocks[::2]))
            led.refresh(blocks[::2])
        compare(ctx, led, f"epoch {k}")
    assert led.age.max() > 0
    ctx.close()


def test_program_counts_from_batches(tmp_path):
    """Every modeled write of a batch programs its page's block."""
    setup = setup_c0()
    ctx = make_context(setup, str(tmp_path))
    n = ctx.retention_configure()
    p = setup.profile
    arrays = wl.c0_trace(300_000, seed=5, range_length=p["capacity_bytes"] - (1 << 20))
    oracle = OracleRun(setup)
    dec = ho.decode(oracle.ranges, oracle.count, oracle.geometry, *arrays[:3])
    want = np.zeros(n, np.int64)
    for lo, hi in ((0, 100_000), (100_000, 300_000)):
        dev = to_device(tuple(a[lo:hi] for a in arrays))
        ctx.retention_record_programs(*dev[:3])
        b = ro.block_ids(dec[lo:hi], dec["status"][lo:hi], arrays[2][lo:hi],
                         p["dies_per_channel"], p["planes_per_die"], 64, p["pages_per_block"])
        want += np.bincount(b, minlength=n)
    st = ctx.retention_state()
    assert want.sum() > 10_000
    assert np.array_equal(st["program_started"], want)
    assert np.array_equal(st["program_completed"], want)
    ctx.close()


def test_due_capacity_and_rejected_temperature(tmp_path):
    """More due blocks than room: the count is still exact and the first
    `capacity` are written.  A temperature that is not positive is rejected
    on the device and reported once by the next read."""
    import ctypes
    import torch
    from hbfsim_b200 import _lib
    setup = setup_c0()
    ctx = make_context(setup, str(tmp_path))
    n = ctx.retention_configure(1.04, 330.0, initial_age_ns=0, initial_wall_age_ns=ro.DAY_NS)
    lib = _lib.load()
    blocks = torch.empty(100, dtype=torch.int32, device="cuda")
    reasons = torch.empty(100, dtype=torch.uint8, device="cuda")
    count = ctypes.c_uint64()
    assert lib.hbfsim_retention_due_v1(ctx.handle, 0, blocks.data_ptr(), reasons.data_ptr(), 100,
                                       ctypes.byref(count), None) == 0
    assert count.value == n
    assert blocks.cpu().tolist() == list(range(100))
    dies = setup.local_channels * setup.profile["dies_per_channel"]
    temps = torch.full((dies,), 330.0, dtype=torch.float64, device="cuda")
    temps[3] = -1.0
    ctx.retention_advance(1000, temps)
    with pytest.raises(Exception):
        ctx.retention_state()
    st = ctx.retention_state()  # reported once
    assert st["frontier_ns"] == 1000
    ctx.close()
