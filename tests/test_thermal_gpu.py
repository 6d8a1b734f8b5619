"""GPU parity of the eq3 thermal step (A6) and the epoch controller (A5).

The CUDA grid step (DCT-diagonalized backward Euler) is checked against the
oracle's sparse direct solve (oracle/thermal_oracle.py, itself pinned to the
reference ThermalModel by tests/golden/thermal_goldens.json) within 1e-9
relative; the controller's integer outputs (refresh permille, throttle level
and permille, admit-after tick) bit for bit against the oracle controller fed
the same die temperatures; and a thermal-coupled run (config-3 shape, reduced)
end to end: timing with the factors of the previous epoch, die activity,
temperatures, factors.
"""
import numpy as np
import pytest

import hbf_oracle as ho
import thermal_oracle as to
from helpers import OracleRun, Setup, activity_of, assert_same, gpu_run, make_context
from hbfsim_b200 import workloads as wl

pytestmark = pytest.mark.gpu

SILICON = {"cv_j_m3_k": 1.66e6, "k_xyz_w_m_k": [148.0, 148.0, 148.0]}
NAND = {"cv_j_m3_k": 1.75e6, "k_xyz_w_m_k": [110.0, 110.0, 35.0]}
REL = 1e-9


def stack_desc(nx, ny, dies):
    """One logic layer under 2 NAND layers per die position."""
    layers = [dict(SILICON, thickness_m=100e-6)] + \
             [dict(NAND, thickness_m=50e-6) for _ in range(2 * dies)]
    return {"nx": nx, "ny": ny, "cell_m": 0.5e-3, "layers": layers,
            "bottom": {"h_w_m2_k": 0.0, "ambient_k": 318.15},
            "top": {"h_w_m2_k": 2.0e4, "ambient_k": 318.15}, "initial_k": 318.15}


def floorplan(stacks, channels_per_stack, dies, nx):
    """Die (g, d): row y = g // stacks, x in the stack's share of the row,
    layers 1 + 2d and 2 + 2d."""
    total = stacks * channels_per_stack
    width = nx // stacks
    fp = {k: np.zeros(total * dies, np.uint32) for k in ("z0", "z_count", "x0", "x1", "y0", "y1")}
    for g in range(total):
        s, row = g % stacks, g // stacks
        for d in range(dies):
            i = g * dies + d
            fp["z0"][i], fp["z_count"][i] = 1 + 2 * d, 2
            fp["x0"][i], fp["x1"][i] = s * width, (s + 1) * width
            fp["y0"][i], fp["y1"][i] = row, row + 1
    return fp


POWER = {"idle_w": 0.02, "read_j_per_byte": 2e-9 / 128, "write_j_per_access": 50e-9}
REFRESH = {"onset_k": 343.15, "step_k": 10.0, "base_permille": 10, "cap_permille": 500}


def close(a, b):
    return np.max(np.abs(a - b) / np.abs(b)) < REL


def make(tmp, stacks, model=3):
    p = wl.c0_profile()
    s = Setup(profile=p, model=model, stacks=stacks, stripe=4096)
    s.ranges = [(wl.RANGE_BASE, p["capacity_bytes"] - (1 << 20), 1, 3)]
    return s


def thresholds_from(trajectory):
    lo, hi = float(np.min(trajectory)), float(np.max(trajectory))
    span = hi - lo
    return {"light_k": lo + 0.25 * span, "severe_k": lo + 0.55 * span,
            "shutdown_k": lo + 0.8 * span, "hysteresis_k": 0.1 * span,
            "light_permille": 1250, "severe_permille": 2000}


@pytest.mark.parametrize("nx,ny", [(16, 16), (18, 18)])
def test_grid_and_controller_match_oracle(tmp_path, nx, ny):
    """The epoch step as one cooperative kernel (sides multiples of 4) and as
    separate launches (18 x 18): grid, die means and factors."""
    import torch
    stacks, dies = 2, 4
    setup = make(tmp_path, stacks)
    channels = stacks * setup.profile["channels"]
    n_dies = channels * dies
    desc = stack_desc(nx, ny, dies)
    fp = floorplan(stacks, setup.profile["channels"], dies, nx)
    owner = to.die_floorplan((len(desc["layers"]), ny, nx), fp["z0"], fp["z_count"],
                             fp["x0"], fp["x1"], fp["y0"], fp["y1"])
    rng = np.random.default_rng(5)
    epochs, dt = 16, 5e-3
    # hot burst on stack 0 for 6 epochs, then nothing: heat, then cool down
    acts = []
    for k in range(epochs):
        rb = rng.integers(0, 1 << 20, n_dies).astype(np.uint64)
        wr = np.zeros(n_dies, np.uint64)
        if k < 6:
            hot = np.array([(i // dies) % stacks == 0 for i in range(n_dies)])
            wr[hot] = rng.integers(100_000, 200_000, int(hot.sum())).astype(np.uint64)
        acts.append((rb, wr))
    # oracle temperatures first, to place the throttle thresholds inside the run
    grid = to.ThermalGrid(desc)
    want_t, want_die = [], []
    for rb, wr in acts:
        p = to.cell_power(owner, n_dies, rb, wr, POWER["idle_w"], POWER["read_j_per_byte"],
                          POWER["write_j_per_access"], dt)
        want_t.append(grid.step(p, dt).copy())
        want_die.append(to.die_mean(owner, n_dies, want_t[-1]))
    hottest = np.array([[max(float(np.max(d[g * dies:(g + 1) * dies]))
                             for g in range(s, channels, stacks)) for s in range(stacks)]
                        for d in want_die])
    throttle = thresholds_from(hottest[:, 0])

    ctx = make_context(setup, str(tmp_path / "ctx"))
    ctx.thermal_configure(desc, fp, POWER, REFRESH, throttle)
    ctrl = to.Controller(stacks, channels, dies, REFRESH, throttle)
    levels_seen = set()
    for k, (rb, wr) in enumerate(acts):
        d_rb = torch.from_numpy(rb.view(np.int64)).cuda()
        d_wr = torch.from_numpy(wr.view(np.int64)).cuda()
        ctx.advance_epoch_global(dt, d_rb, d_wr)
        t = ctx.temperatures(owner.size)
        assert close(t, want_t[k]), f"epoch {k}: grid differs"
        die_t = ctx.die_temperatures(n_dies)
        assert close(die_t, want_die[k]), f"epoch {k}: die means differ"
        next_end = (k + 2) * 5_000_000
        r, th, adm, lv = ctrl.step(die_t, next_end)
        gr, gt, ga, glv = ctx.thermal_factors(channels, stacks)
        assert np.array_equal(gr, r) and np.array_equal(gt, th), f"epoch {k}"
        assert np.array_equal(ga, adm) and np.array_equal(glv, lv), f"epoch {k}"
        cr, ct, ca = ctx.channel_factors(channels, stacks)
        assert np.array_equal(cr, r) and np.array_equal(ct, th) and np.array_equal(ca, adm)
        levels_seen.update(int(x) for x in lv)
    assert levels_seen == {0, 1, 2, 3}, levels_seen
    ctx.close()


def test_thermal_coupled_run(tmp_path):
    """Config-3 shape, reduced: the c0 trace cut into 1 ms epochs; each epoch
    is timed with the factors the previous epoch's temperatures produced."""
    stacks, nx, ny = 1, 16, 16
    setup = make(tmp_path, stacks)
    dies = setup.profile["dies_per_channel"]
    channels = stacks * setup.profile["channels"]
    n_dies = channels * dies
    desc = stack_desc(nx, ny, dies)
    fp = floorplan(stacks, setup.profile["channels"], dies, nx)
    owner = to.die_floorplan((len(desc["layers"]), ny, nx), fp["z0"], fp["z_count"],
                             fp["x0"], fp["x1"], fp["y0"], fp["y1"])
    epochs, dt, epoch_ns = 6, 1e-3, 1_000_000
    arrays = wl.c0_trace(epochs * 480_000, seed=11,
                         range_length=setup.profile["capacity_bytes"] - (1 << 20))
    arrival = arrays[3]
    power = {"idle_w": 0.3, "read_j_per_byte": 2e-9 / 128, "write_j_per_access": 50e-9}
    refresh = {"onset_k": 318.4, "step_k": 0.05, "base_permille": 5, "cap_permille": 400}
    throttle = {"light_k": 318.6, "severe_k": 318.9, "shutdown_k": 319.4,
                "hysteresis_k": 0.05, "light_permille": 1500, "severe_permille": 3000}
    ctx = make_context(setup, str(tmp_path / "ctx"))
    ctx.thermal_configure(desc, fp, power, refresh, throttle)
    oracle = OracleRun(setup)
    grid = to.ThermalGrid(desc)
    ctrl = to.Controller(stacks, channels, dies, refresh, throttle)
    refresh_seen = set()
    for k in range(epochs):
        lo, hi = np.searchsorted(arrival, [k * epoch_ns, (k + 1) * epoch_ns])
        part = tuple(a[lo:hi] for a in arrays)
        got = gpu_run(ctx, part)
        want = oracle.run(*part, threads=8)
        assert_same(got, want, f"epoch {k}")
        rb, wr = activity_of(setup, oracle, part, want[2])
        g_rb, g_wr = ctx.die_activity(n_dies)
        assert np.array_equal(g_rb, rb) and np.array_equal(g_wr, wr), f"epoch {k}: activity"
        ctx.advance_epoch(dt)
        p = to.cell_power(owner, n_dies, rb, wr, power["idle_w"], power["read_j_per_byte"],
                          power["write_j_per_access"], dt)
        t_want = grid.step(p, dt)
        assert close(ctx.temperatures(owner.size), t_want), f"epoch {k}: grid"
        die_t = ctx.die_temperatures(n_dies)
        r, th, adm, _ = ctrl.step(die_t, (k + 2) * epoch_ns)
        gr, gt, ga, _ = ctx.thermal_factors(channels, stacks)
        assert np.array_equal(gr, r) and np.array_equal(gt, th) and np.array_equal(ga, adm)
        oracle.set_factors(r, th, adm)
        refresh_seen.update(int(x) for x in r)
    assert len(refresh_seen) > 1, "the run never changed the refresh factors"
    ctx.close()
