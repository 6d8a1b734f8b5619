"""Parity at the configs' full sizes (the headline trace included).

The other GPU tests check the CUDA path against the oracle on reduced shapes;
these run whole configurations and compare every access bit for bit:

  c1  the full MoE decode trace (279,204,864 accesses on 4 stacks x 16
      channels x 4 dies) in one batch, as the bench times it: done, latency
      and status of every access, and the carried state at the end.  The
      oracle walks the same trace in consecutive pieces on all host threads
      (its state carries across pieces, so that equals one walk).
  c3  the thermal-coupled run at full size: the config-0 trace tiled to
      100 ms (50.5M accesses), 100 epochs of 1 ms on the 9 x 128 x 128 fp64
      grid; per epoch the timing is bit-exact, the die activity exact, the
      temperatures within 1e-9 relative and the refresh / throttle factors
      exact.
"""
import os

import numpy as np
import pytest

import thermal_oracle as to
from helpers import OracleRun, Setup, activity_of, make_context
from hbfsim_b200 import workloads as wl

pytestmark = pytest.mark.gpu

GIB = 1 << 30
REL = 1e-9
PIECE = 1 << 25


def _host(t, dtype):
    return t.cpu().numpy().view(dtype)


def test_c1_full_trace(tmp_path):
    import torch
    setup = Setup(profile=wl.c0_profile(), model=3, stacks=4, stripe=4096)
    setup.ranges = [(wl.RANGE_BASE, 60 * GIB, 1, 1)]
    ctx = make_context(setup, str(tmp_path))
    bases, counts = wl.c1_segments(seed=0, steps=8)
    address, nbytes, op, arrival = wl.expand_segments(bases, counts, device="cuda")
    n = address.numel()
    assert n == 279_204_864
    out = ctx.submit(address, nbytes, op, arrival)
    torch.cuda.synchronize()
    ctx.flush()
    assert ctx.batch_stats()["device_errors"] == 0
    oracle = OracleRun(setup)
    threads = os.cpu_count() or 1
    modeled = 0
    for lo in range(0, n, PIECE):
        hi = min(n, lo + PIECE)
        part = (_host(address[lo:hi], np.uint64), _host(nbytes[lo:hi], np.uint32),
                _host(op[lo:hi], np.uint8), _host(arrival[lo:hi], np.uint64))
        done, latency, status, stats = oracle.run(*part, threads=threads)
        g_status = _host(out.status[lo:hi], np.uint8)
        bad = np.flatnonzero(g_status != status)
        assert bad.size == 0, f"status differs at {lo + bad[:5]}"
        g_done = _host(out.done_ns[lo:hi], np.uint64)
        bad = np.flatnonzero(g_done != done)
        assert bad.size == 0, f"done differs at {lo + bad[:5]}: {g_done[bad[:5]]} vs {done[bad[:5]]}"
        assert np.array_equal(_host(out.latency_ns[lo:hi], np.uint64), latency), f"latency {lo}"
        modeled += stats["modeled"]
    assert np.array_equal(ctx.get_state(), oracle.state), "end state"
    st = ctx.batch_stats()
    assert st["modeled"] == modeled and st["bypass"] == n - modeled
    ctx.close()


def test_c3_full_run(tmp_path):
    import torch
    setup = Setup(profile=wl.c0_profile(), model=3, stacks=1, stripe=4096)
    setup.ranges = [(wl.RANGE_BASE, 64 * GIB, 1, 3)]
    ctx = make_context(setup, str(tmp_path))
    grid, fp, power, refresh, throttle = wl.c3_thermal()
    ctx.thermal_configure(grid, fp, power, refresh, throttle)
    channels, dies = 16, 4
    n_dies = channels * dies
    owner = to.die_floorplan((len(grid["layers"]), grid["ny"], grid["nx"]), fp["z0"],
                             fp["z_count"], fp["x0"], fp["x1"], fp["y0"], fp["y1"])
    oracle = OracleRun(setup)
    ogrid = to.ThermalGrid(grid)
    ctrl = to.Controller(1, channels, dies, refresh, throttle)
    arrays, cuts = wl.c3_trace()
    dev = [torch.from_numpy(a.view(dt)).cuda() for a, dt in
           zip(arrays, (np.int64, np.int32, np.uint8, np.int64))]
    threads = os.cpu_count() or 1
    dt, epoch_ns = wl.C3_EPOCH_NS * 1e-9, wl.C3_EPOCH_NS
    for k in range(wl.C3_EPOCHS):
        lo, hi = cuts[k], cuts[k + 1]
        part = tuple(a[lo:hi] for a in arrays)
        out = ctx.submit(*(t[lo:hi] for t in dev))
        torch.cuda.synchronize()
        want = oracle.run(*part, threads=threads)
        for g, w, name in ((_host(out.status, np.uint8), want[2], "status"),
                           (_host(out.done_ns, np.uint64), want[0], "done"),
                           (_host(out.latency_ns, np.uint64), want[1], "latency")):
            bad = np.flatnonzero(g != w)
            assert bad.size == 0, f"epoch {k}: {name} differs at {lo + bad[:5]}"
        rb, wr = activity_of(setup, oracle, part, want[2])
        g_rb, g_wr = ctx.die_activity(n_dies)
        assert np.array_equal(g_rb, rb) and np.array_equal(g_wr, wr), f"epoch {k}: activity"
        ctx.advance_epoch(dt)
        p = to.cell_power(owner, n_dies, rb, wr, power["idle_w"], power["read_j_per_byte"],
                          power["write_j_per_access"], dt)
        t_want = ogrid.step(p, dt)
        t_got = ctx.temperatures(owner.size)
        rel = np.max(np.abs(t_got - t_want) / np.abs(t_want))
        assert rel < REL, f"epoch {k}: temperatures differ by {rel:.2e}"
        r, th, adm, _ = ctrl.step(ctx.die_temperatures(n_dies), (k + 2) * epoch_ns)
        gr, gt, ga, _ = ctx.thermal_factors(channels, 1)
        assert np.array_equal(gr, r) and np.array_equal(gt, th) and np.array_equal(ga, adm), \
            f"epoch {k}: factors"
        oracle.set_factors(r, th, adm)
    assert np.array_equal(ctx.get_state(), oracle.state)
    ctx.close()

