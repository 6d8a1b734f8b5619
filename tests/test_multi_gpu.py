"""Two GPU ranks (one process per GPU, NCCL): each rank times its own
channels of one trace, then one sharded thermal epoch all-gathers the die
activity and runs the replicated grid step.  Checked against the unsharded
oracle run: per-access ticks, grid temperatures (1e-9) on both ranks, and each
rank's refresh factors for its own channels.  Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest

import thermal_oracle as to
from helpers import OracleRun, Setup, gpu_run, make_context
from hbfsim_b200 import workloads as wl

pytestmark = pytest.mark.gpu

WORLD = 2
STACKS = 2
DT = 1e-3
POWER = {"idle_w": 0.3, "read_j_per_byte": 2e-9 / 128, "write_j_per_access": 50e-9}
REFRESH = {"onset_k": 318.3, "step_k": 0.02, "base_permille": 5, "cap_permille": 400}
THROTTLE = {"light_k": 330.0, "severe_k": 340.0, "shutdown_k": 350.0, "hysteresis_k": 1.0,
            "light_permille": 1500, "severe_permille": 3000}


def setup_for(rank=0, world=1):
    p = wl.c0_profile()
    s = Setup(profile=p, model=3, stacks=STACKS, stripe=4096, shard_rank=rank,
              shard_count=world)
    s.ranges = [(wl.RANGE_BASE, p["capacity_bytes"] - (1 << 20), 1, 3)]
    return s


def grid_setup():
    from test_thermal_gpu import floorplan, stack_desc
    desc = stack_desc(16, 16, 4)
    fp = floorplan(STACKS, 16, 4, 16)
    return desc, fp


def trace():
    return wl.c0_trace(200_000, seed=21, range_length=wl.c0_profile()["capacity_bytes"] - (1 << 20))


def _rank(rank, port, tmp, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch
    import torch.distributed as dist
    from hbfsim_b200 import sharding
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        s = setup_for(rank, WORLD)
        ctx = make_context(s, f"{tmp}/rank{rank}")
        desc, fp = grid_setup()
        ctx.thermal_configure(desc, fp, POWER, REFRESH, THROTTLE)
        done, lat, status = gpu_run(ctx, trace())
        sharding.advance_epoch_sharded(ctx, DT, s.local_channels, 4, s.channels_total)
        cells = 16 * 16 * len(desc["layers"])
        temps = ctx.temperatures(cells)
        refresh, _, _, _ = ctx.thermal_factors(s.local_channels, STACKS)
        die_t = ctx.die_temperatures(s.channels_total * 4)
        q.put((rank, done, status, temps, refresh, die_t))
        ctx.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def test_two_rank_sharded_epoch(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, str(tmp_path), q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(WORLD):
        r, *rest = q.get(timeout=600)
        got[r] = rest
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0

    a = trace()
    full = setup_for()
    want = OracleRun(full).run(*a, threads=8)
    timed = want[2] == 1
    merged = np.zeros_like(want[0])
    for r in range(WORLD):
        done, status = got[r][0], got[r][1]
        merged[status == 1] = done[status == 1]
    assert np.array_equal(merged[timed], want[0][timed])

    # one epoch on the unsharded activity
    import hbf_oracle as ho
    o = OracleRun(full)
    dec = ho.decode(o.ranges, o.count, o.geometry, *a[:3])
    dies = 4
    idx = dec["channel"][timed] * dies + dec["die"][timed]
    n_dies = full.channels_total * dies
    rb = np.bincount(idx, weights=np.where(a[2][timed] == 0, a[1][timed], 0), minlength=n_dies)
    wr = np.bincount(idx, weights=(a[2][timed] == 1), minlength=n_dies)
    desc, fp = grid_setup()
    owner = to.die_floorplan((len(desc["layers"]), 16, 16), fp["z0"], fp["z_count"],
                             fp["x0"], fp["x1"], fp["y0"], fp["y1"])
    grid = to.ThermalGrid(desc)
    p = to.cell_power(owner, n_dies, rb, wr, POWER["idle_w"], POWER["read_j_per_byte"],
                      POWER["write_j_per_access"], DT)
    t_want = grid.step(p, DT)
    for r in range(WORLD):
        temps, refresh, die_t = got[r][2], got[r][3], got[r][4]
        assert np.max(np.abs(temps - t_want) / t_want) < 1e-9, f"rank {r}"
        ctrl = to.Controller(STACKS, full.channels_total, dies, REFRESH, THROTTLE, r, WORLD)
        want_refresh = ctrl.step(die_t, 2 * 1_000_000)[0]
        assert np.array_equal(refresh, want_refresh), f"rank {r}"
    assert np.array_equal(got[0][4], got[1][4])  # replicated step: identical die temps
    assert np.ptp(got[0][4]) > 0  # the dies heated unevenly
