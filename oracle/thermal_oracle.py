"""CPU restatement of the eq3 layered thermal grid step.

TEST INFRASTRUCTURE ONLY: used by tests/ and bench.py's cpu_baseline leg as the
checker for the CUDA thermal solver.  Never imported by the shipped package.

Grid: the exporter's voxel RC network (tools/eq3_layered_export.py:48-114) for
a stack of full-footprint layers on a uniform square xy mesh:
  * lateral edge G = area / (d/(2k) + d/(2k))            (export.py:100-101)
  * vertical edge G = dx*dy / (dz_a/(2kz_a) + dz_b/(2kz_b))
  * Robin boundary on the bottom (z=0) and top (z=nz-1) faces:
      g = dx*dy / (dz/(2kz) + 1/h), ambient = sum(g*T)/sum(g)  (export.py:103-112)
  * capacity = volume * cv                                   (export.py:80-81)
Step: backward Euler, as ThermalModel::advance_to (src/eq3_thermal/thermal.cpp:
242-311): (C/dt + G_b + L) T+ = C/dt T + P + G_b T_amb, solved exactly here with
a sparse LU factor (scipy splu) in place of the reference's dense Cholesky.
"""
from __future__ import annotations

import numpy as np
import scipy.sparse as sp
import scipy.sparse.linalg as spla


def network(stack: dict):
    """Edges (i, j, G), boundary conductance g[n], ambient t[n], capacity c[n].
    Cell index = z*nx*ny + y*nx + x (export.py:57-60 ordering)."""
    nx, ny, cell = stack["nx"], stack["ny"], stack["cell_m"]
    layers = stack["layers"]
    nz = len(layers)
    n = nx * ny * nz
    ii, jj, gg = [], [], []
    gb = np.zeros(n)
    tb = np.zeros(n)
    cap = np.zeros(n)
    for z, layer in enumerate(layers):
        dz = layer["thickness_m"]
        kx, ky, kz = layer["k_xyz_w_m_k"]
        size = (cell, cell, dz)
        for y in range(ny):
            for x in range(nx):
                i = z * nx * ny + y * nx + x
                cap[i] = (cell * cell * dz) * layer["cv_j_m3_k"]
                k = (kx, ky, kz)
                for axis, valid, shift in ((0, x + 1 < nx, 1), (1, y + 1 < ny, nx),
                                           (2, z + 1 < nz, nx * ny)):
                    if not valid:
                        continue
                    if axis < 2:
                        other_size, other_k = size[axis], k[axis]
                    else:
                        other = layers[z + 1]
                        other_size, other_k = other["thickness_m"], other["k_xyz_w_m_k"][2]
                    area = 1.0
                    for a in range(3):
                        if a != axis:
                            area *= size[a]
                    resistance = size[axis] / (2 * k[axis]) + other_size / (2 * other_k)
                    ii.append(i)
                    jj.append(i + shift)
                    gg.append(area / resistance)
                conductance, heat = 0.0, 0.0
                for side, enabled in (("bottom", z == 0), ("top", z == nz - 1)):
                    if not enabled:
                        continue
                    bc = stack[side]
                    h = bc["h_w_m2_k"]
                    g = 0.0 if h == 0 else size[0] * size[1] / (size[2] / (2 * kz) + 1 / h)
                    conductance += g
                    heat += g * bc["ambient_k"]
                gb[i] = conductance
                tb[i] = heat / conductance if conductance else stack["initial_k"]
    return np.array(ii), np.array(jj), np.array(gg), gb, tb, cap


class ThermalGrid:
    """Backward-Euler stepping of the layered grid with an exact sparse solve."""

    def __init__(self, stack: dict):
        self.stack = stack
        self.i, self.j, self.g, self.gb, self.tb, self.cap = network(stack)
        self.n = self.cap.size
        self.temperature = np.full(self.n, float(stack["initial_k"]))
        lap = sp.coo_matrix((self.g, (self.i, self.j)), shape=(self.n, self.n))
        lap = lap + lap.T
        self.lap = sp.diags(np.asarray(lap.sum(axis=1)).ravel()) - lap
        self._factors: dict[float, object] = {}

    def _factor(self, dt: float):
        f = self._factors.get(dt)
        if f is None:
            a = (sp.diags(self.cap / dt + self.gb) + self.lap).tocsc()
            f = spla.splu(a)
            self._factors[dt] = f
        return f

    def step(self, power_w: np.ndarray, dt: float) -> np.ndarray:
        rhs = self.cap / dt * self.temperature + power_w + self.gb * self.tb
        self.temperature = self._factor(dt).solve(rhs)
        return self.temperature

    def run(self, powers, dt: float):
        """Steps at [s*dt, (s+1)*dt): the step length is computed as the
        difference of the two end times, as the reference segments its clock."""
        out = []
        for s, p in enumerate(powers):
            step_dt = dt * (s + 1) - dt * s
            out.append(self.step(np.asarray(p, dtype=np.float64), step_dt).copy())
        return out


# ---------------------------------------------------------------------------
# Epoch coupling: die activity -> cell power, and the refresh / throttle
# controller.  The refresh-doubling law and the per-die power law come from
# the benchmark's thermal-coupled configuration (the reference marks both
# NOT_IMPLEMENTED), so their parity is unpinned; the throttle levels follow CpuService's control
# sample (src/eq3_thermal/cpu_service.cpp:221-247) with the decision applied
# at once at each epoch boundary (no action delay or dwell).

def die_floorplan(owner_shape, z0, z_count, x0, x1, y0, y1):
    """Cell -> owning die (-1 = none), cell index z*nx*ny + y*nx + x."""
    nz, ny, nx = owner_shape
    owner = np.full(nz * ny * nx, -1, np.int64)
    for d in range(len(z0)):
        for z in range(z0[d], z0[d] + z_count[d]):
            for y in range(y0[d], y1[d]):
                for x in range(x0[d], x1[d]):
                    i = z * nx * ny + y * nx + x
                    assert owner[i] < 0, "overlapping dies"
                    owner[i] = d
    return owner


def cell_power(owner, dies, read_bytes, writes, idle_w, j_per_byte, j_per_write, dt):
    """Die power = idle + (read bytes * J/B + writes * J/write) / dt, spread
    evenly over the die's cells."""
    die_w = idle_w + (np.asarray(read_bytes, np.float64) * j_per_byte +
                      np.asarray(writes, np.float64) * j_per_write) / dt
    cells = np.bincount(owner[owner >= 0], minlength=dies).astype(np.float64)
    p = np.zeros(owner.size)
    m = owner >= 0
    p[m] = die_w[owner[m]] / cells[owner[m]]
    return p


def die_mean(owner, dies, temperature):
    m = owner >= 0
    s = np.bincount(owner[m], weights=temperature[m], minlength=dies)
    c = np.bincount(owner[m], minlength=dies)
    return np.where(c > 0, s / np.maximum(c, 1), 0.0)


class Controller:
    """Refresh permille per local channel, throttle level / permille /
    admit-after tick per stack, from per-die temperatures (global die index
    g*D+d; stack of channel g = g mod stacks)."""

    def __init__(self, stacks, channels_total, dies, refresh, throttle,
                 shard_rank=0, shard_count=1):
        self.stacks, self.channels_total, self.dies = stacks, channels_total, dies
        self.refresh, self.throttle = refresh, throttle
        self.rank, self.shards = shard_rank, shard_count
        self.level = np.zeros(stacks, np.int64)

    def step(self, die_temp, next_epoch_end):
        th = self.throttle
        thresholds = (th["light_k"], th["severe_k"], th["shutdown_k"])
        permille = np.zeros(self.stacks, np.uint32)
        admit = np.zeros(self.stacks, np.uint64)
        for s in range(self.stacks):
            hot = 0.0
            for g in range(s, self.channels_total, self.stacks):
                hot = max(hot, float(np.max(die_temp[g * self.dies:(g + 1) * self.dies])))
            applied = int(self.level[s])
            desired = sum(1 for t in thresholds if hot >= t)
            if desired < applied and hot >= thresholds[applied - 1] - th["hysteresis_k"]:
                desired = applied
            self.level[s] = desired
            permille[s] = (th["light_permille"] if desired == 1 else
                           th["severe_permille"] if desired >= 2 else 1000)
            admit[s] = next_epoch_end if desired == 3 else 0
        local = -(-self.channels_total // self.shards)
        refresh = np.zeros(local, np.uint32)
        rf = self.refresh
        for c in range(local):
            g = c * self.shards + self.rank
            total = 0
            if g < self.channels_total:
                for d in range(self.dies):
                    t = float(die_temp[g * self.dies + d])
                    share = rf["base_permille"]
                    if t >= rf["onset_k"]:
                        share <<= min(20, int(np.floor((t - rf["onset_k"]) / rf["step_k"])))
                    total += share
                total //= self.dies
            refresh[c] = min(total, rf["cap_permille"])
        return refresh, permille, admit, self.level.copy()
