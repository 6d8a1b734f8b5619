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
