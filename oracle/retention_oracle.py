"""CPU restatement of the per-block retention-age ledger.

TEST INFRASTRUCTURE ONLY: imported by tests/ (and bench.py's cpu_baseline
leg) as the checker for hbfsim_b200/csrc/retention.cu.  The shipped package
never imports it.

Restates the reference's ReliabilityLedger
(experiments/eq3_system_thermal/reliability.py) over arrays of blocks grouped
by die, as run_maintenance_point.py:189, 225-234 drives it: one cohort per
die per epoch, at the midpoint of the die's previous and current temperature
(or at a given temperature).  Pinned to the reference by
tests/golden/retention_goldens.json, produced by the reference class itself.
"""
from __future__ import annotations

import math

import numpy as np

KB_EV_PER_K = 8.62e-5            # reliability.py:12
DAY_NS = 86_400_000_000_000      # reliability.py:13
TREF_K = 358.15                  # reliability.py:11
NEVER = (1 << 64) - 1


def acceleration(temperature_k: float, ea_ev: float, tref_k: float = TREF_K) -> float:
    """reliability.py:17-23, same operation order."""
    return math.exp(ea_ev / KB_EV_PER_K * (1.0 / tref_k - 1.0 / temperature_k))


class Ledger:
    """Blocks b of die b // blocks_per_die; one accounted frontier."""

    def __init__(self, dies: int, blocks_per_die: int, ea_ev: float = 1.04,
                 initial_age_ns: int = 0, initial_wall_age_ns: int = 0, epoch_ns: int = 0,
                 refresh_trigger: str = "wall_only", initial_temperature_k: float = 318.15):
        n = dies * blocks_per_die
        self.dies, self.blocks_per_die, self.ea_ev = dies, blocks_per_die, ea_ev
        self.trigger = refresh_trigger
        # reliability.py:63-75
        self.age = np.full(n, float(initial_age_ns))
        self.next_due = np.full(n, epoch_ns + DAY_NS - initial_wall_age_ns, np.uint64)
        self.last_commit = np.full(n, NEVER, np.uint64)
        self.counts = np.zeros((4, n), np.uint32)
        self.frontier = epoch_ns
        self.previous = [float(initial_temperature_k)] * dies

    def advance(self, end_ns: int, die_temps, midpoint: bool) -> None:
        """advance_temperature_many (reliability.py:109-135) for every die's
        cohort over [frontier, end_ns)."""
        assert end_ns >= self.frontier
        for d in range(self.dies):
            cur = float(die_temps[d])
            t = (self.previous[d] + cur) / 2 if midpoint else cur
            self.previous[d] = cur
            delta = (end_ns - self.frontier) * acceleration(t, self.ea_ev)
            lo = d * self.blocks_per_die
            self.age[lo:lo + self.blocks_per_die] += delta
        self.frontier = end_ns

    def due(self, at_ns: int):
        """due_reasons (reliability.py:76-88) as bits: 1 wall cadence,
        2 equivalent age (trigger equivalent_age_or_wall)."""
        assert at_ns >= self.frontier
        bits = (np.uint64(at_ns) >= self.next_due).astype(np.uint8)
        if self.trigger == "equivalent_age_or_wall":
            bits |= (self.age >= DAY_NS).astype(np.uint8) * 2
        blocks = np.flatnonzero(bits).astype(np.uint32)
        return blocks, bits[blocks]

    def refresh(self, blocks) -> None:
        """record_refresh_terminal committed at the frontier (172-187)."""
        b = np.asarray(blocks, np.int64)
        self.age[b] = 0.0
        self.last_commit[b] = self.frontier
        self.next_due[b] = self.frontier + DAY_NS

    def erase(self, blocks) -> None:
        """_media_terminal('erase', succeeded, phase_started) (138-159)."""
        for b in blocks:
            self.counts[2, b] += 1
            self.counts[3, b] += 1

    def program(self, blocks) -> None:
        for b in blocks:
            self.counts[0, b] += 1
            self.counts[1, b] += 1


def block_ids(decoded, status, op, dies: int, planes: int, blocks_per_plane: int,
              pages_per_block: int, shard_count: int = 1) -> np.ndarray:
    """Block of every modeled write of a decoded batch (hbf_oracle.decode
    records), in the device ledger's numbering."""
    m = (status == 1) & (op == 1)
    local = decoded["channel"][m] // shard_count
    blk = decoded["page"][m] // pages_per_block
    return (((local.astype(np.int64) * dies + decoded["die"][m]) * planes +
             decoded["plane"][m]) * blocks_per_plane + blk.astype(np.int64))
