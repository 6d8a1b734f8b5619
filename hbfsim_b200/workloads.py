"""Synthetic workloads shaped like the BASELINE configs (seeded, reproducible).

No public dataset or model weights are involved: traces are generated from a
seed with the shapes, sizes and value distributions of the configs, and the
media profiles below follow the legacy profile schema
(configs/schema/hbf-profile.schema.json) unchanged.

c0  timing-only trace: 1,048,576 accesses on one 64 GiB range; 95 % reads;
    128 B (80 %) or 4 KiB (20 %), 128-B aligned; 70 % of accesses in
    sequential 16 KiB runs (128 steps of 128 B) from uniform starts, 30 %
    uniform; exponential arrival gaps of mean 2 ns (rounded to whole ns);
    1 stack x 16 channels x 4 dies x 4 planes, 16 KiB page, tR 3000 ns,
    tPROG 200000 ns, 8 GB/s per channel, 4 KiB striping.  A 4 KiB access that
    would cross a 16 KiB page is moved down to end at the page boundary.
c1  MoE weight-streaming decode shaped like Qwen3-30B-A3B: 48 layers x 128
    experts of 3*(2048*768) bf16 laid out contiguously in a 60 GiB range;
    8 decode steps x 32 tokens; each token picks 8 distinct experts from
    Zipf(1.1) over a per-layer random permutation; every weight byte of the
    union of experts of a layer-step is read in 1 KiB reads.  Attention
    weights (4096*2048 bf16 per layer) live in HBM: they are read too, as
    bypass accesses outside the HBF range.  Arrival process (fixed by this
    build): one 1 KiB read per ns, i.e. arrival = access index.  Profile as
    c0 with 4 stacks (64 channels).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

GIB = 1 << 30
RANGE_BASE = 0x7F00_0000_0000   # synthetic device address of the HBF range
HBM_BASE = 0x7E00_0000_0000     # synthetic address of HBM-resident weights


def c0_profile() -> dict:
    return {
        "name": "baseline-c0",
        "capacity_bytes": 64 * GIB,
        "page_bytes": 16384,
        "read_latency_ns": 3000,
        "program_latency_ns": 200000,
        "channels": 16,
        "dies_per_channel": 4,
        "planes_per_die": 4,
        "pages_per_block": 256,
        "channel_width_bits": 8,
        "channel_transfer_rate_mtps": 8000,
        "queue_depth": 128,
        "aggregate_bandwidth_bytes_per_s": 128_000_000_000,
        "hbm_cache_bytes": 0,
        "reference_sample_rate": 0.0,
        "reference_warmup_requests": 0,
        "time_scale": 1,
        "timing_tolerance_ns": 10000,
    }


def vmem_profile(pages=(1, 4, 16, 64, 256, 512),
                 cumulative=(11_133, 41_495, 168_606, 2_824_351, 10_767_793, 20_254_374),
                 program_ns: int = 408_305, time_scale: int = 1) -> dict:
    """A FAST-model profile with an empirical burst curve (the schema's
    empirical_vmem block): 4 KiB pages, P50 cumulative read time of a run of
    k sequential pages at six breakpoints, the shape of the reference's
    cd8p-vmem-p50 profile.  The source hash is a placeholder."""
    curve = [{"pages": int(k), "cumulative_ns": int(c), "p95_ns": int(c)}
             for k, c in zip(pages, cumulative)]
    return {
        "name": "vmem-burst",
        "capacity_bytes": 16 * GIB,
        "page_bytes": 4096,
        "read_latency_ns": int(cumulative[0]),
        "program_latency_ns": int(program_ns),
        "channels": 32,
        "dies_per_channel": 8,
        "planes_per_die": 4,
        "pages_per_block": 256,
        "channel_width_bits": 8,
        "channel_transfer_rate_mtps": 1600,
        "queue_depth": 1,
        "aggregate_bandwidth_bytes_per_s": 103_540_697,
        "hbm_cache_bytes": 0,
        "reference_sample_rate": 0.0,
        "reference_warmup_requests": 0,
        "time_scale": int(time_scale),
        "timing_tolerance_ns": 27_105,
        "empirical_vmem": {
            "source_kind": "synthetic",
            "source_sha256": "0" * 64,
            "source_capacity_bytes": 16 * GIB,
            "quantile": "p50",
            "sample_count": 1,
            "read_curve": curve,
            "program_p50_ns": int(program_ns),
            "program_p95_ns": int(program_ns),
        },
    }


def vmem_trace(n: int = 1 << 20, seed: int = 0, range_length: int = 15 * GIB,
               base: int = RANGE_BASE, mean_run: float = 48.0, write_p: float = 0.05):
    """Page-granular trace for the empirical burst model: streaks of
    sequential 4 KiB pages (geometric lengths, mean `mean_run`, one operation
    per streak) from uniform start pages; arrivals cumulative exponential
    gaps of mean 2 ns.  Returns (address, bytes, op, arrival) numpy arrays."""
    rng = np.random.default_rng(seed)
    pages_total = range_length // 4096
    streaks = int(n / mean_run * 1.2) + 16
    length = np.minimum(rng.geometric(1.0 / mean_run, streaks), 4096).astype(np.int64)
    while int(length.sum()) < n:
        length = np.concatenate([length, length])
    start = rng.integers(0, pages_total - 4096, length.size, dtype=np.int64)
    writes = (rng.random(length.size) < write_p).astype(np.uint8)
    which = np.repeat(np.arange(length.size), length)[:n]
    first = np.cumsum(length) - length
    page = start[which] + (np.arange(n, dtype=np.int64) - first[which])
    op = writes[which]
    size = np.where(rng.random(n) < 0.5, 4096, 512).astype(np.uint32)
    gaps = np.rint(rng.exponential(2.0, n)).astype(np.uint64)
    arrival = np.cumsum(gaps, dtype=np.uint64)
    address = (base + page.astype(np.uint64) * 4096).astype(np.uint64)
    return address, size, op, arrival


def c4_profile() -> dict:
    p = c0_profile()
    p.update(name="baseline-c4", dies_per_channel=8, capacity_bytes=128 * GIB)
    return p


@dataclass
class Workload:
    name: str
    profile: dict
    stacks: int
    stripe_bytes: int
    range_base: int
    range_length: int
    extra: dict = field(default_factory=dict)

    def write_profile(self, directory: str | os.PathLike) -> str:
        path = Path(directory) / f"{self.profile['name']}.json"
        path.write_text(json.dumps(self.profile, indent=2))
        return str(path)

    @property
    def channels_total(self) -> int:
        return self.stacks * self.profile["channels"]

    @property
    def dies(self) -> int:
        return self.profile["dies_per_channel"]


def c0_workload() -> Workload:
    return Workload("c0", c0_profile(), 1, 4096, RANGE_BASE, 64 * GIB)


def c1_workload() -> Workload:
    return Workload("c1", c0_profile(), 4, 4096, RANGE_BASE, 60 * GIB)


def c0_trace(n: int = 1 << 20, seed: int = 0, range_length: int = 64 * GIB,
             base: int = RANGE_BASE):
    """Returns (address u64, bytes u32, op u8, arrival u64) numpy arrays."""
    rng = np.random.default_rng(seed)
    run = 128                                   # 16 KiB / 128 B
    blocks = (n + run - 1) // run
    sequential = rng.random(blocks) < 0.7
    starts = rng.integers(0, (range_length - 16384) // 128, blocks, dtype=np.int64) * 128
    uniform = rng.integers(0, (range_length - 4096) // 128, n, dtype=np.int64) * 128
    i = np.arange(n, dtype=np.int64)
    b = i // run
    offset = np.where(sequential[b], starts[b] + (i % run) * 128, uniform)
    size = np.where(rng.random(n) < 0.8, 128, 4096).astype(np.int64)
    in_page = offset % 16384
    over = np.maximum(in_page + size - 16384, 0)
    offset = offset - over
    op = (rng.random(n) < 0.05).astype(np.uint8)
    gaps = np.rint(rng.exponential(2.0, n)).astype(np.uint64)
    arrival = np.cumsum(gaps, dtype=np.uint64)
    address = (offset + base).astype(np.uint64)
    return address, size.astype(np.uint32), op, arrival


# ---------------------------------------------------------------------------
# c3: the config-0 trace tiled to 100 ms of arrivals, driving a 9 x 128 x 128
# fp64 grid (one logic layer under 8 NAND layers), 1 ms epochs, 45 C ambient;
# per-die power 0.5 W idle + 2 nJ per 128-B read + 50 nJ per write; refresh
# doubles every 10 C above 70 C, taken from channel bandwidth.
C3_EPOCHS, C3_EPOCH_NS = 100, 1_000_000


def c3_thermal(stacks: int = 1, channels: int = 16, dies: int = 4, cell_m: float = 100e-6):
    """Grid description, floorplan (die -> cell box), power, refresh and
    throttle laws of config 3.  Channels form a square array of cell tiles;
    die d of a channel heats NAND layers 1 + 2d and 2 + 2d (4 dies) -- with
    8 dies, layer 1 + d.  `cell_m` is the cell pitch (100 um: one stack on a
    12.8 mm square)."""
    silicon = {"cv_j_m3_k": 1.66e6, "k_xyz_w_m_k": [148.0, 148.0, 148.0]}
    nand = {"cv_j_m3_k": 1.75e6, "k_xyz_w_m_k": [110.0, 110.0, 35.0]}
    grid = {"nx": 128, "ny": 128, "cell_m": cell_m,
            "layers": [dict(silicon, thickness_m=100e-6)] +
                      [dict(nand, thickness_m=50e-6) for _ in range(8)],
            "bottom": {"h_w_m2_k": 0.0, "ambient_k": 318.15},
            "top": {"h_w_m2_k": 2.0e4, "ambient_k": 318.15}, "initial_k": 318.15}
    total = stacks * channels
    side = int(round(total ** 0.5))
    while total % side:
        side -= 1
    tx, ty = 128 // side, 128 // (total // side)
    per_layer = 8 // dies
    n = total * dies
    fp = {k: np.zeros(n, np.uint32) for k in ("z0", "z_count", "x0", "x1", "y0", "y1")}
    for g in range(total):
        for d in range(dies):
            i = g * dies + d
            fp["z0"][i], fp["z_count"][i] = 1 + per_layer * d, per_layer
            fp["x0"][i], fp["x1"][i] = (g % side) * tx, (g % side) * tx + tx
            fp["y0"][i], fp["y1"][i] = (g // side) * ty, (g // side) * ty + ty
    power = {"idle_w": 0.5, "read_j_per_byte": 2e-9 / 128, "write_j_per_access": 50e-9}
    refresh = {"onset_k": 343.15, "step_k": 10.0, "base_permille": 10, "cap_permille": 500}
    throttle = {"light_k": 358.15, "severe_k": 368.15, "shutdown_k": 378.15,
                "hysteresis_k": 2.0, "light_permille": 1500, "severe_permille": 3000}
    return grid, fp, power, refresh, throttle


def c3_trace(epochs: int = C3_EPOCHS, epoch_ns: int = C3_EPOCH_NS, seed: int = 0):
    """The config-0 trace tiled in time until it covers `epochs` epochs:
    (address, bytes, op, arrival) numpy arrays cut at the last epoch's end,
    and the epoch boundaries as indices (cuts[k]..cuts[k+1] is epoch k)."""
    a, b, o, t = c0_trace(1 << 20, seed=seed)
    span = int(t[-1]) + 1
    reps = -(-epochs * epoch_ns // span)
    arrival = (np.tile(t, reps) +
               np.repeat(np.arange(reps, dtype=np.uint64) * np.uint64(span), t.size))
    cuts = np.searchsorted(arrival, np.arange(epochs + 1, dtype=np.uint64) * np.uint64(epoch_ns))
    n = int(cuts[-1])
    return ((np.tile(a, reps)[:n], np.tile(b, reps)[:n], np.tile(o, reps)[:n], arrival[:n]),
            [int(c) for c in cuts])


EXPERT_BYTES = 3 * 2048 * 768 * 2
ATTN_BYTES = 4096 * 2048 * 2
READ_BYTES = 1024


def c1_segments(seed: int = 0, steps: int = 8, layers: int = 48, experts: int = 128,
                batch: int = 32, topk: int = 8, zipf_s: float = 1.1):
    """Read segments of the MoE decode trace, in issue order.

    Returns (base u64[S], count i64[S]): segment k is `count[k]` consecutive
    1 KiB reads starting at `base[k]`.  Per layer-step: the layer's attention
    weights (HBM, bypass) then the union of selected experts (HBF), in
    ascending expert id."""
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, experts + 1, dtype=np.float64)
    p = ranks ** -zipf_s
    p /= p.sum()
    perms = np.stack([rng.permutation(experts) for _ in range(layers)])
    bases, counts = [], []
    for _ in range(steps):
        for layer in range(layers):
            chosen = set()
            for _ in range(batch):
                picks = rng.choice(experts, size=topk, replace=False, p=p)
                chosen.update(int(perms[layer][r]) for r in picks)
            bases.append(HBM_BASE + layer * ATTN_BYTES)
            counts.append(ATTN_BYTES // READ_BYTES)
            for e in sorted(chosen):
                bases.append(RANGE_BASE + (layer * experts + e) * EXPERT_BYTES)
                counts.append(EXPERT_BYTES // READ_BYTES)
    return np.array(bases, dtype=np.uint64), np.array(counts, dtype=np.int64)


def expand_segments(bases, counts, device=None):
    """Expand read segments into SoA arrays.  With `device` set the expansion
    runs in torch on that device (int64 tensors carry the u64 bit patterns);
    otherwise numpy arrays are returned."""
    n = int(counts.sum())
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int64)
    if device is None:
        seg_base = np.repeat(bases.astype(np.int64), counts)
        seg_start = np.repeat(starts, counts)
        idx = np.arange(n, dtype=np.int64)
        address = (seg_base + (idx - seg_start) * READ_BYTES).astype(np.uint64)
        return (address, np.full(n, READ_BYTES, np.uint32), np.zeros(n, np.uint8),
                idx.astype(np.uint64))
    import torch
    c = torch.as_tensor(counts, device=device)
    seg_base = torch.repeat_interleave(torch.as_tensor(bases.astype(np.int64), device=device), c)
    seg_start = torch.repeat_interleave(torch.as_tensor(starts, device=device), c)
    idx = torch.arange(n, dtype=torch.int64, device=device)
    address = seg_base + (idx - seg_start) * READ_BYTES
    del seg_base, seg_start
    nbytes = torch.full((n,), READ_BYTES, dtype=torch.int32, device=device)
    op = torch.zeros(n, dtype=torch.uint8, device=device)
    return address, nbytes, op, idx


# ---------------------------------------------------------------------------
# c2: Capacity-mode paged KV shaped like Llama-3-8B.  32 layers x 8 KV heads
# x head_dim 128 x bf16 x (K, V) = 4096 B per token-layer: one 4 KiB LRU page
# per token and layer.  64 sequences with lengths uniform on [1024, 32768];
# each decode step, layer by layer and sequence by sequence, writes the new
# token's page (the append) and then reads every page of the sequence
# including it.  HBM holds 20 % of the KV pages.  KV of (layer, sequence)
# is contiguous, with room for the tokens the run appends.
C2_LAYERS, C2_SEQS, C2_PAGE = 32, 64, 4096


def c2_lengths(seed: int = 0, seqs: int = C2_SEQS, lmin: int = 1024, lmax: int = 32768):
    return np.random.default_rng(seed).integers(lmin, lmax + 1, seqs)


def c2_step(lengths, step: int, steps_total: int, layers: int = C2_LAYERS,
            base: int = RANGE_BASE, device=None):
    """(address u64, bytes u32, op u8) of one decode step, in issue order.
    With `device` set, torch tensors built on that device (int64 carrying
    the u64 addresses)."""
    if device is not None:
        return _c2_step_torch(lengths, step, steps_total, layers, base, device)
    lengths = np.asarray(lengths, np.int64)
    room = lengths + steps_total
    region = np.concatenate([[0], np.cumsum(np.tile(room, layers))[:-1]])  # per (layer, seq)
    cur = lengths + step                       # tokens before this step's append
    per = np.tile(cur + 2, layers)             # 1 write + (cur + 1) reads
    n = int(per.sum())
    starts = np.concatenate([[0], np.cumsum(per)[:-1]])
    k = np.arange(n, dtype=np.int64) - np.repeat(starts, per)   # position in group
    grp_region = np.repeat(region, per)
    grp_cur = np.repeat(np.tile(cur, layers), per)
    token = np.where(k == 0, grp_cur, k - 1)                   # write new, then read 0..cur
    page = grp_region + token
    op = (k == 0).astype(np.uint8)
    address = (base + page * C2_PAGE).astype(np.uint64)
    return address, np.full(n, C2_PAGE, np.uint32), op


def c2_frames(lengths, layers: int = C2_LAYERS, fraction: float = 0.2) -> int:
    return int(int(np.asarray(lengths).sum()) * layers * fraction)


def _c2_step_torch(lengths, step, steps_total, layers, base, device):
    import torch
    lengths = torch.as_tensor(np.asarray(lengths, np.int64), device=device)
    room = lengths + steps_total
    tiled_room = room.repeat(layers)
    region = torch.cumsum(tiled_room, 0) - tiled_room
    cur = (lengths + step).repeat(layers)
    per = cur + 2
    n = int(per.sum().item())
    starts = torch.cumsum(per, 0) - per
    k = torch.arange(n, dtype=torch.int64, device=device) - torch.repeat_interleave(starts, per)
    token = torch.where(k == 0, torch.repeat_interleave(cur, per), k - 1)
    page = torch.repeat_interleave(region, per) + token
    address = base + page * C2_PAGE
    op = (k == 0).to(torch.uint8)
    return address, torch.full((n,), C2_PAGE, dtype=torch.int32, device=device), op


# ---------------------------------------------------------------------------
# c4: 2^32 accesses on 16 stacks x 16 channels x 8 dies x 4 planes; 60 % the
# MoE weight-streaming pattern (config 1's expert reads), 40 % the paged-KV
# pattern (config 2's page reads and appends, here plain timed accesses of a
# second range), interleaved by arrival.  Global access i is a MoE access
# when i % 5 < 3 and a KV access otherwise, each stream consumed in its own
# order; arrival(i) = floor(i * span / 2^32): the whole trace covers `span`
# ns of simulated time (100 epochs of 1 ms, as config 3), about 43 accesses
# per ns.  Channels are sharded across ranks (channel g on rank g % world),
# and each rank keeps only its accesses: generation is replicated, no trace
# record crosses between GPUs.
C4_N = 1 << 32
C4_STACKS = 16
C4_SHARDS = 8      # channel shards (channel g in shard g % 8), spread over the GPUs
C4_SPAN_NS = C3_EPOCHS * C3_EPOCH_NS
C4_MOE_LENGTH = 60 * GIB
C4_KV_BASE = RANGE_BASE + 64 * GIB


def c4_kv_length(lengths, steps_total: int) -> int:
    """Bytes of the KV range: every (layer, sequence) region holds its
    tokens plus the ones the run appends."""
    room = int(np.asarray(lengths, np.int64).sum()) + len(lengths) * steps_total
    return room * C2_LAYERS * C2_PAGE


class C4Trace:
    """Device-side generator of the config-4 trace, filtered to one rank's
    channels.  `channel_of(address)` must give the global channel of an
    address (the context's decode); `keep(channel)` selects the rank's."""

    def __init__(self, device, seed: int = 0, n: int = C4_N, span_ns: int = C4_SPAN_NS):
        self.device = device
        self.n = n
        self.span = span_ns
        self.n_moe = 3 * (n // 5) + min(3, n % 5)
        self.n_kv = n - self.n_moe
        # MoE: config-1 expert segments (attention weights left out: they
        # live in HBM), enough decode steps for the MoE share
        per_step = 48 * 77 * (EXPERT_BYTES // READ_BYTES)
        steps = self.n_moe // per_step + 2
        bases, counts = c1_segments(seed=seed, steps=steps)
        expert = bases >= RANGE_BASE
        self.moe_bases, self.moe_counts = bases[expert], counts[expert]
        while int(self.moe_counts.sum()) < self.n_moe:  # Zipf unions vary: top up
            b, c = c1_segments(seed=seed + 1000 + steps, steps=4)
            e = b >= RANGE_BASE
            self.moe_bases = np.concatenate([self.moe_bases, b[e]])
            self.moe_counts = np.concatenate([self.moe_counts, c[e]])
            steps += 4
        # KV: config-2 decode steps until the KV share is covered
        self.lengths = c2_lengths(seed)
        per = C2_LAYERS * (int(self.lengths.sum()) + 2 * C2_SEQS)
        self.kv_steps = self.n_kv // per + 2
        self.kv_length = c4_kv_length(self.lengths, self.kv_steps)

    def _moe(self):
        """MoE accesses in order, as (address, count) tensors per group of
        segments."""
        import torch
        seg = 0
        group = 4096
        while seg < len(self.moe_bases):
            b, c = self.moe_bases[seg:seg + group], self.moe_counts[seg:seg + group]
            address, _, _, _ = expand_segments(b, c, device=self.device)
            yield address, torch.full_like(address, READ_BYTES, dtype=torch.int32), \
                torch.zeros_like(address, dtype=torch.uint8)
            seg += group

    def _kv(self):
        for step in range(self.kv_steps):
            yield c2_step(self.lengths, step, self.kv_steps, base=C4_KV_BASE,
                          device=self.device)

    def chunks(self, channel_of, keep, m: int = 1 << 22):
        """Yields the rank's accesses (address, bytes, op, arrival) of
        consecutive blocks of 5*m global indices."""
        import torch
        streams = {"moe": self._moe(), "kv": self._kv()}
        bufs = {"moe": [], "kv": []}
        have = {"moe": 0, "kv": 0}

        def take(name, count):
            while have[name] < count:
                parts = next(streams[name])
                bufs[name].append(parts)
                have[name] += parts[0].numel()
            cat = [torch.cat([p[k] for p in bufs[name]]) for k in range(3)]
            out = [t[:count] for t in cat]
            rest = [t[count:] for t in cat]
            bufs[name] = [rest] if rest[0].numel() else []
            have[name] -= count
            return out

        i0 = 0
        while i0 < self.n:
            blocks = min(m, (self.n - i0) // 5)
            if blocks == 0:  # the tail: fewer than 5 accesses, MoE first
                tail = self.n - i0
                a, b, o = take("moe", min(3, tail))
                if tail > 3:
                    ka, kb, ko = take("kv", tail - 3)
                    a, b, o = torch.cat([a, ka]), torch.cat([b, kb]), torch.cat([o, ko])
                count = a.numel()
            else:
                ma, mb, mo = take("moe", 3 * blocks)
                ka, kb, ko = take("kv", 2 * blocks)
                a = torch.cat([ma.view(blocks, 3), ka.view(blocks, 2)], 1).view(-1)
                b = torch.cat([mb.view(blocks, 3), kb.view(blocks, 2)], 1).view(-1)
                o = torch.cat([mo.view(blocks, 3), ko.view(blocks, 2)], 1).view(-1)
                count = 5 * blocks
            idx = torch.arange(i0, i0 + count, dtype=torch.int64, device=self.device)
            arrival = idx * self.span // self.n
            mine = keep(channel_of(a))
            yield a[mine], b[mine], o[mine], arrival[mine]
            i0 += count
