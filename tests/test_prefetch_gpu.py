"""GPU parity of the prefetch-model sweep (reference:
src/prefetch/prefetch_model.cpp simulate_prefetch, one warp per sweep cell):
every statistic equal to the reference model's (tests/golden/
prefetch_goldens.json, produced by the reference compiled from source) and to
the oracle's (oracle/hbf_oracle.c or_prefetch_run, pinned to the same
goldens) on larger sweeps."""
import json
from pathlib import Path

import numpy as np
import pytest

import hbf_oracle as ho
from hbfsim_b200 import prefetch_sweep

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "prefetch_goldens.json"
KEYS = ("policy", "accuracy", "lead", "buffer", "in_flight", "read_ns", "compute_ns", "seed")


def as_cell(c):
    return {"policy": int(c["policy"]), "accuracy": c["accuracy"],
            "lead_distance": c["lead"], "buffer_pages": c["buffer"],
            "max_in_flight": c["in_flight"], "read_latency_ns": c["read_ns"],
            "compute_ns_per_access": c["compute_ns"], "seed": c["seed"]}


def device_pages(pages):
    import torch
    return torch.from_numpy(np.ascontiguousarray(pages, np.uint64).view(np.int64)).cuda()


def test_reference_cells():
    for s in json.loads(GOLDEN.read_text()):
        cells = [dict(zip(KEYS, row[:8])) for row in s["cells"]]
        got = prefetch_sweep(device_pages(s["pages"]), [as_cell(c) for c in cells])
        for row, g in zip(s["cells"], got):
            assert [g[f] for f in ho.PREFETCH_STATS] == row[8:], (s["stream"], row[:8])


def moe_stream(rng, tokens, layers=48, experts=128, top=8, pages_per_expert=2):
    out = []
    for _ in range(tokens):
        for layer in range(layers):
            chosen = rng.permutation(experts)[:top]
            base = (layer * experts + chosen) * pages_per_expert
            out.append((base[:, None] + np.arange(pages_per_expert)).ravel())
    return np.concatenate(out).astype(np.uint64)


def test_large_sweep_matches_oracle():
    """A 200k-access mixed stream (MoE-shaped pages, sequential runs, a
    looping working set) and 48 random cells, against the oracle."""
    rng = np.random.default_rng(3)
    moe = moe_stream(rng, 100)
    seq = np.arange(50_000, dtype=np.uint64) + (1 << 30)
    loop = (np.arange(73_200) % 97).astype(np.uint64) + (1 << 31)
    pages = np.concatenate([moe, seq, loop])
    cells = []
    for _ in range(48):
        cells.append({"policy": int(rng.choice([0, 1, 2, 2, 2])),
                      "accuracy": float(rng.choice([0.0, 0.25, 0.6, 0.9, 0.99, 1.0])),
                      "lead": int(rng.choice([1, 4, 16, 100, 3000])),
                      "buffer": int(rng.choice([1, 16, 64, 96, 300])),
                      "in_flight": int(rng.choice([1, 8, 32, 1000, 5000])),
                      "read_ns": int(rng.choice([1_000, 5_000, 20_000])),
                      "compute_ns": int(rng.choice([0, 200, 4_000])),
                      "seed": int(rng.integers(0, 1 << 62))})
    got = prefetch_sweep(device_pages(pages), [as_cell(c) for c in cells])
    for c, g in zip(cells, got):
        want = ho.prefetch_run(pages, c)
        assert [g[f] for f in ho.PREFETCH_STATS] == list(want), c


def test_edge_cases():
    import torch
    from hbfsim_b200 import HbfsimError
    empty = torch.empty(0, dtype=torch.int64, device="cuda")
    out = prefetch_sweep(empty, [as_cell(dict(zip(KEYS, (2, 0.5, 1, 64, 32, 10_000, 0, 1))))])
    assert all(v == 0 for v in out[0].values())
    pages = np.array([5, 6, 7, 5, 6, 7, 100, 5], np.uint64)
    cells = [dict(zip(KEYS, c)) for c in ((2, 1.0, 1, 0, 0, 1_000, 0, 9),   # zero -> one
                                          (2, 0.5, 0, 8, 4, 1_000, 10, 9),  # lead 0: no prefetch
                                          (1, 0.0, 3, 2, 1, 700, 5, 9))]
    got = prefetch_sweep(device_pages(pages), [as_cell(c) for c in cells])
    for c, g in zip(cells, got):
        assert [g[f] for f in ho.PREFETCH_STATS] == list(ho.prefetch_run(pages, c))
    with pytest.raises(HbfsimError):
        prefetch_sweep(device_pages(pages), [{"policy": 7}])
