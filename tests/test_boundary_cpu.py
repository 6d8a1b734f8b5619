"""CPU-side checks of the drop-in boundary: the library loads, exports every
symbol the public headers declare, and validates arguments the way the
reference C API does -- without any compute call (no GPU here)."""
import ctypes
import json
import re
from pathlib import Path

import pytest

from hbfsim_b200 import _lib, build, workloads

REPO = Path(__file__).resolve().parent.parent


def declared_functions():
    names = set()
    for header in (REPO / "include" / "hbfsim").glob("*.h"):
        text = header.read_text()
        names.update(re.findall(r"\b(hbfsim_[a-z0-9_]+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 25
    for name in names:
        assert hasattr(lib, name), name
    assert set(_lib.SIGNATURES) == names


def test_abi_version(lib):
    assert lib.hbfsim_abi_version() == 1


def _create(lib, profile_path, report_dir, mode=3, ring=64, timeout=10**9):
    enc = lambda v: None if v is None else str(v).encode()
    opts = _lib.Options(enc(profile_path), enc(report_dir), mode, ring, timeout)
    h = ctypes.c_void_p()
    rc = lib.hbfsim_context_create(ctypes.byref(opts), ctypes.byref(h))
    return rc, h


@pytest.mark.parametrize("ring,mode,timeout", [(3, 1, 1), (1, 1, 1), (8192, 1, 1),
                                               (64, 4, 1), (64, 1, 0)])
def test_option_validation(lib, tmp_path, ring, mode, timeout):
    p = workloads.c0_workload().write_profile(tmp_path)
    rc, h = _create(lib, p, tmp_path / "r", mode, ring, timeout)
    assert rc == 1 and not h.value


def test_null_and_empty_paths(lib, tmp_path):
    assert lib.hbfsim_context_create(None, None) == 1
    rc, _ = _create(lib, None, tmp_path)
    assert rc == 1
    rc, _ = _create(lib, "", tmp_path)
    assert rc == 1


@pytest.mark.parametrize("field,value", [("page_bytes", 3000), ("page_bytes", 256),
                                         ("read_latency_ns", 0), ("channels", 0),
                                         ("capacity_bytes", 12345),
                                         ("reference_sample_rate", 1.5),
                                         ("plane_allocation_scheme", "XYZW"),
                                         ("hbm_cache_bytes", 1 << 40)])
def test_profile_validation(lib, tmp_path, field, value):
    p = workloads.c0_profile()
    p[field] = value
    path = tmp_path / "bad.json"
    path.write_text(json.dumps(p))
    rc, _ = _create(lib, path, tmp_path / "r")
    assert rc == 1


def test_missing_field_and_bad_json(lib, tmp_path):
    p = workloads.c0_profile()
    del p["queue_depth"]
    (tmp_path / "a.json").write_text(json.dumps(p))
    assert _create(lib, tmp_path / "a.json", tmp_path / "r")[0] == 1
    (tmp_path / "b.json").write_text("{\"name\": ")
    assert _create(lib, tmp_path / "b.json", tmp_path / "r")[0] == 1
    assert _create(lib, tmp_path / "missing.json", tmp_path / "r")[0] == 1


def test_reference_profiles_parse(lib, tmp_path):
    """The shipped reference profile shape (nominal) is accepted up to the
    CUDA step: on a CPU-only host creation stops at HBFSIM_CUDA_ERROR."""
    nominal = {"name": "nominal", "capacity_bytes": 1099511627776, "page_bytes": 16384,
               "read_latency_ns": 10000, "program_latency_ns": 100000, "channels": 32,
               "dies_per_channel": 8, "planes_per_die": 4, "pages_per_block": 256,
               "channel_width_bits": 8, "channel_transfer_rate_mtps": 1600,
               "queue_depth": 128, "aggregate_bandwidth_bytes_per_s": 512000000000,
               "hbm_cache_bytes": 8589934592, "reference_sample_rate": 0.01,
               "reference_warmup_requests": 1024, "time_scale": 100,
               "timing_tolerance_ns": 10000}
    path = tmp_path / "nominal.json"
    path.write_text(json.dumps(nominal))
    import torch
    rc, h = _create(lib, path, tmp_path / "r", mode=1)
    if torch.cuda.is_available():
        assert rc == 0
        lib.hbfsim_context_destroy(h)
    else:
        assert rc == 3


def test_null_context_calls(lib):
    assert lib.hbfsim_flush(None) == 1
    assert lib.hbfsim_get_stats(None, None) == 1
    assert lib.hbfsim_unregister(None, None) == 1
    assert lib.hbfsim_register_device(None, None, 0, None) == 1
    out = ctypes.c_void_p(1)
    assert lib.hbfsim_map_file(None, b"x", 0, 1, None, ctypes.byref(out)) == 1
    assert out.value is None
    lib.hbfsim_context_destroy(None)


def test_stateless_entry_argument_checks(lib):
    """The prefetch-sweep and link-batch entries refuse bad arguments before
    any device work (no GPU needed)."""
    pf_cells = (_lib.PrefetchCellV1 * 2)()
    pf_cells[0] = _lib.PrefetchCellV1(2, 1, 0.5, 64, 32, 1000, 0, 1)
    pf_cells[1] = _lib.PrefetchCellV1(7, 1, 0.5, 64, 32, 1000, 0, 1)  # policy 7
    out = (_lib.PrefetchStatsV1 * 2)()
    assert lib.hbfsim_prefetch_sweep_v1(None, 10, pf_cells, 2, out, None) == 1  # no pages
    assert lib.hbfsim_prefetch_sweep_v1(ctypes.c_void_p(8), 10, pf_cells, 2, out, None) == 1
    assert lib.hbfsim_prefetch_sweep_v1(ctypes.c_void_p(8), 1 << 33, pf_cells, 1, out,
                                        None) == 5  # 2^33 accesses: HBFSIM_UNSUPPORTED
    assert lib.hbfsim_prefetch_sweep_v1(None, 0, pf_cells, 0, out, None) == 0
    # zero accesses: every statistic 0, no device work
    assert lib.hbfsim_prefetch_sweep_v1(None, 0, pf_cells, 1, out, None) == 0
    assert out[0].total_ns == 0 and out[0].demand_accesses == 0

    def link(gt=16, ar=12, r=56, accepted=4, prop=0):
        return _lib.LinkProfileV1(gt, ar, r, accepted, prop, (ctypes.c_uint64 * 2)(0, 0))

    offsets = (ctypes.c_uint64 * 2)(0, 0)
    res = (_lib.LinkResultV1 * 1)()
    for bad in (link(gt=64), link(ar=2), link(r=13), link(accepted=0), link(ar=70000),
                link(prop=2_000_000_000)):
        profiles = (_lib.LinkProfileV1 * 1)(bad)
        assert lib.hbfsim_link_batch_v1(profiles, 1, offsets, None, None, None, res, None) == 1
    assert lib.hbfsim_link_batch_v1(None, 0, None, None, None, None, None, None) == 0
    offsets_bad = (ctypes.c_uint64 * 2)(0, 5)  # messages but no device arrays
    profiles = (_lib.LinkProfileV1 * 1)(link())
    assert lib.hbfsim_link_batch_v1(profiles, 1, offsets_bad, None, None, None, res, None) == 1


def test_ledger_entries_without_a_ledger(lib):
    assert lib.hbfsim_retention_blocks_v1(None) == 0
    assert lib.hbfsim_retention_advance_v1(None, 0, None, None) == 1
    count = ctypes.c_uint64()
    assert lib.hbfsim_retention_due_v1(None, 0, None, None, 0, ctypes.byref(count), None) == 1
    assert lib.hbfsim_retention_refresh_v1(None, None, 0, None) == 1
    assert lib.hbfsim_get_retention_v1(None, None, None, None, None, 0, None) == 1
    cfg = _lib.RetentionConfigV1(ctypes.sizeof(_lib.RetentionConfigV1), 1, 1.05, 358.15,
                                 86_400_000_000_000, 0, 0, 0, 330.0, 0, 0)
    assert lib.hbfsim_retention_configure_v1(None, ctypes.byref(cfg)) == 1
