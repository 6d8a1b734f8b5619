"""ctypes binding of libhbfsim_b200.so (include/hbfsim/api.h + batch_v1.h).

The struct definitions below mirror the C headers field for field.  Loading
fails loudly when the library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libhbfsim_b200.so"

u8, u32, u64, dbl = ctypes.c_uint8, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_double
vp, cp, i32 = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int

HBFSIM_OK = 0
ERROR_NAMES = {0: "HBFSIM_OK", 1: "HBFSIM_INVALID_ARGUMENT", 2: "HBFSIM_IO_ERROR",
               3: "HBFSIM_CUDA_ERROR", 4: "HBFSIM_TIMEOUT", 5: "HBFSIM_UNSUPPORTED",
               6: "HBFSIM_DAEMON_LOST"}
MODEL_REFERENCE, MODEL_FAST, MODEL_HYBRID, MODEL_DIE = 0, 1, 2, 3
RANGE_TIMING, RANGE_CAPACITY = 1, 2
READ, WRITE, READ_WRITE = 1, 2, 3
ACCESS_MODELED, ACCESS_UNSUPPORTED, ACCESS_BYPASS, ACCESS_FOREIGN = 1, 6, 8, 9
THERMAL_MAX_LAYERS = 32


class Options(ctypes.Structure):
    _fields_ = [("profile_path", cp), ("report_dir", cp), ("mode", u32),
                ("ring_capacity", u32), ("request_timeout_ns", u64)]


class RangeOptions(ctypes.Structure):
    _fields_ = [("mode", u32), ("permissions", u32), ("cache_policy", u32),
                ("stream_id", u32)]


class Stats(ctypes.Structure):
    _fields_ = [("requests_submitted", u64), ("requests_completed", u64),
                ("fast_requests", u64), ("reference_requests", u64),
                ("fast_modeled_ns", u64)]


class CapacityStatsV1(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("version", u32), ("enabled", u32),
                ("reserved0", u32)] + [(name, u64) for name in (
                    "page_bytes", "vmm_granularity", "pool_allocated_bytes",
                    "logical_frame_count", "service_resolve_calls",
                    "service_resident_hits", "service_reclaimed_hits",
                    "service_misses", "successful_backing_read_pages",
                    "successful_backing_read_bytes", "successful_h2d_fill_pages",
                    "successful_h2d_fill_bytes", "successful_resolve_evictions",
                    "service_ready_results", "successful_d2h_readback_pages",
                    "successful_d2h_readback_bytes", "successful_backing_write_pages",
                    "successful_backing_write_bytes")]


class GeometryV1(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("version", u32), ("stacks", u32),
                ("stripe_bytes", u32), ("shard_rank", u32), ("shard_count", u32),
                ("reserved", u32 * 2)]


class AccessBatchV1(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("version", u32), ("count", u64),
                ("address", vp), ("bytes", vp), ("operation", vp),
                ("arrival_ns", vp), ("done_ns", vp), ("latency_ns", vp),
                ("status", vp)]


class BatchStatsV1(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("version", u32)] + [(n, u64) for n in (
        "modeled", "bypass", "unsupported", "foreign", "latency_sum_ns",
        "max_done_ns", "fast_modeled_ns", "batches", "device_errors")]


class KernelTimesV1(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("version", u32), ("launches", u64 * 8),
                ("total_ms", dbl * 8)]


KERNEL_SLOTS = ("pass1", "scan", "pass2", "sequential", "decode", "thermal",
                "controller", "other")


class DecodedV1(ctypes.Structure):
    _fields_ = [("media_address", u64), ("page", u64), ("status", u32),
                ("range_index", u32), ("stack", u32), ("channel", u32),
                ("die", u32), ("plane", u32)]


class CapacityBatchV1(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("version", u32), ("count", u64),
                ("address", vp), ("bytes", vp), ("operation", vp), ("arrival_ns", vp),
                ("hit", vp), ("victim_page", vp), ("victim_dirty", vp), ("status", vp),
                ("done_ns", vp), ("latency_ns", vp)]


class ThermalLayerV1(ctypes.Structure):
    _fields_ = [("thickness_m", dbl), ("cv_j_m3_k", dbl), ("k_xyz_w_m_k", dbl * 3)]


class ThermalConfigV1(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("version", u32), ("nx", u32), ("ny", u32),
                ("layer_count", u32), ("reserved0", u32), ("cell_m", dbl),
                ("layers", ThermalLayerV1 * THERMAL_MAX_LAYERS),
                ("bottom_h_w_m2_k", dbl), ("bottom_ambient_k", dbl),
                ("top_h_w_m2_k", dbl), ("top_ambient_k", dbl), ("initial_k", dbl),
                ("die_idle_w", dbl), ("read_j_per_byte", dbl),
                ("write_j_per_access", dbl), ("refresh_onset_k", dbl),
                ("refresh_step_k", dbl), ("refresh_base_permille", u32),
                ("refresh_cap_permille", u32), ("light_k", dbl), ("severe_k", dbl),
                ("shutdown_k", dbl), ("hysteresis_k", dbl), ("light_permille", u32),
                ("severe_permille", u32), ("reserved1", u32 * 2),
                ("die_z0", vp), ("die_z_count", vp), ("die_x0", vp),
                ("die_x1", vp), ("die_y0", vp), ("die_y1", vp)]


class RetentionConfigV1(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("version", u32), ("ea_ev", dbl), ("tref_k", dbl),
                ("period_ns", u64), ("initial_age_ns", u64), ("initial_wall_age_ns", u64),
                ("epoch_ns", u64), ("initial_temperature_k", dbl),
                ("refresh_trigger", u32), ("reserved", u32)]


class PrefetchCellV1(ctypes.Structure):
    _fields_ = [("policy", u32), ("lead_distance", u32), ("accuracy", dbl),
                ("buffer_pages", u32), ("max_in_flight", u32), ("read_latency_ns", u64),
                ("compute_ns_per_access", u64), ("seed", u64)]


class PrefetchStatsV1(ctypes.Structure):
    _fields_ = [("total_ns", u64), ("stall_ns", u64), ("demand_accesses", u64),
                ("demand_misses", u64), ("prefetch_hits", u64), ("prefetch_issued", u64),
                ("prefetch_wasted", u64)]


class LinkProfileV1(ctypes.Structure):
    _fields_ = [("gt_per_second", u32), ("initial_ar_granules", u32),
                ("initial_r_granules", u32), ("max_accepted", u32), ("propagation_ns", u64),
                ("consume_ns", u64 * 2)]


class LinkResultV1(ctypes.Structure):
    _fields_ = [("counters", (u64 * 8) * 2), ("now", u64), ("ar_credits", u32),
                ("r_credits", u32), ("status", i32), ("reserved", u32)]


# Every exported function with its signature (restype, argtypes).
SIGNATURES = {
    "hbfsim_abi_version": (u32, []),
    "hbfsim_context_create": (i32, [ctypes.POINTER(Options), ctypes.POINTER(vp)]),
    "hbfsim_register_device": (i32, [vp, vp, ctypes.c_size_t, ctypes.POINTER(RangeOptions)]),
    "hbfsim_map_file": (i32, [vp, cp, u64, ctypes.c_size_t, ctypes.POINTER(RangeOptions),
                              ctypes.POINTER(vp)]),
    "hbfsim_flush": (i32, [vp]),
    "hbfsim_get_stats": (i32, [vp, ctypes.POINTER(Stats)]),
    "hbfsim_get_capacity_stats_v1": (i32, [vp, ctypes.POINTER(CapacityStatsV1)]),
    "hbfsim_unregister": (i32, [vp, vp]),
    "hbfsim_context_destroy": (None, [vp]),
    "hbfsim_set_geometry_v1": (i32, [vp, ctypes.POINTER(GeometryV1)]),
    "hbfsim_submit_access_batch_v1": (i32, [vp, ctypes.POINTER(AccessBatchV1), vp]),
    "hbfsim_submit_access_batch_host_v1": (i32, [vp, ctypes.POINTER(AccessBatchV1)]),
    "hbfsim_submit_access_batch_static_v1": (i32, [vp, ctypes.POINTER(AccessBatchV1), vp]),
    "hbfsim_get_simulated_time_v1": (i32, [vp, ctypes.POINTER(u64)]),
    "hbfsim_reset_state_v1": (i32, [vp, vp]),
    "hbfsim_set_profiling_v1": (i32, [vp, i32]),
    "hbfsim_get_kernel_times_v1": (i32, [vp, ctypes.POINTER(KernelTimesV1)]),
    "hbfsim_get_batch_stats_v1": (i32, [vp, ctypes.POINTER(BatchStatsV1)]),
    "hbfsim_decode_batch_v1": (i32, [vp, vp, vp, vp, u64, vp, vp]),
    "hbfsim_sample_batch_v1": (i32, [vp, vp, vp, vp, u64, vp, vp]),
    "hbfsim_capacity_configure_v1": (i32, [vp, u64, u32]),
    "hbfsim_capacity_policy_v1": (i32, [vp, u32]),
    "hbfsim_get_capacity_rounds_v1": (i32, [vp, vp, vp, vp]),
    "hbfsim_submit_capacity_batch_v1": (i32, [vp, ctypes.POINTER(CapacityBatchV1), vp]),
    "hbfsim_get_capacity_state_v1": (i32, [vp, vp, vp, u64, ctypes.POINTER(u64)]),
    "hbfsim_set_channel_factors_v1": (i32, [vp, vp, vp, vp]),
    "hbfsim_get_channel_factors_v1": (i32, [vp, vp, vp, vp]),
    "hbfsim_get_state_v1": (i32, [vp, vp, u64]),
    "hbfsim_set_state_v1": (i32, [vp, vp, u64]),
    "hbfsim_state_words_v1": (u64, [vp]),
    "hbfsim_get_die_activity_v1": (i32, [vp, vp, vp, u64]),
    "hbfsim_thermal_configure_v1": (i32, [vp, ctypes.POINTER(ThermalConfigV1)]),
    "hbfsim_advance_epoch_v1": (i32, [vp, dbl, vp]),
    "hbfsim_get_temperatures_v1": (i32, [vp, vp, u64]),
    "hbfsim_get_die_temperatures_v1": (i32, [vp, vp, u64]),
    "hbfsim_advance_epoch_global_v1": (i32, [vp, dbl, vp, vp, vp]),
    "hbfsim_copy_die_activity_v1": (i32, [vp, vp, vp, vp]),
    "hbfsim_get_thermal_factors_v1": (i32, [vp, vp, vp, vp, vp]),
    "hbfsim_retention_configure_v1": (i32, [vp, ctypes.POINTER(RetentionConfigV1)]),
    "hbfsim_retention_blocks_v1": (u64, [vp]),
    "hbfsim_retention_advance_v1": (i32, [vp, u64, vp, vp]),
    "hbfsim_retention_due_v1": (i32, [vp, u64, vp, vp, u64, ctypes.POINTER(u64), vp]),
    "hbfsim_retention_refresh_v1": (i32, [vp, vp, u64, vp]),
    "hbfsim_retention_record_erase_v1": (i32, [vp, vp, u64, vp]),
    "hbfsim_retention_record_programs_v1": (i32, [vp, vp, vp, vp, u64, vp]),
    "hbfsim_get_retention_v1": (i32, [vp, vp, vp, vp, vp, u64, ctypes.POINTER(u64)]),
    "hbfsim_prefetch_sweep_v1": (i32, [vp, u64, vp, u32, vp, vp]),
    "hbfsim_link_batch_v1": (i32, [vp, u32, vp, vp, vp, vp, vp, vp]),  # arrays by address
}


class HbfsimError(RuntimeError):
    """A non-zero hbfsim_error code from the C ABI."""

    def __init__(self, code: int, call: str):
        self.code = code
        super().__init__(f"{call} failed: {ERROR_NAMES.get(code, code)}")


_LIB: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the CUDA library; raise ImportError if it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m hbfsim_b200.build` "
            "(nvcc, sm_100a); there is no CPU fallback")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def check(code: int, call: str) -> None:
    if code != HBFSIM_OK:
        raise HbfsimError(code, call)
