"""Python host side of the B200 access-timing path.

`Context` mirrors the reference C API (include/hbfsim/api.h:92-107) call for
call -- context_create, register_device, flush, get_stats, unregister,
context_destroy -- and adds the batch exports of include/hbfsim/batch_v1.h.
Errors raise HbfsimError carrying the hbfsim_error code, the way the
reference vLLM loader turns a non-zero status into an exception
(adapters/vllm/hbfsim_loader.py:287-380).  torch is used only to hand device
buffers and streams to the library.
"""
from __future__ import annotations

import ctypes
import tempfile
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import HbfsimError, check

__all__ = ["Context", "HbfsimError", "BatchResult", "prefetch_sweep", "PREFETCH_POLICIES",
           "link_batch", "link_profiles", "LINK_PROFILE_DTYPE", "LINK_RESULT_DTYPE"]

PREFETCH_POLICIES = {"none": 0, "next_page": 1, "accuracy": 2}


@dataclass
class BatchResult:
    done_ns: object
    latency_ns: object
    status: object


CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy: the legacy default stream


def _stream_handle(stream) -> int:
    """cudaStream_t for the C ABI.  torch reports the legacy default stream
    as 0, which the C ABI reads as "the context's own stream", so map it to
    cudaStreamLegacy to keep the caller's stream ordering."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream or CUDA_STREAM_LEGACY


def _ptr(t) -> int:
    if t is None:
        return 0
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return t.data_ptr()


class Context:
    """One hbfsim context bound to the current CUDA device."""

    def __init__(self, profile_path: str, report_dir: str | None = None,
                 mode: int = _lib.MODEL_DIE, ring_capacity: int = 64,
                 request_timeout_ns: int = 1_000_000_000):
        self._lib = _lib.load()
        self._tmp = None
        if report_dir is None:
            self._tmp = tempfile.TemporaryDirectory(prefix="hbfsim-report-")
            report_dir = self._tmp.name
        opts = _lib.Options(str(profile_path).encode(), str(report_dir).encode(),
                            mode, ring_capacity, request_timeout_ns)
        handle = ctypes.c_void_p()
        check(self._lib.hbfsim_context_create(ctypes.byref(opts), ctypes.byref(handle)),
              "hbfsim_context_create")
        self.handle = handle
        self.mode = mode

    # ---- reference API -------------------------------------------------
    def register_device(self, base: int, length: int, mode: int = _lib.RANGE_TIMING,
                        permissions: int = _lib.READ_WRITE, cache_policy: int = 0,
                        stream_id: int = 0) -> None:
        o = _lib.RangeOptions(mode, permissions, cache_policy, stream_id)
        check(self._lib.hbfsim_register_device(self.handle, ctypes.c_void_p(base),
                                               length, ctypes.byref(o)),
              "hbfsim_register_device")

    def unregister(self, base: int) -> None:
        check(self._lib.hbfsim_unregister(self.handle, ctypes.c_void_p(base)),
              "hbfsim_unregister")

    def flush(self) -> None:
        check(self._lib.hbfsim_flush(self.handle), "hbfsim_flush")

    def get_stats(self) -> dict:
        s = _lib.Stats()
        check(self._lib.hbfsim_get_stats(self.handle, ctypes.byref(s)), "hbfsim_get_stats")
        return {f: getattr(s, f) for f, _ in _lib.Stats._fields_}

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.hbfsim_context_destroy(self.handle)
            self.handle = None
        if self._tmp is not None:
            self._tmp.cleanup()
            self._tmp = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- batch_v1 -------------------------------------------------------
    def set_geometry(self, stacks: int = 1, stripe_bytes: int = 0, shard_rank: int = 0,
                     shard_count: int = 1) -> None:
        g = _lib.GeometryV1(ctypes.sizeof(_lib.GeometryV1), 1, stacks, stripe_bytes,
                            shard_rank, shard_count)
        check(self._lib.hbfsim_set_geometry_v1(self.handle, ctypes.byref(g)),
              "hbfsim_set_geometry_v1")

    @staticmethod
    def _batch(count, address, nbytes, op, arrival, done, latency, status):
        return _lib.AccessBatchV1(ctypes.sizeof(_lib.AccessBatchV1), 1, count,
                                  _ptr(address), _ptr(nbytes), _ptr(op), _ptr(arrival),
                                  _ptr(done), _ptr(latency), _ptr(status))

    def submit(self, address, nbytes, op, arrival, out: BatchResult | None = None,
               stream=None) -> BatchResult:
        """Time a batch held in device tensors (uint64/int64 address and
        arrival, int32 bytes, uint8 op).  Asynchronous on `stream`."""
        import torch
        n = address.numel()
        if out is None:
            dev = address.device
            out = BatchResult(torch.empty(n, dtype=torch.int64, device=dev),
                              torch.empty(n, dtype=torch.int64, device=dev),
                              torch.empty(n, dtype=torch.uint8, device=dev))
        b = self._batch(n, address, nbytes, op, arrival, out.done_ns, out.latency_ns,
                        out.status)
        s = _stream_handle(stream)
        check(self._lib.hbfsim_submit_access_batch_v1(self.handle, ctypes.byref(b),
                                                      ctypes.c_void_p(s)),
              "hbfsim_submit_access_batch_v1")
        return out

    def submit_host(self, address, nbytes, op, arrival, out: BatchResult | None = None
                    ) -> BatchResult:
        """Time a batch held in host memory (numpy arrays or pinned CPU
        tensors); copies are pipelined inside the library.  Synchronous."""
        n = int(address.shape[0])
        if out is None:
            out = BatchResult(np.empty(n, np.uint64), np.empty(n, np.uint64),
                              np.empty(n, np.uint8))
        b = self._batch(n, address, nbytes, op, arrival, out.done_ns, out.latency_ns,
                        out.status)
        check(self._lib.hbfsim_submit_access_batch_host_v1(self.handle, ctypes.byref(b)),
              "hbfsim_submit_access_batch_host_v1")
        return out

    def reset_state(self, stream=None) -> None:
        """Idle every die and channel at tick 0 (asynchronous on `stream`)."""
        import torch
        s = _stream_handle(stream)
        check(self._lib.hbfsim_reset_state_v1(self.handle, ctypes.c_void_p(s)),
              "hbfsim_reset_state_v1")

    def set_profiling(self, enable: bool) -> None:
        check(self._lib.hbfsim_set_profiling_v1(self.handle, 1 if enable else 0),
              "hbfsim_set_profiling_v1")

    def kernel_times(self) -> dict:
        """{slot: (launches, total_ms)} since the last call; synchronizes."""
        k = _lib.KernelTimesV1(ctypes.sizeof(_lib.KernelTimesV1), 1)
        check(self._lib.hbfsim_get_kernel_times_v1(self.handle, ctypes.byref(k)),
              "hbfsim_get_kernel_times_v1")
        return {name: (k.launches[i], k.total_ms[i]) for i, name in enumerate(_lib.KERNEL_SLOTS)}

    def simulated_time(self) -> int:
        v = ctypes.c_uint64()
        check(self._lib.hbfsim_get_simulated_time_v1(self.handle, ctypes.byref(v)),
              "hbfsim_get_simulated_time_v1")
        return v.value

    def batch_stats(self) -> dict:
        s = _lib.BatchStatsV1(ctypes.sizeof(_lib.BatchStatsV1), 1)
        check(self._lib.hbfsim_get_batch_stats_v1(self.handle, ctypes.byref(s)),
              "hbfsim_get_batch_stats_v1")
        return {f: getattr(s, f) for f, _ in _lib.BatchStatsV1._fields_[2:]}

    def decode(self, address, nbytes, op, stream=None):
        """Range lookup + stripe decode of device tensors; returns a uint8
        device tensor viewed as hbfsim_decoded_v1 records (40 bytes each)."""
        import torch
        n = address.numel()
        out = torch.empty(n * ctypes.sizeof(_lib.DecodedV1), dtype=torch.uint8,
                          device=address.device)
        s = _stream_handle(stream)
        check(self._lib.hbfsim_decode_batch_v1(self.handle, _ptr(address), _ptr(nbytes),
                                               _ptr(op), n, _ptr(out), ctypes.c_void_p(s)),
              "hbfsim_decode_batch_v1")
        return out

    # ---- Capacity mode ----
    def capacity_configure(self, frames: int, page_bytes: int = 4096,
                           policy: str = "lru") -> None:
        """Capacity mode over `frames` HBM frames of `page_bytes` pages.
        policy "lru": exact LRU (the offline LruCache); "clock": the
        reference runtime's second-chance CLOCK (HbmCache)."""
        check(self._lib.hbfsim_capacity_configure_v1(self.handle, frames, page_bytes),
              "hbfsim_capacity_configure_v1")
        codes = {"lru": 0, "clock": 1}
        if policy not in codes:
            raise ValueError(f"unknown capacity policy {policy!r}")
        if codes[policy]:
            check(self._lib.hbfsim_capacity_policy_v1(self.handle, codes[policy]),
                  "hbfsim_capacity_policy_v1")

    def submit_capacity(self, address, nbytes, op, arrival=None, stream=None, timed=False):
        """Replacement decisions (the configured policy) for device tensors: (hit u8, victim page
        int64 (-1 = none), victim dirty u8, status u8) device tensors; with
        timed=True also (done, latency) int64 tensors of the media actions."""
        import torch
        n = address.numel()
        dev = address.device
        hit = torch.empty(n, dtype=torch.uint8, device=dev)
        victim = torch.empty(n, dtype=torch.int64, device=dev)
        dirty = torch.empty(n, dtype=torch.uint8, device=dev)
        status = torch.empty(n, dtype=torch.uint8, device=dev)
        done = torch.empty(n, dtype=torch.int64, device=dev) if timed else None
        latency = torch.empty(n, dtype=torch.int64, device=dev) if timed else None
        b = _lib.CapacityBatchV1(ctypes.sizeof(_lib.CapacityBatchV1), 1, n, _ptr(address),
                                 _ptr(nbytes), _ptr(op), _ptr(arrival), _ptr(hit),
                                 _ptr(victim), _ptr(dirty), _ptr(status), _ptr(done),
                                 _ptr(latency))
        check(self._lib.hbfsim_submit_capacity_batch_v1(
            self.handle, ctypes.byref(b), ctypes.c_void_p(_stream_handle(stream))),
            "hbfsim_submit_capacity_batch_v1")
        if timed:
            return hit, victim, dirty, status, done, latency
        return hit, victim, dirty, status

    def capacity_rounds(self):
        """(fixed-point rounds, pieces, walked) of the last timed capacity
        batch."""
        r, p, w = ctypes.c_uint32(), ctypes.c_uint64(), ctypes.c_uint32()
        check(self._lib.hbfsim_get_capacity_rounds_v1(self.handle, ctypes.byref(r),
                                                      ctypes.byref(p), ctypes.byref(w)),
              "hbfsim_get_capacity_rounds_v1")
        return r.value, p.value, w.value

    def capacity_stats(self) -> dict:
        """hbfsim_get_capacity_stats_v1 as a dict (the reference's counter
        names)."""
        st = _lib.CapacityStatsV1()
        st.struct_size = ctypes.sizeof(st)
        st.version = 1
        check(self._lib.hbfsim_get_capacity_stats_v1(self.handle, ctypes.byref(st)),
              "hbfsim_get_capacity_stats_v1")
        return {f: getattr(st, f) for f, _ in _lib.CapacityStatsV1._fields_}

    def capacity_state(self):
        """(resident pages, their dirty bits) as numpy arrays: oldest first
        under LRU, in frame order under CLOCK."""
        count = ctypes.c_uint64()
        check(self._lib.hbfsim_get_capacity_state_v1(self.handle, None, None, 0,
                                                     ctypes.byref(count)),
              "hbfsim_get_capacity_state_v1")
        pages = np.zeros(count.value, np.uint64)
        dirty = np.zeros(count.value, np.uint8)
        check(self._lib.hbfsim_get_capacity_state_v1(self.handle, _ptr(pages), _ptr(dirty),
                                                     count.value, ctypes.byref(count)),
              "hbfsim_get_capacity_state_v1")
        return pages, dirty

    def sample(self, address, nbytes, op, stream=None):
        """Hybrid sampler bits of device tensors (uint8 device tensor; 1 =
        the hybrid model would send the access to the reference model)."""
        import torch
        out = torch.empty(address.numel(), dtype=torch.uint8, device=address.device)
        check(self._lib.hbfsim_sample_batch_v1(self.handle, _ptr(address), _ptr(nbytes), _ptr(op),
                                               address.numel(), _ptr(out),
                                               ctypes.c_void_p(_stream_handle(stream))),
              "hbfsim_sample_batch_v1")
        return out

    def set_channel_factors(self, refresh_permille=None, throttle_permille=None,
                            admit_after_ns=None) -> None:
        r = None if refresh_permille is None else np.ascontiguousarray(refresh_permille, np.uint32)
        t = None if throttle_permille is None else np.ascontiguousarray(throttle_permille, np.uint32)
        a = None if admit_after_ns is None else np.ascontiguousarray(admit_after_ns, np.uint64)
        check(self._lib.hbfsim_set_channel_factors_v1(self.handle, _ptr(r), _ptr(t), _ptr(a)),
              "hbfsim_set_channel_factors_v1")

    def channel_factors(self, channels: int, stacks: int):
        r = np.zeros(channels, np.uint32)
        t = np.zeros(stacks, np.uint32)
        a = np.zeros(stacks, np.uint64)
        check(self._lib.hbfsim_get_channel_factors_v1(self.handle, _ptr(r), _ptr(t), _ptr(a)),
              "hbfsim_get_channel_factors_v1")
        return r, t, a

    def state_words(self) -> int:
        return int(self._lib.hbfsim_state_words_v1(self.handle))

    def get_state(self) -> np.ndarray:
        w = np.zeros(self.state_words(), np.uint64)
        check(self._lib.hbfsim_get_state_v1(self.handle, _ptr(w), w.size), "hbfsim_get_state_v1")
        return w

    def set_state(self, words: np.ndarray) -> None:
        w = np.ascontiguousarray(words, np.uint64)
        check(self._lib.hbfsim_set_state_v1(self.handle, _ptr(w), w.size), "hbfsim_set_state_v1")

    def die_activity(self, dies_total: int):
        rb = np.zeros(dies_total, np.uint64)
        wr = np.zeros(dies_total, np.uint64)
        check(self._lib.hbfsim_get_die_activity_v1(self.handle, _ptr(rb), _ptr(wr), dies_total),
              "hbfsim_get_die_activity_v1")
        return rb, wr

    # ---- eq3 thermal grid and epoch controller ----
    def thermal_configure(self, stack: dict, floorplan: dict, power: dict,
                          refresh: dict, throttle: dict) -> None:
        """Configures the layered thermal grid and the epoch controller.

        stack: {"nx", "ny", "cell_m", "layers": [{"thickness_m", "cv_j_m3_k",
        "k_xyz_w_m_k"}], "bottom": {"h_w_m2_k", "ambient_k"}, "top": {...},
        "initial_k"} (the layered-export description).
        floorplan: arrays z0, z_count, x0, x1, y0, y1 indexed g*D+d.
        power: {"idle_w", "read_j_per_byte", "write_j_per_access"}.
        refresh: {"onset_k", "step_k", "base_permille", "cap_permille"}.
        throttle: {"light_k", "severe_k", "shutdown_k", "hysteresis_k",
        "light_permille", "severe_permille"}."""
        c = _lib.ThermalConfigV1()
        c.struct_size = ctypes.sizeof(_lib.ThermalConfigV1)
        c.version = 1
        c.nx, c.ny = stack["nx"], stack["ny"]
        c.layer_count = len(stack["layers"])
        c.cell_m = stack["cell_m"]
        for i, layer in enumerate(stack["layers"]):
            c.layers[i].thickness_m = layer["thickness_m"]
            c.layers[i].cv_j_m3_k = layer["cv_j_m3_k"]
            for a in range(3):
                c.layers[i].k_xyz_w_m_k[a] = layer["k_xyz_w_m_k"][a]
        c.bottom_h_w_m2_k = stack["bottom"]["h_w_m2_k"]
        c.bottom_ambient_k = stack["bottom"]["ambient_k"]
        c.top_h_w_m2_k = stack["top"]["h_w_m2_k"]
        c.top_ambient_k = stack["top"]["ambient_k"]
        c.initial_k = stack["initial_k"]
        c.die_idle_w = power["idle_w"]
        c.read_j_per_byte = power["read_j_per_byte"]
        c.write_j_per_access = power["write_j_per_access"]
        c.refresh_onset_k = refresh["onset_k"]
        c.refresh_step_k = refresh["step_k"]
        c.refresh_base_permille = refresh["base_permille"]
        c.refresh_cap_permille = refresh["cap_permille"]
        for key in ("light_k", "severe_k", "shutdown_k", "hysteresis_k",
                    "light_permille", "severe_permille"):
            setattr(c, key, throttle[key])
        keep = {}
        for key in ("z0", "z_count", "x0", "x1", "y0", "y1"):
            keep[key] = np.ascontiguousarray(floorplan[key], np.uint32)
            setattr(c, "die_" + key, keep[key].ctypes.data)
        check(self._lib.hbfsim_thermal_configure_v1(self.handle, ctypes.byref(c)),
              "hbfsim_thermal_configure_v1")

    def advance_epoch(self, epoch_s: float, stream=None) -> None:
        check(self._lib.hbfsim_advance_epoch_v1(self.handle, ctypes.c_double(epoch_s),
                                                ctypes.c_void_p(_stream_handle(stream))),
              "hbfsim_advance_epoch_v1")

    def advance_epoch_global(self, epoch_s: float, read_bytes, writes, stream=None) -> None:
        """Epoch step driven by the activity of every global die (device
        tensors of uint64 viewed as int64, index g*D+d)."""
        check(self._lib.hbfsim_advance_epoch_global_v1(
            self.handle, ctypes.c_double(epoch_s), _ptr(read_bytes), _ptr(writes),
            ctypes.c_void_p(_stream_handle(stream))), "hbfsim_advance_epoch_global_v1")

    def copy_die_activity(self, read_bytes, writes, stream=None) -> None:
        check(self._lib.hbfsim_copy_die_activity_v1(self.handle, _ptr(read_bytes), _ptr(writes),
                                                    ctypes.c_void_p(_stream_handle(stream))),
              "hbfsim_copy_die_activity_v1")

    def temperatures(self, cells: int) -> np.ndarray:
        out = np.zeros(cells, np.float64)
        check(self._lib.hbfsim_get_temperatures_v1(self.handle, _ptr(out), cells),
              "hbfsim_get_temperatures_v1")
        return out

    def die_temperatures(self, dies_total: int) -> np.ndarray:
        out = np.zeros(dies_total, np.float64)
        check(self._lib.hbfsim_get_die_temperatures_v1(self.handle, _ptr(out), dies_total),
              "hbfsim_get_die_temperatures_v1")
        return out

    def thermal_factors(self, channels: int, stacks: int):
        """(refresh per local channel, throttle, admit-after, level per stack)."""
        r = np.zeros(channels, np.uint32)
        t = np.zeros(stacks, np.uint32)
        a = np.zeros(stacks, np.uint64)
        lv = np.zeros(stacks, np.uint32)
        check(self._lib.hbfsim_get_thermal_factors_v1(self.handle, _ptr(r), _ptr(t), _ptr(a),
                                                      _ptr(lv)),
              "hbfsim_get_thermal_factors_v1")
        return r, t, a, lv

    # ---- per-block retention-age ledger ---------------------------------
    def retention_configure(self, ea_ev: float = 1.04, initial_temperature_k: float = 318.15,
                            initial_age_ns: int = 0, initial_wall_age_ns: int = 0,
                            epoch_ns: int = 0, refresh_trigger: str = "wall_only") -> int:
        """Ledger over every block of the local channels (reliability.py
        ReliabilityLedger); returns the block count."""
        cfg = _lib.RetentionConfigV1(ctypes.sizeof(_lib.RetentionConfigV1), 1, float(ea_ev),
                                     358.15, 86_400_000_000_000, int(initial_age_ns),
                                     int(initial_wall_age_ns), int(epoch_ns),
                                     float(initial_temperature_k),
                                     {"wall_only": 0, "equivalent_age_or_wall": 1}[refresh_trigger],
                                     0)
        check(self._lib.hbfsim_retention_configure_v1(self.handle, ctypes.byref(cfg)),
              "hbfsim_retention_configure_v1")
        return self.retention_blocks()

    def retention_blocks(self) -> int:
        return int(self._lib.hbfsim_retention_blocks_v1(self.handle))

    def retention_advance(self, end_ns: int, die_temp_k=None, stream=None) -> None:
        """Age every block to end_ns: at the given per-local-die temperatures
        (float64 device tensor), or at the midpoint of the thermal model's
        die temperatures (None)."""
        check(self._lib.hbfsim_retention_advance_v1(
            self.handle, int(end_ns), None if die_temp_k is None else _ptr(die_temp_k),
            ctypes.c_void_p(_stream_handle(stream))), "hbfsim_retention_advance_v1")

    def retention_due(self, at_ns: int, stream=None):
        """(block ids, reason bits) of the blocks due at at_ns, ascending."""
        import torch
        n = self.retention_blocks()
        blocks = torch.empty(max(1, n), dtype=torch.int32, device="cuda")
        reasons = torch.empty(max(1, n), dtype=torch.uint8, device="cuda")
        count = ctypes.c_uint64()
        check(self._lib.hbfsim_retention_due_v1(self.handle, int(at_ns), _ptr(blocks),
                                                _ptr(reasons), n, ctypes.byref(count),
                                                ctypes.c_void_p(_stream_handle(stream))),
              "hbfsim_retention_due_v1")
        k = int(count.value)
        return (blocks[:k].cpu().numpy().view(np.uint32), reasons[:k].cpu().numpy())

    def retention_refresh(self, blocks, stream=None) -> None:
        """Committed refresh of the listed blocks (int32 device tensor)."""
        check(self._lib.hbfsim_retention_refresh_v1(self.handle, _ptr(blocks), blocks.numel(),
                                                    ctypes.c_void_p(_stream_handle(stream))),
              "hbfsim_retention_refresh_v1")

    def retention_record_erase(self, blocks, stream=None) -> None:
        check(self._lib.hbfsim_retention_record_erase_v1(
            self.handle, _ptr(blocks), blocks.numel(), ctypes.c_void_p(_stream_handle(stream))),
            "hbfsim_retention_record_erase_v1")

    def retention_record_programs(self, address, nbytes, op, stream=None) -> None:
        check(self._lib.hbfsim_retention_record_programs_v1(
            self.handle, _ptr(address), _ptr(nbytes), _ptr(op), address.numel(),
            ctypes.c_void_p(_stream_handle(stream))), "hbfsim_retention_record_programs_v1")

    def retention_state(self) -> dict:
        """Host copies: age_ns, next_wall_due_ns, last_refresh_commit_ns,
        program_started, program_completed, erase_started, erase_completed,
        frontier_ns."""
        n = self.retention_blocks()
        age = np.zeros(n, np.float64)
        due = np.zeros(n, np.uint64)
        last = np.zeros(n, np.uint64)
        counts = np.zeros(4 * n, np.uint32)
        frontier = ctypes.c_uint64()
        check(self._lib.hbfsim_get_retention_v1(self.handle, _ptr(age), _ptr(due), _ptr(last),
                                                _ptr(counts), n, ctypes.byref(frontier)),
              "hbfsim_get_retention_v1")
        c = counts.reshape(4, n)
        return {"age_ns": age, "next_wall_due_ns": due, "last_refresh_commit_ns": last,
                "program_started": c[0], "program_completed": c[1], "erase_started": c[2],
                "erase_completed": c[3], "frontier_ns": int(frontier.value)}


def prefetch_sweep(pages, cells, stream=None) -> list[dict]:
    """The prefetch model (hbfsim::simulate_prefetch) for every cell on one
    page stream (uint64/int64 device tensor).  A cell is a dict with keys
    policy ("none" | "next_page" | "accuracy"), accuracy, lead_distance,
    buffer_pages, max_in_flight, read_latency_ns, compute_ns_per_access,
    seed (the reference's PrefetchConfig defaults fill missing keys).
    Returns one stats dict per cell."""
    lib = _lib.load()
    n = len(cells)
    arr = (_lib.PrefetchCellV1 * max(1, n))()
    for k, c in enumerate(cells):
        policy = c.get("policy", "none")
        arr[k] = _lib.PrefetchCellV1(PREFETCH_POLICIES.get(policy, policy),
                                     int(c.get("lead_distance", 1)),
                                     float(c.get("accuracy", 1.0)),
                                     int(c.get("buffer_pages", 64)),
                                     int(c.get("max_in_flight", 32)),
                                     int(c.get("read_latency_ns", 10_000)),
                                     int(c.get("compute_ns_per_access", 0)),
                                     int(c.get("seed", 1)))
    out = (_lib.PrefetchStatsV1 * max(1, n))()
    check(lib.hbfsim_prefetch_sweep_v1(_ptr(pages), pages.numel(), arr, n, out,
                                       ctypes.c_void_p(_stream_handle(stream))),
          "hbfsim_prefetch_sweep_v1")
    return [{f: getattr(out[k], f) for f, _ in _lib.PrefetchStatsV1._fields_} for k in range(n)]


LINK_PROFILE_DTYPE = np.dtype([("gt_per_second", "<u4"), ("initial_ar_granules", "<u4"),
                               ("initial_r_granules", "<u4"), ("max_accepted", "<u4"),
                               ("propagation_ns", "<u8"), ("consume_ns", "<u8", (2,))])
LINK_RESULT_DTYPE = np.dtype([("counters", "<u8", (2, 8)), ("now", "<u8"),
                              ("ar_credits", "<u4"), ("r_credits", "<u4"), ("status", "<i4"),
                              ("reserved", "<u4")])


def link_profiles(count: int, gt_per_second=16, initial_ar_granules=12, initial_r_granules=56,
                  max_accepted=4, propagation_ns=0, consume_ns=(0, 0)) -> np.ndarray:
    """A structured array of `count` link profiles (hbfsim_link_profile_v1),
    every field a scalar or a per-link array; the defaults are the
    reference LinkProfile's scenario values."""
    p = np.zeros(count, LINK_PROFILE_DTYPE)
    p["gt_per_second"] = gt_per_second
    p["initial_ar_granules"] = initial_ar_granules
    p["initial_r_granules"] = initial_r_granules
    p["max_accepted"] = max_accepted
    p["propagation_ns"] = propagation_ns
    p["consume_ns"] = np.asarray(consume_ns, np.uint64)
    return p


def link_batch(profiles: np.ndarray, offsets, direction, ready, stream=None):
    """UCIe streaming-link timing (hbfsim::ucie::StreamingLink) for a batch
    of links.  profiles: structured array of LINK_PROFILE_DTYPE (see
    link_profiles); offsets: links + 1 message offsets (host); direction
    (uint8, 0 AR / 1 R) and ready (int64 ticks, non-decreasing per link):
    device tensors.  Returns (delivered device tensor, structured array of
    LINK_RESULT_DTYPE, one row per link)."""
    import torch
    lib = _lib.load()
    profiles = np.ascontiguousarray(profiles, LINK_PROFILE_DTYPE)
    n = profiles.size
    off = np.ascontiguousarray(offsets, np.uint64)
    delivered = torch.empty(max(1, int(off[-1])), dtype=torch.int64, device=ready.device)
    res = np.zeros(max(1, n), LINK_RESULT_DTYPE)
    check(lib.hbfsim_link_batch_v1(profiles.ctypes.data, n, off.ctypes.data, _ptr(direction),
                                   _ptr(ready), _ptr(delivered), res.ctypes.data,
                                   ctypes.c_void_p(_stream_handle(stream))),
          "hbfsim_link_batch_v1")
    return delivered[:int(off[-1])], res[:n]


def link_messages(stack, arrival, done, modeled, stacks: int):
    """The UCIe messages of a timed batch (device tensors), per stack: for
    every modeled access an AR (request, direction 0) ready at its arrival
    and an R (response, direction 1) ready at its die completion, on the
    link of its stack, each link's messages in ready order (an AR before an
    R of the same tick, otherwise batch order).  Returns (offsets per link
    (host, links + 1), direction, ready, access index) in link order."""
    import torch
    idx = torch.nonzero(modeled).flatten()
    n = idx.numel()
    st = stack[idx]
    m_stack = torch.cat([st, st])
    m_ready = torch.cat([arrival[idx], done[idx]])
    m_dir = torch.cat([torch.zeros(n, dtype=torch.uint8, device=idx.device),
                       torch.ones(n, dtype=torch.uint8, device=idx.device)])
    m_idx = torch.cat([idx, idx])
    order = torch.sort(m_ready, stable=True).indices
    order = order[torch.sort(m_stack[order], stable=True).indices]
    counts = torch.bincount(m_stack, minlength=stacks).cpu().numpy()
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint64)
    return offsets, m_dir[order].contiguous(), m_ready[order].contiguous(), m_idx[order]


def submit_linked(ctx: "Context", address, nbytes, op, arrival, profiles: np.ndarray,
                  stacks: int, stream=None):
    """One batch through the per-die model and then each stack's UCIe
    streaming link (hbfsim::ucie::StreamingLink, src/ucie/link.cpp), composed
    per stack: the request of every modeled access crosses its stack's link
    as an AR message at the access's arrival, and the response as an R
    message once the die model has completed it; the access completes when
    its R message is delivered.  Accesses the die model does not time keep
    its outputs.  profiles: one link profile per stack (link_profiles).
    Returns (BatchResult with the linked completions, the die model's
    BatchResult, per-link LINK_RESULT_DTYPE rows, the AR delivery ticks per
    access (-1 when not modeled))."""
    import torch
    die = ctx.submit(address, nbytes, op, arrival, stream=stream)
    rec = ctx.decode(address, nbytes, op, stream)
    stack = rec.view(torch.int32).view(-1, 10)[:, 6].to(torch.int64)
    modeled = die.status == _lib.ACCESS_MODELED
    offsets, direction, ready, index = link_messages(stack, arrival, die.done_ns, modeled,
                                                     stacks)
    delivered, res = link_batch(profiles, offsets, direction, ready, stream)
    done = die.done_ns.clone()
    ar = torch.full_like(die.done_ns, -1)
    is_r = direction == 1
    done[index[is_r]] = delivered[is_r]
    ar[index[~is_r]] = delivered[~is_r]
    out = BatchResult(done, done - arrival, die.status)
    return out, die, res, ar
