"""The batch entry point that allocates nothing (hbfsim_submit_access_batch_static_v1).

It exists for callers that cannot call cudaMalloc while they run -- a server
that reserved nearly all device memory for its own pool up front, or code that
cannot afford the device-wide synchronization a first cudaMalloc may cause.
Its scratch lives in one fixed device array that the library defines, so this
test checks, through the C ABI, that two calls in a row give exactly what the
allocating entry point gives (integer ticks: bit-exact), including a shape
whose CTA grid must shrink to fit the array, a context whose tick bound sends
every batch down the exact sequential path, and the FAST model with an
empirical burst curve (whose batch error word also lives in the array).

Kept in a file of its own so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

from helpers import Setup, make_context, to_device
from hbfsim_b200 import _lib
from hbfsim_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def _submit(lib, ctx, fn_name, dev):
    import torch
    address, nbytes, op, arrival = dev
    n = address.numel()
    out = [torch.empty(n, dtype=torch.int64, device="cuda"),
           torch.empty(n, dtype=torch.int64, device="cuda"),
           torch.empty(n, dtype=torch.uint8, device="cuda")]
    batch = _lib.AccessBatchV1(ctypes.sizeof(_lib.AccessBatchV1), 1, n,
                               address.data_ptr(), nbytes.data_ptr(), op.data_ptr(),
                               arrival.data_ptr(), out[0].data_ptr(), out[1].data_ptr(),
                               out[2].data_ptr())
    stream = torch.cuda.current_stream().cuda_stream or 1  # 1 = cudaStreamLegacy
    rc = getattr(lib, fn_name)(ctx.handle, ctypes.byref(batch), ctypes.c_void_p(stream))
    assert rc == 0, f"{fn_name} returned {rc}"
    torch.cuda.synchronize()
    return [t.cpu().numpy() for t in out]


STATIC_BYTES = 8 << 20      # the array's size (csrc/context.cu kStaticScratchBytes)
STATIC_ERROR_BYTES = 256    # its padded error word
# then the range scan's counters and flags (2 + 16384 words, padded to 256 B)
STATIC_HEAD_BYTES = STATIC_ERROR_BYTES + (4 * (2 + 16384) + 255) // 256 * 256


def _compare(lib, setup, arrays, tmp_path):
    n = arrays[0].size
    split = n * 3 // 5
    calls = [tuple(a[:split] for a in arrays), tuple(a[split:] for a in arrays)]
    reference = make_context(setup, str(tmp_path / "alloc"))
    static = make_context(setup, str(tmp_path / "static"))
    for k, part in enumerate(calls):
        dev = to_device(part)
        want = _submit(lib, reference, "hbfsim_submit_access_batch_v1", dev)
        got = _submit(lib, static, "hbfsim_submit_access_batch_static_v1", dev)
        for w, g, name in zip(want, got, ("done", "latency", "status")):
            assert np.array_equal(w, g), f"call {k}: {name} differs"
        assert np.array_equal(reference.get_state(), static.get_state()), f"call {k}: state"
    reference.flush()
    static.flush()
    want, got = reference.batch_stats(), static.batch_stats()
    assert want["modeled"] == got["modeled"] and got["device_errors"] == 0
    reference.close()
    static.close()
    return got


@pytest.mark.parametrize("model,dies,stacks,n,time_scale",
                         [(3, 4, 1, 70001, 1), (1, 4, 1, 50000, 1), (3, 8, 4, 1600000, 1),
                          (3, 4, 1, 40000, 1 << 16)])
def test_static_entry_matches_allocating_entry(tmp_path, model, dies, stacks, n, time_scale):
    import torch
    lib = _lib.load()
    p = wl.c0_profile()
    p["dies_per_channel"] = dies
    p["time_scale"] = time_scale
    p["capacity_bytes"] = p["page_bytes"] * 16 * dies * 4 * 256 * 64
    setup = Setup(profile=p, model=model, stacks=stacks, stripe=4096)
    setup.ranges = [(wl.RANGE_BASE, p["capacity_bytes"] - (1 << 20), 1, 3)]
    arrays = wl.c0_trace(n, seed=77 + n, range_length=p["capacity_bytes"] - (1 << 20))
    if stacks == 4:
        # 64 local channels, K = 9 state words: one CTA needs
        # C*K*(K+1) + C*K words (and a share of the scan's group words), so
        # the array holds at most `fits` CTAs,
        # while the plan asks for 2 per SM (the piece kernel, C*(K+1) > 512)
        # once a call has that many tiles of at most 2048 accesses: the grid
        # of both calls must shrink
        C, K = 16 * stacks, dies + 1
        fits = (STATIC_BYTES - STATIC_HEAD_BYTES) // (8 * (C * K * (K + 1) + C * K))
        sms = torch.cuda.get_device_properties(0).multi_processor_count
        smaller_call = n - n * 3 // 5
        assert -(-smaller_call // 2048) >= 2 * sms > fits
    if time_scale > 1:
        # a 4 KiB transfer times the scale exceeds the 24-bit field of the
        # parallel path: the host sends each batch down the sequential path
        assert 512 * time_scale > 0xFFFFFF
    _compare(lib, setup, arrays, tmp_path)


def test_static_entry_empirical_burst_curve(tmp_path):
    """The FAST model with an empirical burst-curve profile keeps its scratch
    with the context but its batch error word in the array."""
    lib = _lib.load()
    setup = Setup(profile=wl.vmem_profile(), model=1)
    setup.ranges = [(wl.RANGE_BASE, 15 << 30, 1, 3)]
    arrays = wl.vmem_trace(90001, seed=5)
    got = _compare(lib, setup, arrays, tmp_path)
    assert got["modeled"] > 0
