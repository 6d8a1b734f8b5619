"""The seeded synthetic traces the bench and the parity tests run (CPU).

Their sizes are the ones the benchmark lines quote, and the config-4
generator (run here with torch on the CPU) interleaves its two streams,
spreads the arrivals and splits the trace among channel shards as its
docstring says.
"""
import numpy as np
import pytest
import torch

from hbfsim_b200 import workloads as wl


def test_c1_trace_size_and_bypass_share():
    bases, counts = wl.c1_segments(seed=0)
    assert int(counts.sum()) == 279_204_864
    hbm = bases < wl.RANGE_BASE            # attention weights, resident in HBM
    assert int(counts[hbm].sum()) == 6_291_456
    assert np.all(counts[hbm] == wl.ATTN_BYTES // wl.READ_BYTES)
    assert np.all(counts[~hbm] == wl.EXPERT_BYTES // wl.READ_BYTES)
    # the same seed gives the same trace
    b2, c2 = wl.c1_segments(seed=0)
    assert np.array_equal(bases, b2) and np.array_equal(counts, c2)


def test_c3_trace_epochs():
    (a, b, o, t), cuts = wl.c3_trace()
    assert len(cuts) == wl.C3_EPOCHS + 1 and cuts[0] == 0
    assert cuts[-1] == a.size == 50_502_640
    assert np.all(np.diff(t.astype(np.int64)) >= 0)
    for k in (0, 37, wl.C3_EPOCHS - 1):
        lo, hi = cuts[k], cuts[k + 1]
        assert t[lo] >= k * wl.C3_EPOCH_NS and t[hi - 1] < (k + 1) * wl.C3_EPOCH_NS


def _collect(trace, channel_of, keep, m):
    parts = list(trace.chunks(channel_of, keep, m=m))
    return [torch.cat([p[k] for p in parts]) for k in range(4)]


@pytest.mark.parametrize("n", [5 * 3001 + 4, 5 * 3001 + 2])
def test_c4_trace_interleave_arrivals_and_shards(n):
    trace = wl.C4Trace("cpu", seed=0, n=n)
    channel_of = lambda a: (a >> 12) % 256      # any function of the address
    a, b, o, t = _collect(trace, channel_of, lambda ch: torch.ones_like(ch, dtype=torch.bool),
                          m=777)
    assert a.numel() == n
    i = torch.arange(n, dtype=torch.int64)
    assert torch.equal(t, i * wl.C4_SPAN_NS // n)
    moe = i % 5 < 3
    assert int(moe.sum()) == trace.n_moe
    # MoE accesses: config-1 expert reads in segment order
    want_moe = wl.expand_segments(trace.moe_bases, trace.moe_counts)[0][:trace.n_moe]
    assert np.array_equal(a[moe].numpy().view(np.uint64), want_moe)
    assert torch.all(b[moe] == wl.READ_BYTES) and torch.all(o[moe] == 0)
    # KV accesses: config-2 appends and page reads of the second range, in order
    kv_a, kv_b, kv_o = wl.c2_step(trace.lengths, 0, trace.kv_steps, base=wl.C4_KV_BASE)
    assert np.array_equal(a[~moe].numpy().view(np.uint64), kv_a[:trace.n_kv])
    assert np.array_equal(b[~moe].numpy(), kv_b[:trace.n_kv].astype(np.int32))
    assert np.array_equal(o[~moe].numpy(), kv_o[:trace.n_kv])
    # channel shards: each keeps exactly its channels' accesses, in order
    # (three of the eight shards; every chunks() call regenerates the KV
    # step, a few seconds on the CPU)
    if n % 5 != 4:
        return
    ch = channel_of(a)
    for r in (0, 3, wl.C4_SHARDS - 1):
        sa, sb, so, st = _collect(trace, channel_of,
                                  lambda c, r=r: c % wl.C4_SHARDS == r, m=1000)
        mine = ch % wl.C4_SHARDS == r
        assert torch.equal(sa, a[mine]) and torch.equal(st, t[mine])
        assert torch.equal(sb, b[mine]) and torch.equal(so, o[mine])
