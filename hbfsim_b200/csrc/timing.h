// timing.h -- host-side entry points of the timing kernels (timing.cu).
#pragma once

#include "common.h"

#include <cuda_runtime.h>

namespace hbfb {

struct BatchPlan {
    u32 T, L, C, K, group_channels, ctas, tiles_per_cta, smem_bytes;
    u32 direct;  // 1: one register chain per channel; 0: pieces of L accesses
    u32 dies;
};

struct BatchIO {
    const u64* address;
    const u32* bytes;
    const u8* op;
    const u64* arrival;
    u64* done;
    u64* latency;
    u8* status;
    u64 n;
    bool aligned;
};

struct BatchScratch {
    i64* agg;
    i64* incoming;
    u32* error;
    u64* last_arrival;
    DevCounters* counters;
    const u64* state_in;
    u64* state_out;
    // range scan by look-back (optional: null selects one CTA per channel):
    // group maps and states, lb_group_words(ctas, C, K) words; and the
    // counters and flags, 2 + kLbFlagWords words at a fixed address, zero
    // before the first batch (each scan leaves them zero)
    i64* scan_groups = nullptr;
    u32* scan_lb = nullptr;
    // ranges agg / incoming / scan_groups can hold (a CTA may time two)
    u64 ranges_capacity = 0;
};

constexpr u32 kLbFlagWords = 16384;  // groups x local channels of one scan, at most

// Words of the look-back scan's group maps and states for `ctas` ranges
// (groups of 32 ranges).
inline u64 lb_group_words(u64 ctas, u64 C, u64 K)
{
    return (ctas + 31) / 32 * C * (K * (K + 1) + K);
}

// Optional launch markers (profiling): mark(slot, 0) before a launch and
// mark(slot, 1) after it, on the launching stream.
struct LaunchHooks {
    void* owner = nullptr;
    void (*mark)(void* owner, int slot, int phase, cudaStream_t stream) = nullptr;
    void operator()(int slot, int phase, cudaStream_t s) const
    {
        if (mark) mark(owner, slot, phase, s);
    }
};

enum KernelSlot : int {
    kSlotPass1 = 0, kSlotScan = 1, kSlotPass2 = 2, kSlotSequential = 3,
    kSlotDecode = 4, kSlotThermal = 5, kSlotController = 6, kSlotOther = 7,
};

// Tile size, channel grouping and grid for a batch of n accesses.
int plan_batch(u64 n, u32 C, u32 K, u32 dies, int sm_count, BatchPlan* plan);

cudaError_t launch_batch(const DecodeParams& dp, const TimingParams& tp,
                         const BatchIO& io, const BatchPlan& plan,
                         const BatchScratch& s, bool force_sequential,
                         cudaStream_t stream, const LaunchHooks& hooks = {});

cudaError_t launch_decode(const DecodeParams& dp, const u64* address,
                          const u32* bytes, const u8* op, u64 n, void* out,
                          cudaStream_t stream, const LaunchHooks& hooks = {});

// Hybrid sampler bits of n accesses (1 = the hybrid model would send the
// access to the reference media model); `seq` is the device-side running
// count of timed accesses, `counts` scratch of max_ctas words.
cudaError_t launch_sample(const DecodeParams& dp, const u64* address, const u32* bytes,
                          const u8* op, u64 n, u8* sample, u32 warmup, u64 threshold,
                          u64* seq, u64* counts, u32 max_ctas, cudaStream_t stream,
                          const LaunchHooks& hooks = {});

// Chained media actions: raise arrival[index] to done[chain[index]].
cudaError_t launch_chain_fixup(u64* arrival, const u64* done, const u32* chain, u64 index,
                               cudaStream_t stream);
// Exact single-thread walk of n chained actions (state_in -> state_out).
cudaError_t launch_chain_sequential(const DecodeParams& dp, const TimingParams& tp,
                                    const u64* address, const u32* bytes, const u8* op,
                                    u64* arrival, const u32* chain, u64 n, u32 K,
                                    const u64* state_in, u64* state_out, u64 words, u64* done,
                                    u64* latency, u8* status, cudaStream_t stream);

}  // namespace hbfb
