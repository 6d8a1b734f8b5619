// common.h -- host/device shared definitions for the B200 access-timing path.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define HD __host__ __device__ __forceinline__
#else
#define HD inline
#endif

namespace hbfb {

using u8 = std::uint8_t;
using u16 = std::uint16_t;
using u32 = std::uint32_t;
using u64 = std::uint64_t;
using i64 = std::int64_t;

// "minus infinity" of the max-plus algebra.  All real ticks handled by the
// parallel kernels are below 2^60 (checked on the host before launch), so a
// NEG-derived value stays below -2^61 after any number of additions the
// kernels perform and always loses a max against a real tick.
constexpr i64 kNeg = -(i64{1} << 62);
constexpr i64 kTickLimit = i64{1} << 60;

enum Status : u8 {
    kModeled = 1,
    kUnsupported = 6,
    kBypass = 8,
    kForeign = 9,
};

enum Model : u32 { kModelFast = 1, kModelDie = 3 };

// Device range record: the fields of the reference SharedRangeRecord
// (hbf_device.cuh:105-118) the batch path reads.
struct DevRange {
    u64 base;
    u64 length;
    u64 file_offset;
    u64 page_bytes;
    u32 range_id;
    u32 mode;
    u32 permissions;
    u32 reserved;      // log2(page_bytes)
    u64 end;           // base + length (registration rejects an overflow)
    u32 ok;            // mode 1 or 2, 0 < page_bytes <= 2^32
    u32 timing;        // timing path: bit op set = operation op allowed
                       // (ok, mode 1, permission bit); 0 for other ranges
};
static_assert(sizeof(DevRange) == 64, "range record layout");

// Divide a 32-bit value by an invariant 32-bit divisor with one 64-bit
// multiply-high (Lemire, Kaser & Kurz, "Faster remainder by direct
// computation", 2019: M = floor(2^64 / d) + 1 gives exact quotients for all
// 32-bit numerators).
struct FastDiv {
    u64 magic;
    u32 d;
    u32 pad;
};

HD FastDiv make_fastdiv(u32 d)
{
    FastDiv f{};
    f.d = d;
    f.magic = d <= 1 ? 0 : (~u64{0} / d) + 1;
    return f;
}

#if defined(__CUDACC__)
__device__ __forceinline__ u32 fastdiv_q(u32 n, const FastDiv& f)
{
    return f.d <= 1 ? n : static_cast<u32>(__umul64hi(f.magic, n));
}
#endif

// The one registered range of a context that has exactly one, by value in
// the kernel arguments so that its fields are read from the constant bank
// instead of being held in registers across the decode loops.
struct SingleRange {
    u64 base, length, file_offset, page_mask;  // page_mask = page_bytes - 1
    u32 allowed;  // DevRange::timing
    u32 valid;    // 0: decode against `ranges`
};

struct DecodeParams {
    const DevRange* ranges;  // sorted by base
    u32 range_count;
    SingleRange one;         // valid when ranges holds exactly one registered range
    u32 stripe_shift;
    u32 stacks;
    u32 dies;
    u32 planes;
    u32 page_bytes;
    u32 shard_rank;
    u32 shard_count;
    u32 channels_total;      // stacks * channels_per_stack
    u32 local_channels;      // ceil(channels_total / shard_count) (this shard)
    u8 order[4];             // fastest first: 0=C 1=W 2=D 3=P
    FastDiv radix[4];        // per letter
    FastDiv shard_div;
    FastDiv stack_div;
    FastDiv chan_stride;     // product of the radices faster than C
    FastDiv die_stride;      // product of the radices faster than D
    u32 pow2;                // every stride, radix and the shard count are 2^k
    u32 chan_shift, chan_mask, die_shift, die_mask, shard_shift, shard_mask;
};

struct TimingParams {
    u32 model;
    u32 dies;                // D (die model); 0 for fast
    u32 state_k;             // K = D+1 (die) or 1 (fast)
    u32 time_scale;
    // fast model constants (already scaled)
    i64 fast_x;
    i64 fast_l_read;
    i64 fast_l_prog;
    u64 fast_service_read;   // fast_service_ns, unscaled, per op (stats)
    u64 fast_service_prog;
    // die model per local channel tables (device pointers)
    const u64* chan_bw;      // effective bytes/s
    const i64* chan_t_read;  // scaled, throttled
    const i64* chan_t_prog;
    const i64* chan_admit;   // admit-after tick
    // per-die activity accumulation (NULL = off); index c*D+d
    unsigned long long* die_read_bytes;
    unsigned long long* die_writes;
    // activity counted by pass 1, [C*D][2] (read bytes, writes); the range
    // scan adds it to the die counters once the batch is accepted
    unsigned long long* act_stage;
    // 1: the batch order need not follow the arrival order (media actions
    // whose arrival waits for an earlier action's completion)
    u32 any_order;
    // < 32: every channel's transfer is (bytes + 2^x_shift - 1) >> x_shift
    // ticks before scaling; 0xff: per channel (ChanInfo)
    u32 x_shift;
    // bound on one access's transfer plus die time (scaled ticks, including
    // what the thermal controller may set); 0: unknown
    i64 step_max;
    // 1: every admission tick is 0 and stays 0 (thermal bounds included)
    u32 admit_zero;
};

// Device-side counters (one block of u64 per context).
struct DevCounters {
    unsigned long long modeled;
    unsigned long long bypass;
    unsigned long long unsupported;
    unsigned long long foreign;
    unsigned long long latency_sum;
    unsigned long long max_done;
    unsigned long long fast_modeled_ns;
    unsigned long long batches;
    unsigned long long errors;       // batches refused on the device
    unsigned long long error_code;   // last error bits
    unsigned long long pad[6];
};

// Error word of one batch.  kErrUnsorted refuses the batch (state kept);
// kErrNeedSeq reroutes it to the exact sequential kernel (a tick may reach
// 2^60, or a transfer time does not fit the packed 24-bit field).
enum DeviceError : u32 {
    kErrUnsorted = 1u,
    kErrNeedSeq = 2u,
    kErrWait = 4u,  // a bounded device wait gave up (fused thermal step)
};
constexpr u64 kArrivalLimit = u64{1} << 59;

}  // namespace hbfb
