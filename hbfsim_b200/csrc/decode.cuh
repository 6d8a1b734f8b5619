// decode.cuh -- device helpers shared by the batch kernels: saturating
// arithmetic, the reference range lookup and the access classification +
// stripe decode (A1/A2).
#pragma once

#include "common.h"

namespace hbfb {

// ---------------------------------------------------------------- helpers
__device__ __forceinline__ i64 imax(i64 a, i64 b) { return a > b ? a : b; }

__device__ __forceinline__ u64 sat_add_u64(u64 a, u64 b)
{
    return b > ~u64{0} - a ? ~u64{0} : a + b;
}

__device__ __forceinline__ u64 sat_mul_u64(u64 a, u32 b)
{
    return b != 0 && a > ~u64{0} / b ? ~u64{0} : a * b;
}

// ceil(n / d) for n < 2^63, d >= 1, quotient below 2^40: a double estimate
// corrected by integer checks (the estimate is within one of the quotient).
__device__ __forceinline__ u64 ceil_div_u64(u64 n, u64 d)
{
    u64 q = static_cast<u64>(static_cast<double>(n) / static_cast<double>(d));
#pragma unroll 1
    for (int k = 0; k < 3 && q * d > n; ++k) --q;
#pragma unroll 1
    for (int k = 0; k < 3 && n - q * d >= d; ++k) ++q;
    return q + (n != q * d ? 1u : 0u);
}

// hbf_device.cuh:826-841 -- upper-bound binary search on the sorted bases.
// `r` may point to global or shared memory.
__device__ __forceinline__ u32 find_range_index(const DevRange* r, u32 count,
                                                u64 address)
{
    u32 first = 0, last = count;
    while (first < last) {
        const u32 middle = first + (last - first) / 2;
        if (r[middle].base <= address) first = middle + 1;
        else last = middle;
    }
    return first == 0 ? count : first - 1;
}

// hbf_device.cuh:873-884
__device__ __forceinline__ bool range_overlaps(const DevRange& r, u64 a,
                                               u32 bytes)
{
    if (bytes == 0 || r.length == 0 || r.base > ~u64{0} - r.length ||
        a > ~u64{0} - bytes)
        return false;
    return a < r.base + r.length && r.base < a + bytes;
}

struct Decoded {
    u32 status;
    u32 range_index;
    u32 channel;   // global
    u32 local;     // local channel (this shard)
    u32 stack;
    u32 die;
    u32 plane;
    u64 media;
    u64 page;
};

// Classification in the order of __hbfsim_resolve (hbf_device.cu:997-1003
// zero bytes, 1083-1127 lookup / straddle / bypass, 1152-1179 media
// descriptor via access_supported hbf_device.cuh:843-862 and 929-944),
// followed by the stripe decode.  Page sizes are powers of two (profile
// validation), so the page arithmetic uses the range's page shift.
__device__ __forceinline__ Decoded classify_decode(const DecodeParams& p,
                                                   u64 a, u32 bytes, u32 op,
                                                   bool want_geometry)
{
    Decoded d{};
    d.range_index = p.range_count;
    if (bytes == 0) { d.status = kUnsupported; return d; }
    const u32 index = find_range_index(p.ranges, p.range_count, a);
    DevRange r{};
    if (index != p.range_count) r = p.ranges[index];
    if (index == p.range_count || a < r.base || a - r.base >= r.length) {
        const u32 successor = index == p.range_count ? 0u : index + 1u;
        if (successor < p.range_count &&
            range_overlaps(p.ranges[successor], a, bytes))
            d.status = kUnsupported;
        else
            d.status = kBypass;
        return d;
    }
    // access_supported (hbf_device.cuh:843-862)
    const u32 shift = r.reserved;
    if (op > 1 || (r.mode != 1 && r.mode != 2) || r.page_bytes == 0 ||
        r.page_bytes > 0xffffffffull || r.length > ~u64{0} - r.base ||
        bytes > ~u64{0} - a || a + bytes > r.base + r.length ||
        (r.permissions & (1u << op)) == 0) {
        d.status = kUnsupported;
        return d;
    }
    const u64 offset = a - r.base;
    if ((offset >> shift) != ((offset + bytes - 1) >> shift)) {
        d.status = kUnsupported;
        return d;
    }
    const u64 page_offset = (offset >> shift) << shift;
    if (page_offset > ~u64{0} - r.file_offset || r.mode != 1) {
        d.status = kUnsupported;
        return d;
    }
    d.media = r.file_offset + page_offset;
    d.range_index = index;
    d.status = kModeled;
    const u64 m = r.file_offset + offset;
    u32 u = static_cast<u32>(m >> p.stripe_shift);  // host: m>>shift < 2^32
    if (!want_geometry) return d;
    // stripe decode: mixed radix in allocation order, fastest letter first
    u32 digit[4] = {0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const u32 letter = p.order[k];
        const u32 q = fastdiv_q(u, p.radix[letter]);
        digit[letter] = u - q * p.radix[letter].d;
        u = q;
    }
    d.channel = digit[0];
    d.die = digit[2];
    d.plane = digit[3];
    const u32 sq = fastdiv_q(d.channel, p.stack_div);
    d.stack = d.channel - sq * p.stack_div.d;
    const u64 stripe_mask = (u64{1} << p.stripe_shift) - 1;
    d.page = ((static_cast<u64>(u) << p.stripe_shift) + (m & stripe_mask)) >>
             shift;
    const u32 lq = fastdiv_q(d.channel, p.shard_div);
    d.local = lq;
    if (p.shard_count > 1 && d.channel - lq * p.shard_div.d != p.shard_rank)
        d.status = kForeign;
    return d;
}

}  // namespace hbfb
