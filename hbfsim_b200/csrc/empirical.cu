// empirical.cu -- B200 kernels for the FAST model with an empirical
// burst-curve profile.
//
// The reference (src/cuda_runtime/device/hbf_device.cu:797-838) puts every
// access through two compare-and-swap loops on context-wide words: the packed
// burst state (run length of consecutive pages of one operation, capped at
// 1023, hbf_device.cuh:1058-1081) and the channel tail
// (target = max(tail, arrival) + scaled service).  Both are scans:
//
//   burst  every timed access carries key = 2*page + op + 1; its run length
//          is the length of the streak of keys stepping by 2 that ends at it,
//          capped.  Streak summaries (first key, last key, run at the last
//          key, whole-streak flag) compose associatively (burst_join).
//   tail   tail' = max(tail, a) + s is the max-plus map x -> max(x + s, a + s);
//          maps compose as (s1 + s2, max(m1 + s2, m2)) (mp_join).
//
// The run length fixes the service, so the burst scan comes first:
//   1 emp_burst_kernel       every CTA owns a contiguous range of 2048-access
//                            tiles: classification (one 8-byte record per
//                            access left in the latency buffer), burst
//                            summary of the range
//   2 emp_burst_scan_kernel  one CTA: incoming burst state of every range and
//                            the batch's final packed state
//   3 emp_reduce_kernel      run lengths (from the 8-byte records pass 1
//                            left in the latency buffer), services, max-plus
//                            summary of the range, arrival checks
//   4 emp_tail_scan_kernel   one CTA: incoming tail of every range; commits
//                            the state when the batch is accepted
//   5 emp_replay_kernel      per tile a burst block scan and a max-plus block
//                            scan give every access its run length and its
//                            completion tick; outputs written coalesced
// Integer and bit-exact: the host bounds the services, pass 3 checks the
// arrivals and pass 4 the carried tail, so every tick stays below 2^60 and
// signed max-plus arithmetic equals the reference's saturating arithmetic;
// otherwise the exact single-thread kernel runs instead.
#include "empirical.h"
#include "decode.cuh"

#include <algorithm>

namespace hbfb {

// ---------------------------------------------------------------- host side
namespace {

u64 host_sat_add(u64 a, u64 b) { return b > ~u64{0} - a ? ~u64{0} : a + b; }
u64 host_sat_mul(u64 a, u32 b) { return b != 0 && a > ~u64{0} / b ? ~u64{0} : a * b; }

// hbf_device.cuh:959-976: ceil(delta * offset / span), the product formed as
// whole spans times offset (saturating) plus the rounded-up share of the rest.
u64 scaled_ceiling(u64 delta, u32 offset, u32 span)
{
    if (delta == 0 || offset == 0) return 0;
    if (span == 0) return ~u64{0};
    const u64 whole = host_sat_mul(delta / span, offset);
    const u64 part = ((delta % span) * offset + span - 1) / span;
    return host_sat_add(whole, part);
}

// hbf_device.cuh:978-1019: cumulative time of a run of `run` pages, linear
// between breakpoints; past the last breakpoint the last segment extends.
u64 cumulative_ns(const u32* pages, const u64* cum, u32 count, u32 run)
{
    if (run == 0) return 0;
    if (!pages || !cum || count == 0) return ~u64{0};
    u32 hi = 0;
    while (hi < count && run > pages[hi]) ++hi;
    if (hi == count) hi = count - 1;
    const u32 lo_pages = hi ? pages[hi - 1] : 0;
    const u64 lo_ns = hi ? cum[hi - 1] : 0;
    if (pages[hi] <= lo_pages || cum[hi] < lo_ns || run < lo_pages) return ~u64{0};
    return host_sat_add(lo_ns, scaled_ceiling(cum[hi] - lo_ns, run - lo_pages,
                                              pages[hi] - lo_pages));
}

}  // namespace

bool empirical_control_valid(u32 flags, u32 count, u64 program_ns, const u32* pages,
                             const u64* cumulative)
{
    if (flags != 1 || count != 6 || program_ns == 0) return false;
    for (u32 i = 0; i < 6; ++i) {
        if (pages[i] == 0 || cumulative[i] == 0) return false;
        if (i && (pages[i] <= pages[i - 1] || cumulative[i] <= cumulative[i - 1])) return false;
    }
    return pages[5] <= kRunCap;
}

void empirical_service_table(const u32* pages, const u64* cumulative, u32 count, u64* out)
{
    out[0] = 0;
    u64 prev = 0;  // cumulative time of a run of 0 pages
    for (u32 r = 1; r <= kRunCap; ++r) {
        const u64 cur = cumulative_ns(pages, cumulative, count, r);
        out[r] = cur < prev ? ~u64{0} : cur - prev;
        prev = cur;
    }
}

// -------------------------------------------------------------- device side
namespace {

constexpr u32 kEThreads = 256;
constexpr u32 kEItems = 8;
constexpr u32 kETile = kEThreads * kEItems;
constexpr u32 kEWarps = kEThreads / 32;
constexpr u32 kScanThreads = kEmpMaxCtas;
constexpr u32 kWhole = 0x80000000u;
// Tile arrays are padded by one word per 8 so that a thread's 8 consecutive
// words (the blocked phase) fall on distinct banks.
constexpr u32 kEPad = kETile + kETile / kEItems;
__device__ __forceinline__ u32 pad(u32 e) { return e + (e >> 3); }

// Scratch words of CTA g: [8g+0..2] burst summary of its range, [8g+3..4]
// incoming burst (last key, run), [8g+5..6] max-plus summary (s, m),
// [8g+7] incoming tail.  Word 8*kEmpMaxCtas: the batch's final packed state.
constexpr u32 kFinalWord = 8 * kEmpMaxCtas;

struct EArgs {
    DecodeParams dp;
    EmpiricalParams ep;
    const u64* address;
    const u32* bytes;
    const u8* op;
    const u64* arrival;
    u64* done;
    u64* latency;
    u8* status;
    u64 n;
    u64 tiles;
    u32 ctas;    // CTAs of passes 3 and 5 (one contiguous tile range each)
    u32 ctas1;   // CTAs of pass 1: `split` per range
    u32 split;
    u64* words;
    u32* error;
    u64* last_arrival;
    DevCounters* counters;
    const u64* state_in;
    u64* state_out;
};

struct Burst {
    u64 first;  // key of the first timed access (0: none)
    u64 last;   // key of the last
    u32 tail;   // run length at `last` counted inside the stretch (capped);
                // kWhole when the whole stretch is one streak
};

struct MaxPlus {
    i64 s;  // x -> max(x + s, m)
    i64 m;
};

__device__ __forceinline__ Burst burst_join(const Burst& a, const Burst& b)
{
    if (b.first == 0) return a;
    if (a.first == 0) return b;
    Burst r{a.first, b.last, b.tail & ~kWhole};
    if ((b.tail & kWhole) && b.first == a.last + 2) {
        const u32 t = (a.tail & ~kWhole) + r.tail;
        r.tail = (t > kRunCap ? kRunCap : t) | (a.tail & kWhole);
    }
    return r;
}

__device__ __forceinline__ MaxPlus mp_join(const MaxPlus& a, const MaxPlus& b)
{
    return {a.s + b.s, imax(a.m + b.s, b.m)};
}

__device__ __forceinline__ Burst shfl_up(const Burst& v, u32 d)
{
    return {__shfl_up_sync(0xffffffffu, v.first, d), __shfl_up_sync(0xffffffffu, v.last, d),
            __shfl_up_sync(0xffffffffu, v.tail, d)};
}

__device__ __forceinline__ MaxPlus shfl_up(const MaxPlus& v, u32 d)
{
    return {__shfl_up_sync(0xffffffffu, v.s, d), __shfl_up_sync(0xffffffffu, v.m, d)};
}

// Exclusive scan over the block's threads in thread order; `total` gets the
// block's aggregate.  `tot` is shared scratch of THREADS/32 + 1 entries.
template <u32 THREADS, class T, class Join>
__device__ __forceinline__ T block_exclusive(const T& v, const T& id, T* tot, T& total,
                                             Join join)
{
    const u32 lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    T inc = v;
#pragma unroll
    for (u32 d = 1; d < 32; d <<= 1) {
        const T o = shfl_up(inc, d);
        if (lane >= d) inc = join(o, inc);
    }
    T exc = shfl_up(inc, 1);
    if (lane == 0) exc = id;
    if (lane == 31) tot[warp] = inc;
    __syncthreads();
    if (threadIdx.x == 0) {
        T run = id;
        for (u32 w = 0; w < THREADS / 32; ++w) {
            const T t = tot[w];
            tot[w] = run;
            run = join(run, t);
        }
        tot[THREADS / 32] = run;
    }
    __syncthreads();
    const T res = join(tot[warp], exc);
    total = tot[THREADS / 32];
    __syncthreads();
    return res;
}

// The carried packed state (hbf_device.cuh:1036-1056) as a one-access streak;
// a state that cannot continue a burst (zero, run 0, no page) is empty.
__device__ __forceinline__ Burst burst_of_state(u64 packed)
{
    const u32 run = static_cast<u32>(packed & kRunCap);
    const u64 page_plus_one = packed >> 11;
    if (packed == 0 || run == 0 || page_plus_one == 0) return {0, 0, 0};
    const u64 key = 2 * page_plus_one + ((packed >> 10) & 1u) - 1;
    return {key, key, run};
}

__device__ __forceinline__ u64 state_of(u64 key, u32 run)
{
    return (((key + 1) >> 1) << 11) | (((key - 1) & 1u) << 10) | run;
}

__device__ __forceinline__ Burst carried(u64 key, u32 run)
{
    return key ? Burst{key, key, run} : Burst{0, 0, 0};
}

// Classification in the reference order (zero bytes, lookup, straddle,
// bypass, media descriptor), then the empirical branch's own checks
// (hbf_device.cu:797-801): a 4 KiB media page on a 4 KiB boundary, the
// control header valid.  Returns the access's key, 0 when it is not timed.
__device__ __forceinline__ u64 access_key(const EArgs& a, u64 address, u32 bytes, u32 op,
                                          u32& status)
{
    const Decoded d = classify_decode(a.dp, address, bytes, op, false);
    status = d.status;
    if (d.status != kModeled) return 0;
    if (!a.ep.ok || a.dp.ranges[d.range_index].reserved != 12 || (d.media & 4095u) != 0) {
        status = kUnsupported;
        return 0;
    }
    return ((d.media >> 12) << 1) + op + 1;
}

// The same classification for a context with one registered range, its
// record in registers: access_supported and media_descriptor reduce to
// offset checks (registration rules out overflow), and the empirical checks
// (4 KiB pages, aligned file offset, header valid) are properties of the
// range, folded into `timed`.
struct KeyRange {
    u64 base, length, file_offset, page_mask;
    u32 allowed;  // DevRange::timing: operations a timing range allows
    u32 timed;    // the empirical checks pass for this range
};

__device__ __forceinline__ KeyRange key_range(const DevRange& r, u32 ok)
{
    const bool timed = ok && r.reserved == 12 && (r.file_offset & 4095u) == 0;
    return KeyRange{r.base, r.length, r.file_offset, (u64{1} << r.reserved) - 1, r.timing,
                    timed ? 1u : 0u};
}

__device__ __forceinline__ u64 key_single(const KeyRange& r, u64 a, u32 bytes, u32 op,
                                          u32& status)
{
    status = kUnsupported;
    if (bytes == 0) return 0;
    const u64 offset = a - r.base;  // wraps when a < base
    if (offset >= r.length) {
        // below the range: unsupported if it straddles into it; else bypass
        status = a < r.base && a <= ~u64{0} - bytes && r.base < a + bytes ? kUnsupported
                                                                          : kBypass;
        return 0;
    }
    if (op > 1 || ((r.allowed >> op) & 1u) == 0 || bytes > r.length - offset) return 0;
    if ((offset & r.page_mask) + bytes > r.page_mask + 1 || !r.timed) return 0;
    status = kModeled;
    return (((r.file_offset + offset) >> 12) << 1) + op + 1;
}

// Pass 1 leaves one 8-byte record per access in the caller's latency
// buffer: the key of a timed access (below 2^54: pages are below 2^52), or
// the status of any other access in the top byte.  Passes 3 and 5 read it
// instead of classifying again; pass 5 overwrites it with the latency.
constexpr u32 kStatusShift = 56;

__device__ __forceinline__ u64 record_key(u64 rec)
{
    return rec < (u64{1} << kStatusShift) ? rec : 0;
}

__device__ __forceinline__ void cta_range(u64 tiles, u32 ctas, u64& t0, u64& t1)
{
    t0 = tiles * blockIdx.x / ctas;
    t1 = tiles * (blockIdx.x + 1) / ctas;
}

__device__ __forceinline__ u32 tile_size(const EArgs& a, u64 t)
{
    const u64 start = t * kETile;
    return a.n - start < kETile ? static_cast<u32>(a.n - start) : kETile;
}

__device__ __forceinline__ Burst thread_burst(const u64* key)
{
    Burst own{0, 0, 0};
#pragma unroll
    for (u32 j = 0; j < kEItems; ++j)
        if (key[j]) own = burst_join(own, Burst{key[j], key[j], 1u | kWhole});
    return own;
}

// ------------------------------------------------------------ 1: burst sums
// `split` CTAs per range of the later passes (more loads in flight): CTA h
// covers tiles [h * tiles / ctas1, (h + 1) * tiles / ctas1), and range g of
// the later passes is exactly the union of CTAs g * split .. g * split + split - 1.
struct RawTile {
    u64 addr[kEItems];
    u32 bytes[kEItems];
    u32 op[kEItems];
};

__device__ __forceinline__ void load_raw(const EArgs& a, u64 start, u32 nt, RawTile& r)
{
#pragma unroll
    for (u32 k = 0; k < kEItems; ++k) {
        const u32 e = k * kEThreads + threadIdx.x;
        if (e < nt) {
            r.addr[k] = a.address[start + e];
            r.bytes[k] = a.bytes[start + e];
            r.op[k] = a.op[start + e];
        }
    }
}

__global__ void __launch_bounds__(kEThreads, 3) emp_burst_kernel(const EArgs a)
{
    __shared__ u64 s_key[kEPad];
    __shared__ Burst s_bt[kEWarps + 1];
    const u32 tid = threadIdx.x;
    u64 t0, t1;
    cta_range(a.tiles, a.ctas1, t0, t1);
    const bool single = a.dp.range_count == 1;
    const KeyRange kr = single ? key_range(a.dp.ranges[0], a.ep.ok) : KeyRange{};
    Burst acc{0, 0, 0};
    RawTile raw;
    if (t0 < t1) load_raw(a, t0 * kETile, tile_size(a, t0), raw);
    for (u64 t = t0; t < t1; ++t) {
        const u64 start = t * kETile;
        const u32 nt = tile_size(a, t);
#pragma unroll
        for (u32 k = 0; k < kEItems; ++k) {
            const u32 e = k * kEThreads + tid;
            u64 key = 0;
            if (e < nt) {
                u32 st;
                key = single ? key_single(kr, raw.addr[k], raw.bytes[k], raw.op[k], st)
                             : access_key(a, raw.addr[k], raw.bytes[k], raw.op[k], st);
                // the record the later passes read instead of classifying again
                a.latency[start + e] = key ? key : static_cast<u64>(st) << kStatusShift;
            }
            s_key[pad(e)] = key;
        }
        // the next tile's loads overlap this tile's scan
        if (t + 1 < t1) load_raw(a, start + kETile, tile_size(a, t + 1), raw);
        __syncthreads();
        u64 key[kEItems];
#pragma unroll
        for (u32 j = 0; j < kEItems; ++j) key[j] = s_key[pad(tid * kEItems + j)];
        Burst total;
        block_exclusive<kEThreads>(thread_burst(key), Burst{0, 0, 0}, s_bt, total, burst_join);
        acc = burst_join(acc, total);
    }
    if (tid == 0) {
        u64* w = a.words + 8ull * blockIdx.x;
        w[0] = acc.first;
        w[1] = acc.last;
        w[2] = acc.tail;
    }
}

// ------------------------------------------------------------ 2: burst scan
__global__ void __launch_bounds__(kScanThreads) emp_burst_scan_kernel(const EArgs a)
{
    __shared__ Burst s_bt[kScanThreads / 32 + 1];
    const u32 h = threadIdx.x;
    Burst v{0, 0, 0};
    if (h < a.ctas1) {
        const u64* w = a.words + 8ull * h;
        v = Burst{w[0], w[1], static_cast<u32>(w[2])};
    }
    Burst total;
    const Burst pre = block_exclusive<kScanThreads>(v, Burst{0, 0, 0}, s_bt, total, burst_join);
    const u64 packed = a.state_in[1];
    const Burst st = burst_of_state(packed);
    if (h < a.ctas1 && h % a.split == 0) {  // first pass-1 CTA of range g
        const Burst in = burst_join(st, pre);
        const u64 g = h / a.split;
        a.words[8 * g + 3] = in.last;
        a.words[8 * g + 4] = in.tail & ~kWhole;
    }
    if (h == 0) {
        // no timed access: the state stays as it was, whatever it holds
        const Burst out = burst_join(st, total);
        a.words[kFinalWord] = total.first ? state_of(out.last, out.tail & ~kWhole) : packed;
    }
}

// Passes 3 and 5 stage each tile's records and arrivals in shared memory
// with cp.async, double-buffered: the next tile streams in while the current
// one is scanned.  Layout of the dynamic shared memory: [2 buffers][records,
// arrivals][kEPad] u64.
__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gmem_src)
{
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst), "l"(gmem_src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all()
{
    asm volatile("cp.async.wait_all;\n" ::: "memory");
}

constexpr u32 kStageBytes = 4u * kEPad * 8u;

__device__ __forceinline__ void stage_tile(const EArgs& a, u64 start, u32 nt, u64* s_rec,
                                           u64* s_arr)
{
#pragma unroll
    for (u32 k = 0; k < kEItems; ++k) {
        const u32 e = k * kEThreads + threadIdx.x;
        if (e < nt) {
            cp_async8(&s_rec[pad(e)], a.latency + start + e);
            cp_async8(&s_arr[pad(e)], a.arrival + start + e);
        } else {
            s_rec[pad(e)] = 0;  // no access: no key
        }
    }
    cp_async_commit();
}

// One staged tile, blocked phase: each thread's 8 consecutive accesses get
// their run lengths from the burst scan and their scaled services.
struct TileWork {
    u64 rec[kEItems];
    u64 arr[kEItems];
    i64 s[kEItems];
    u64 svc_sum;     // unscaled services of the thread's timed accesses
    MaxPlus own;     // the thread's accesses as one max-plus map
    Burst btotal;    // the tile's burst summary
};

__device__ __forceinline__ void tile_services(const EArgs& a, const u64* s_rec, const u64* s_arr,
                                              const u64* s_svc, Burst* s_bt, u64 in_key,
                                              u32 in_run, u32 nt, TileWork& w)
{
    const u32 tid = threadIdx.x;
    u64 key[kEItems];
#pragma unroll
    for (u32 j = 0; j < kEItems; ++j) {
        const u32 e = tid * kEItems + j;
        w.rec[j] = s_rec[pad(e)];
        key[j] = record_key(w.rec[j]);
        w.arr[j] = e < nt ? s_arr[pad(e)] : 0;
    }
    const Burst pre = block_exclusive<kEThreads>(thread_burst(key), Burst{0, 0, 0}, s_bt,
                                                 w.btotal, burst_join);
    const Burst in = burst_join(carried(in_key, in_run), pre);
    u64 last = in.last;
    u32 run = in.tail & ~kWhole;
    w.own = MaxPlus{0, kNeg};
    w.svc_sum = 0;
#pragma unroll
    for (u32 j = 0; j < kEItems; ++j) {
        w.s[j] = 0;
        const u64 k = key[j];
        if (!k) continue;
        run = last != 0 && k == last + 2 ? (run < kRunCap ? run + 1 : kRunCap) : 1u;
        last = k;
        const u64 svc = ((k - 1) & 1u) ? a.ep.program_ns : s_svc[run];
        w.svc_sum += svc;
        w.s[j] = static_cast<i64>(svc * a.ep.time_scale);
        w.own = mp_join(w.own, MaxPlus{w.s[j], static_cast<i64>(w.arr[j]) + w.s[j]});
    }
}

// ---------------------------------------------------------- 3: tail summary
__global__ void __launch_bounds__(kEThreads, 2) emp_reduce_kernel(const EArgs a)
{
    extern __shared__ __align__(16) u64 e_smem[];
    __shared__ u64 s_svc[kRunCap + 1];
    __shared__ Burst s_bt[kEWarps + 1];
    __shared__ MaxPlus s_mt[kEWarps + 1];
    const u32 tid = threadIdx.x;
    for (u32 r = tid; r <= kRunCap; r += kEThreads) s_svc[r] = a.ep.service[r];
    u64 t0, t1;
    cta_range(a.tiles, a.ctas, t0, t1);
    const u64* cw = a.words + 8ull * blockIdx.x;
    u64 in_key = cw[3];
    u32 in_run = static_cast<u32>(cw[4]);
    MaxPlus acc{0, kNeg};
    bool unsorted = false, over = false;
    if (t0 < t1) stage_tile(a, t0 * kETile, tile_size(a, t0), e_smem, e_smem + kEPad);
    u32 b = 0;
    for (u64 t = t0; t < t1; ++t, b ^= 1u) {
        const u64 start = t * kETile;
        const u32 nt = tile_size(a, t);
        u64* s_rec = e_smem + 2 * b * kEPad;
        u64* s_arr = s_rec + kEPad;
        cp_async_wait_all();
        __syncthreads();  // tile t visible; everyone is done with the other buffer
        if (t + 1 < t1) {
            u64* n_rec = e_smem + 2 * (b ^ 1u) * kEPad;
            stage_tile(a, start + kETile, tile_size(a, t + 1), n_rec, n_rec + kEPad);
        }
        // arrival order across the whole batch (and after the previous batch)
        u64 prev = tid > 0 ? s_arr[pad(tid * kEItems - 1)]
                           : (start > 0 ? a.arrival[start - 1] : *a.last_arrival);
        TileWork w;
        tile_services(a, s_rec, s_arr, s_svc, s_bt, in_key, in_run, nt, w);
#pragma unroll
        for (u32 j = 0; j < kEItems; ++j) {
            if (tid * kEItems + j >= nt) break;
            unsorted |= w.arr[j] < prev;
            prev = w.arr[j];
            over |= record_key(w.rec[j]) != 0 && w.arr[j] >= kArrivalLimit;
        }
        MaxPlus mtotal;
        block_exclusive<kEThreads>(w.own, MaxPlus{0, kNeg}, s_mt, mtotal, mp_join);
        acc = mp_join(acc, mtotal);
        const Burst nb = burst_join(carried(in_key, in_run), w.btotal);
        in_key = nb.last;
        in_run = nb.tail & ~kWhole;
    }
    if (unsorted) atomicOr(a.error, kErrUnsorted);
    if (over) atomicOr(a.error, kErrNeedSeq);
    if (tid == 0) {
        u64* w = a.words + 8ull * blockIdx.x;
        w[5] = static_cast<u64>(acc.s);
        w[6] = static_cast<u64>(acc.m);
    }
}

// ------------------------------------------------------------- 4: tail scan
__global__ void __launch_bounds__(kScanThreads) emp_tail_scan_kernel(const EArgs a)
{
    __shared__ MaxPlus s_mt[kScanThreads / 32 + 1];
    const u32 g = threadIdx.x;
    const u32 err = *a.error;
    if (err & kErrUnsorted) {  // refused: the state is kept
        if (g == 0) {
            a.state_out[0] = a.state_in[0];
            a.state_out[1] = a.state_in[1];
            atomicAdd(&a.counters->errors, 1ull);
            atomicOr(&a.counters->error_code, static_cast<unsigned long long>(err));
        }
        return;
    }
    if (err & kErrNeedSeq) return;
    const u64 tail0 = a.state_in[0];
    if (tail0 >= kArrivalLimit) {
        if (g == 0) atomicOr(a.error, kErrNeedSeq);
        return;
    }
    MaxPlus v{0, kNeg};
    if (g < a.ctas) {
        const u64* w = a.words + 8ull * g;
        v = MaxPlus{static_cast<i64>(w[5]), static_cast<i64>(w[6])};
    }
    MaxPlus total;
    const MaxPlus pre = block_exclusive<kScanThreads>(v, MaxPlus{0, kNeg}, s_mt, total, mp_join);
    const i64 x = static_cast<i64>(tail0);
    if (g < a.ctas) a.words[8ull * g + 7] = static_cast<u64>(imax(x + pre.s, pre.m));
    if (g == 0) {
        a.state_out[0] = static_cast<u64>(imax(x + total.s, total.m));
        a.state_out[1] = a.words[kFinalWord];
        if (a.n) *a.last_arrival = a.arrival[a.n - 1];
        atomicAdd(&a.counters->batches, 1ull);
    }
}

__device__ void flush_counts(DevCounters* c, u64 mod, u64 byp, u64 uns, u64 lat, u64 mx,
                             u64 svc)
{
    __shared__ u64 s_red[kEWarps][6];
    const u32 lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
#pragma unroll
    for (u32 d = 16; d; d >>= 1) {
        mod += __shfl_down_sync(0xffffffffu, mod, d);
        byp += __shfl_down_sync(0xffffffffu, byp, d);
        uns += __shfl_down_sync(0xffffffffu, uns, d);
        lat += __shfl_down_sync(0xffffffffu, lat, d);
        svc += __shfl_down_sync(0xffffffffu, svc, d);
        const u64 o = __shfl_down_sync(0xffffffffu, mx, d);
        mx = o > mx ? o : mx;
    }
    if (lane == 0) {
        s_red[warp][0] = mod;
        s_red[warp][1] = byp;
        s_red[warp][2] = uns;
        s_red[warp][3] = lat;
        s_red[warp][4] = mx;
        s_red[warp][5] = svc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (u32 w = 1; w < kEWarps; ++w) {
            mod += s_red[w][0];
            byp += s_red[w][1];
            uns += s_red[w][2];
            lat += s_red[w][3];
            mx = s_red[w][4] > mx ? s_red[w][4] : mx;
            svc += s_red[w][5];
        }
        atomicAdd(&c->modeled, static_cast<unsigned long long>(mod));
        atomicAdd(&c->bypass, static_cast<unsigned long long>(byp));
        atomicAdd(&c->unsupported, static_cast<unsigned long long>(uns));
        atomicAdd(&c->latency_sum, static_cast<unsigned long long>(lat));
        atomicAdd(&c->fast_modeled_ns, static_cast<unsigned long long>(svc));
        atomicMax(&c->max_done, static_cast<unsigned long long>(mx));
    }
}

// ---------------------------------------------------------------- 5: replay
__global__ void __launch_bounds__(kEThreads, 2) emp_replay_kernel(const EArgs a)
{
    extern __shared__ __align__(16) u64 e_smem[];  // records -> completion ticks
    __shared__ u64 s_svc[kRunCap + 1];
    __shared__ u8 s_st[kETile];
    __shared__ Burst s_bt[kEWarps + 1];
    __shared__ MaxPlus s_mt[kEWarps + 1];
    if (*a.error) return;  // refused, or the sequential kernel times it
    const u32 tid = threadIdx.x;
    for (u32 r = tid; r <= kRunCap; r += kEThreads) s_svc[r] = a.ep.service[r];
    u64 t0, t1;
    cta_range(a.tiles, a.ctas, t0, t1);
    const u64* cw = a.words + 8ull * blockIdx.x;
    u64 in_key = cw[3];
    u32 in_run = static_cast<u32>(cw[4]);
    i64 tail = static_cast<i64>(cw[7]);
    u64 n_mod = 0, n_byp = 0, n_uns = 0, lat = 0, mx = 0, svc = 0;
    if (t0 < t1) stage_tile(a, t0 * kETile, tile_size(a, t0), e_smem, e_smem + kEPad);
    u32 b = 0;
    for (u64 t = t0; t < t1; ++t, b ^= 1u) {
        const u64 start = t * kETile;
        const u32 nt = tile_size(a, t);
        u64* s_rec = e_smem + 2 * b * kEPad;
        u64* s_arr = s_rec + kEPad;
        cp_async_wait_all();
        __syncthreads();  // tile t visible; everyone is done with the other buffer
        if (t + 1 < t1) {
            u64* n_rec = e_smem + 2 * (b ^ 1u) * kEPad;
            stage_tile(a, start + kETile, tile_size(a, t + 1), n_rec, n_rec + kEPad);
        }
        TileWork w;
        tile_services(a, s_rec, s_arr, s_svc, s_bt, in_key, in_run, nt, w);
        svc += w.svc_sum;
        MaxPlus mtotal;
        const MaxPlus pre = block_exclusive<kEThreads>(w.own, MaxPlus{0, kNeg}, s_mt, mtotal,
                                                       mp_join);
        i64 x = imax(tail + pre.s, pre.m);
#pragma unroll
        for (u32 j = 0; j < kEItems; ++j) {
            const u32 e = tid * kEItems + j;
            if (e >= nt) break;
            u64 d = w.arr[j];
            u32 st = static_cast<u32>(w.rec[j] >> kStatusShift);
            if (record_key(w.rec[j])) {
                x = imax(x, static_cast<i64>(w.arr[j])) + w.s[j];
                d = static_cast<u64>(x);
                lat += d - w.arr[j];
                mx = d > mx ? d : mx;
                st = kModeled;
                ++n_mod;
            } else if (st == kBypass) {
                ++n_byp;
            } else {
                ++n_uns;
            }
            s_rec[pad(e)] = d;
            s_st[e] = static_cast<u8>(st);
        }
        __syncthreads();
#pragma unroll 4
        for (u32 k = 0; k < kEItems; ++k) {
            const u32 e = k * kEThreads + tid;
            if (e < nt) {
                const u64 d = s_rec[pad(e)];
                a.done[start + e] = d;
                a.latency[start + e] = d - s_arr[pad(e)];
                a.status[start + e] = s_st[e];
            }
        }
        const Burst nb = burst_join(carried(in_key, in_run), w.btotal);
        in_key = nb.last;
        in_run = nb.tail & ~kWhole;
        tail = imax(tail + mtotal.s, mtotal.m);
    }
    flush_counts(a.counters, n_mod, n_byp, n_uns, lat, mx, svc);
}

// --------------------------------------------------- exact sequential walk
// hbf_device.cu:797-838 one access at a time, with the reference's
// saturating arithmetic (hbf_device.cuh:946-957) and burst update
// (hbf_device.cuh:1058-1081).  Runs only when the error word asks for it.
__global__ void emp_sequential_kernel(const EArgs a)
{
    const u32 flags = *a.error;
    if ((flags & kErrUnsorted) || !(flags & kErrNeedSeq)) return;
    u64 prev = *a.last_arrival;
    for (u64 i = 0; i < a.n; ++i) {
        if (a.arrival[i] < prev) {  // refused: the state is kept
            a.state_out[0] = a.state_in[0];
            a.state_out[1] = a.state_in[1];
            atomicAdd(&a.counters->errors, 1ull);
            atomicOr(&a.counters->error_code,
                     static_cast<unsigned long long>(flags | kErrUnsorted));
            return;
        }
        prev = a.arrival[i];
    }
    u64 tail = a.state_in[0], burst = a.state_in[1];
    unsigned long long n_mod = 0, n_byp = 0, n_uns = 0, lat = 0, mx = 0, svc_sum = 0;
    for (u64 i = 0; i < a.n; ++i) {
        u32 st;
        const u64 key = access_key(a, a.address[i], a.bytes[i], a.op[i], st);
        const u64 arr = a.arrival[i];
        a.status[i] = static_cast<u8>(st);
        if (!key) {
            a.done[i] = arr;
            a.latency[i] = 0;
            if (st == kBypass) ++n_byp;
            else ++n_uns;
            continue;
        }
        const u64 page = (key - 1) >> 1;
        const u32 op = static_cast<u32>((key - 1) & 1u);
        const u32 prev_run = static_cast<u32>(burst & kRunCap);
        const u64 prev_page_plus_one = burst >> 11;
        u32 run = 1;
        if (burst != 0 && prev_run != 0 && ((burst >> 10) & 1u) == op &&
            prev_page_plus_one != 0 && prev_page_plus_one == page)
            run = prev_run == kRunCap ? kRunCap : prev_run + 1;
        burst = ((page + 1) << 11) | (static_cast<u64>(op) << 10) | run;
        const u64 svc = op ? a.ep.program_ns : a.ep.service[run];
        const u64 start = tail > arr ? tail : arr;
        tail = sat_add_u64(start, sat_mul_u64(svc, a.ep.time_scale));
        a.done[i] = tail;
        a.latency[i] = tail - arr;
        ++n_mod;
        lat += tail - arr;
        mx = tail > mx ? tail : mx;
        svc_sum += svc;
    }
    a.state_out[0] = tail;
    a.state_out[1] = burst;
    atomicAdd(&a.counters->modeled, n_mod);
    atomicAdd(&a.counters->bypass, n_byp);
    atomicAdd(&a.counters->unsupported, n_uns);
    atomicAdd(&a.counters->latency_sum, lat);
    atomicAdd(&a.counters->fast_modeled_ns, svc_sum);
    atomicMax(&a.counters->max_done, mx);
    atomicAdd(&a.counters->batches, 1ull);
    if (a.n) *a.last_arrival = a.arrival[a.n - 1];
}

const u32 kSeqFlag = kErrNeedSeq;

}  // namespace

cudaError_t launch_empirical(const DecodeParams& dp, const EmpiricalParams& ep,
                             const BatchIO& io, const EmpiricalScratch& s,
                             bool force_sequential, int sm_count, cudaStream_t stream,
                             const LaunchHooks& hooks)
{
    cudaError_t err = cudaMemsetAsync(s.error, 0, sizeof(u32), stream);
    if (err != cudaSuccess) return err;
    if (force_sequential) {
        err = cudaMemcpyAsync(s.error, &kSeqFlag, sizeof(u32), cudaMemcpyHostToDevice, stream);
        if (err != cudaSuccess) return err;
    }
    EArgs a{};
    a.dp = dp;
    a.ep = ep;
    a.address = io.address;
    a.bytes = io.bytes;
    a.op = io.op;
    a.arrival = io.arrival;
    a.done = io.done;
    a.latency = io.latency;
    a.status = io.status;
    a.n = io.n;
    a.tiles = (io.n + kETile - 1) / kETile;
    for (auto k : {emp_reduce_kernel, emp_replay_kernel}) {
        err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(kStageBytes));
        if (err != cudaSuccess) return err;
    }
    // one wave: as many CTAs as the replay kernel keeps resident
    static int resident = 0;
    if (resident == 0 &&
        (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, emp_replay_kernel, kEThreads,
                                                       kStageBytes) != cudaSuccess ||
         resident < 1))
        resident = 1;
    const u64 want = static_cast<u64>(resident) * static_cast<u64>(sm_count > 0 ? sm_count : 148);
    a.ctas = static_cast<u32>(a.tiles < want ? a.tiles : want);
    if (a.ctas > kEmpMaxCtas) a.ctas = kEmpMaxCtas;
    // pass 1 splits every range over up to 4 CTAs (its loads want more CTAs)
    a.split = a.ctas ? std::min<u32>(4u, kEmpMaxCtas / a.ctas) : 1u;
    a.ctas1 = a.ctas * a.split;
    a.words = s.words;
    a.error = s.error;
    a.last_arrival = s.last_arrival;
    a.counters = s.counters;
    a.state_in = s.state_in;
    a.state_out = s.state_out;
    if (!force_sequential && a.ctas > 0) {
        hooks(kSlotPass1, 0, stream);
        emp_burst_kernel<<<a.ctas1, kEThreads, 0, stream>>>(a);
        hooks(kSlotPass1, 1, stream);
        hooks(kSlotScan, 0, stream);
        emp_burst_scan_kernel<<<1, kScanThreads, 0, stream>>>(a);
        hooks(kSlotScan, 1, stream);
        hooks(kSlotPass1, 0, stream);
        emp_reduce_kernel<<<a.ctas, kEThreads, kStageBytes, stream>>>(a);
        hooks(kSlotPass1, 1, stream);
        hooks(kSlotScan, 0, stream);
        emp_tail_scan_kernel<<<1, kScanThreads, 0, stream>>>(a);
        hooks(kSlotScan, 1, stream);
        hooks(kSlotPass2, 0, stream);
        emp_replay_kernel<<<a.ctas, kEThreads, kStageBytes, stream>>>(a);
        hooks(kSlotPass2, 1, stream);
    }
    hooks(kSlotSequential, 0, stream);
    emp_sequential_kernel<<<1, 1, 0, stream>>>(a);
    hooks(kSlotSequential, 1, stream);
    return cudaGetLastError();
}

}  // namespace hbfb
