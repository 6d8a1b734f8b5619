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
//                            tiles: classification, burst summary of the range
//   2 emp_burst_scan_kernel  one CTA: incoming burst state of every range and
//                            the batch's final packed state
//   3 emp_reduce_kernel      classification again, run lengths, services,
//                            max-plus summary of the range, arrival checks
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
    u32 ctas;
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
__device__ __forceinline__ u64 access_key(const EArgs& a, u64 i, u32& status)
{
    const u32 op = a.op[i];
    const Decoded d = classify_decode(a.dp, a.address[i], a.bytes[i], op, false);
    status = d.status;
    if (d.status != kModeled) return 0;
    if (!a.ep.ok || a.dp.ranges[d.range_index].reserved != 12 || (d.media & 4095u) != 0) {
        status = kUnsupported;
        return 0;
    }
    return ((d.media >> 12) << 1) + op + 1;
}

__device__ __forceinline__ void cta_tiles(const EArgs& a, u64& t0, u64& t1)
{
    t0 = a.tiles * blockIdx.x / a.ctas;
    t1 = a.tiles * (blockIdx.x + 1) / a.ctas;
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
__global__ void __launch_bounds__(kEThreads) emp_burst_kernel(const EArgs a)
{
    __shared__ u64 s_key[kEPad];
    __shared__ Burst s_bt[kEWarps + 1];
    const u32 tid = threadIdx.x;
    u64 t0, t1;
    cta_tiles(a, t0, t1);
    Burst acc{0, 0, 0};
    for (u64 t = t0; t < t1; ++t) {
        const u64 start = t * kETile;
        const u32 nt = a.n - start < kETile ? static_cast<u32>(a.n - start) : kETile;
#pragma unroll 2
        for (u32 k = 0; k < kEItems; ++k) {
            const u32 e = k * kEThreads + tid;
            u32 st;
            s_key[pad(e)] = e < nt ? access_key(a, start + e, st) : 0;
        }
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
    const u32 g = threadIdx.x;
    Burst v{0, 0, 0};
    if (g < a.ctas) {
        const u64* w = a.words + 8ull * g;
        v = Burst{w[0], w[1], static_cast<u32>(w[2])};
    }
    Burst total;
    const Burst pre = block_exclusive<kScanThreads>(v, Burst{0, 0, 0}, s_bt, total, burst_join);
    const u64 packed = a.state_in[1];
    const Burst st = burst_of_state(packed);
    if (g < a.ctas) {
        const Burst in = burst_join(st, pre);
        a.words[8ull * g + 3] = in.last;
        a.words[8ull * g + 4] = in.tail & ~kWhole;
    }
    if (g == 0) {
        // no timed access: the state stays as it was, whatever it holds
        const Burst out = burst_join(st, total);
        a.words[kFinalWord] = total.first ? state_of(out.last, out.tail & ~kWhole) : packed;
    }
}

// One tile through shared memory: keys and arrivals staged (striped,
// coalesced), then each thread's 8 consecutive accesses (blocked) get their
// run lengths from the burst scan and their scaled services.
struct TileWork {
    u64 key[kEItems];
    u64 arr[kEItems];
    i64 s[kEItems];
    u64 svc_sum;     // unscaled services of the thread's timed accesses
    MaxPlus own;     // the thread's accesses as one max-plus map
    Burst btotal;    // the tile's burst summary
};

__device__ __forceinline__ void tile_services(const EArgs& a, const u64* s_key, const u64* s_arr,
                                              const u64* s_svc, Burst* s_bt, u64 in_key,
                                              u32 in_run, u32 nt, TileWork& w)
{
    const u32 tid = threadIdx.x;
#pragma unroll
    for (u32 j = 0; j < kEItems; ++j) {
        const u32 e = tid * kEItems + j;
        w.key[j] = s_key[pad(e)];
        w.arr[j] = e < nt ? s_arr[pad(e)] : 0;
    }
    const Burst pre = block_exclusive<kEThreads>(thread_burst(w.key), Burst{0, 0, 0}, s_bt,
                                                 w.btotal, burst_join);
    const Burst in = burst_join(carried(in_key, in_run), pre);
    u64 last = in.last;
    u32 run = in.tail & ~kWhole;
    w.own = MaxPlus{0, kNeg};
    w.svc_sum = 0;
#pragma unroll
    for (u32 j = 0; j < kEItems; ++j) {
        w.s[j] = 0;
        const u64 k = w.key[j];
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
__global__ void __launch_bounds__(kEThreads, 3) emp_reduce_kernel(const EArgs a)
{
    __shared__ u64 s_key[kEPad];
    __shared__ u64 s_arr[kEPad];
    __shared__ u64 s_svc[kRunCap + 1];
    __shared__ Burst s_bt[kEWarps + 1];
    __shared__ MaxPlus s_mt[kEWarps + 1];
    const u32 tid = threadIdx.x;
    for (u32 r = tid; r <= kRunCap; r += kEThreads) s_svc[r] = a.ep.service[r];
    u64 t0, t1;
    cta_tiles(a, t0, t1);
    const u64* cw = a.words + 8ull * blockIdx.x;
    u64 in_key = cw[3];
    u32 in_run = static_cast<u32>(cw[4]);
    MaxPlus acc{0, kNeg};
    bool unsorted = false, over = false;
    for (u64 t = t0; t < t1; ++t) {
        const u64 start = t * kETile;
        const u32 nt = a.n - start < kETile ? static_cast<u32>(a.n - start) : kETile;
#pragma unroll 2
        for (u32 k = 0; k < kEItems; ++k) {
            const u32 e = k * kEThreads + tid;
            u64 key = 0;
            if (e < nt) {
                u32 st;
                key = access_key(a, start + e, st);
                s_arr[pad(e)] = a.arrival[start + e];
            }
            s_key[pad(e)] = key;
        }
        __syncthreads();
        // arrival order across the whole batch (and after the previous batch)
        u64 prev = tid > 0 ? s_arr[pad(tid * kEItems - 1)]
                           : (start > 0 ? a.arrival[start - 1] : *a.last_arrival);
        TileWork w;
        tile_services(a, s_key, s_arr, s_svc, s_bt, in_key, in_run, nt, w);
#pragma unroll
        for (u32 j = 0; j < kEItems; ++j) {
            if (tid * kEItems + j >= nt) break;
            unsorted |= w.arr[j] < prev;
            prev = w.arr[j];
            over |= w.key[j] != 0 && w.arr[j] >= kArrivalLimit;
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
__global__ void __launch_bounds__(kEThreads, 3) emp_replay_kernel(const EArgs a)
{
    __shared__ u64 s_key[kEPad];  // keys, then completion ticks
    __shared__ u64 s_arr[kEPad];
    __shared__ u64 s_svc[kRunCap + 1];
    __shared__ Burst s_bt[kEWarps + 1];
    __shared__ MaxPlus s_mt[kEWarps + 1];
    if (*a.error) return;  // refused, or the sequential kernel times it
    const u32 tid = threadIdx.x;
    for (u32 r = tid; r <= kRunCap; r += kEThreads) s_svc[r] = a.ep.service[r];
    u64 t0, t1;
    cta_tiles(a, t0, t1);
    const u64* cw = a.words + 8ull * blockIdx.x;
    u64 in_key = cw[3];
    u32 in_run = static_cast<u32>(cw[4]);
    i64 tail = static_cast<i64>(cw[7]);
    u64 n_mod = 0, n_byp = 0, n_uns = 0, lat = 0, mx = 0, svc = 0;
    for (u64 t = t0; t < t1; ++t) {
        const u64 start = t * kETile;
        const u32 nt = a.n - start < kETile ? static_cast<u32>(a.n - start) : kETile;
#pragma unroll 2
        for (u32 k = 0; k < kEItems; ++k) {
            const u32 e = k * kEThreads + tid;
            u64 key = 0;
            if (e < nt) {
                u32 st;
                key = access_key(a, start + e, st);
                a.status[start + e] = static_cast<u8>(st);
                n_mod += st == kModeled;
                n_byp += st == kBypass;
                n_uns += st != kModeled && st != kBypass;
                s_arr[pad(e)] = a.arrival[start + e];
            }
            s_key[pad(e)] = key;
        }
        __syncthreads();
        TileWork w;
        tile_services(a, s_key, s_arr, s_svc, s_bt, in_key, in_run, nt, w);
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
            if (w.key[j]) {
                x = imax(x, static_cast<i64>(w.arr[j])) + w.s[j];
                d = static_cast<u64>(x);
                lat += d - w.arr[j];
                mx = d > mx ? d : mx;
            }
            s_key[pad(e)] = d;
        }
        __syncthreads();
#pragma unroll 2
        for (u32 k = 0; k < kEItems; ++k) {
            const u32 e = k * kEThreads + tid;
            if (e < nt) {
                const u64 d = s_key[pad(e)];
                a.done[start + e] = d;
                a.latency[start + e] = d - s_arr[pad(e)];
            }
        }
        const Burst nb = burst_join(carried(in_key, in_run), w.btotal);
        in_key = nb.last;
        in_run = nb.tail & ~kWhole;
        tail = imax(tail + mtotal.s, mtotal.m);
        __syncthreads();  // the next tile overwrites the staged arrays
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
        const u64 key = access_key(a, i, st);
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
    // one wave: as many CTAs as the replay kernel keeps resident
    static int resident = 0;
    if (resident == 0 &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, emp_replay_kernel, kEThreads, 0) !=
            cudaSuccess)
        resident = 2;
    if (resident < 1) resident = 1;
    const u64 want = static_cast<u64>(resident) * static_cast<u64>(sm_count > 0 ? sm_count : 148);
    a.ctas = static_cast<u32>(a.tiles < want ? a.tiles : want);
    if (a.ctas > kEmpMaxCtas) a.ctas = kEmpMaxCtas;
    a.words = s.words;
    a.error = s.error;
    a.last_arrival = s.last_arrival;
    a.counters = s.counters;
    a.state_in = s.state_in;
    a.state_out = s.state_out;
    if (!force_sequential && a.ctas > 0) {
        hooks(kSlotPass1, 0, stream);
        emp_burst_kernel<<<a.ctas, kEThreads, 0, stream>>>(a);
        hooks(kSlotPass1, 1, stream);
        hooks(kSlotScan, 0, stream);
        emp_burst_scan_kernel<<<1, kScanThreads, 0, stream>>>(a);
        hooks(kSlotScan, 1, stream);
        hooks(kSlotPass1, 0, stream);
        emp_reduce_kernel<<<a.ctas, kEThreads, 0, stream>>>(a);
        hooks(kSlotPass1, 1, stream);
        hooks(kSlotScan, 0, stream);
        emp_tail_scan_kernel<<<1, kScanThreads, 0, stream>>>(a);
        hooks(kSlotScan, 1, stream);
        hooks(kSlotPass2, 0, stream);
        emp_replay_kernel<<<a.ctas, kEThreads, 0, stream>>>(a);
        hooks(kSlotPass2, 1, stream);
    }
    hooks(kSlotSequential, 0, stream);
    emp_sequential_kernel<<<1, 1, 0, stream>>>(a);
    hooks(kSlotSequential, 1, stream);
    return cudaGetLastError();
}

}  // namespace hbfb
