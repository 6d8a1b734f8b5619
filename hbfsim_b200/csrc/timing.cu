// timing.cu -- B200 kernels for the batched HBF access-timing path.
//
// One batch is timed by three launches on one stream:
//
//   pass 1  (timing_pass_kernel<..., 1>)  every CTA owns a contiguous range of
//           tiles.  Per tile: stage the SoA inputs in shared memory, run the
//           range lookup + stripe decode (A1/A2), partition the tile by local
//           channel with a stable in-SMEM counting sort, and build the max-plus
//           matrix of every piece (<= L consecutive accesses of one channel).
//           The pieces are folded into the CTA's range aggregate R_b
//           (per channel a K x (K+1) max-plus affine map, K = state words).
//   scan    (range_scan_kernel)  one CTA per channel applies R_0, R_1, ...
//           to the channel's carried state and writes each CTA's incoming
//           state.
//   pass 2  (timing_pass_kernel<..., 2>)  every CTA re-stages its tiles,
//           propagates its incoming state through the pieces (one max-plus
//           matrix-vector product per piece) and replays each piece from its
//           exact incoming state, writing completion tick, latency and status.
//
// The direct kernel (direct_pass_kernel, die model with few dies) keeps the
// state in registers instead of pieces, and its pass 1 leaves one compact
// record per access in the latency buffer, so that its pass 2 re-reads only
// arrivals and records: no second decode or partition.
//
// Why max-plus: both timing models are max-plus affine in the per-channel
// state (see the step functions below), so a chunk of accesses is summarized
// exactly by a K x (K+1) matrix, and chunks compose associatively.  Column r
// of a piece's matrix is the piece replayed from the unit state e_r (r < K,
// arrivals ignored) or from the all-NEG state with real arrivals (r == K).
//
// Integer, bit-exact: the host proves every tick stays below 2^60, so signed
// 64-bit max-plus arithmetic equals the reference's saturating unsigned
// arithmetic; batches that fail the proof run the sequential kernel instead.
#include "timing.h"
#include "decode.cuh"

namespace hbfb {

// Timing decode: status, local channel and die only -- the classification
// of classify_decode on the precomputed range record, then the channel and
// die digits straight from their strides in the allocation order
// (digit = (u / stride) % radix): shifts and masks when every factor is a
// power of two, invariant divisions otherwise.
struct TimingDecoded {
    u32 status;
    u32 local;
    u32 die;
};

__device__ __forceinline__ TimingDecoded classify_timing(const DecodeParams& p, u64 a,
                                                         u32 bytes, u32 op)
{
    TimingDecoded d{kUnsupported, 0, 0};
    if (bytes == 0) return d;                                  // hbf_device.cu:997-1003
    const u32 index = p.range_count == 1 ? (p.ranges[0].base <= a ? 0u : 1u)
                                         : find_range_index(p.ranges, p.range_count, a);
    const u64 offset = index < p.range_count ? a - p.ranges[index].base : 0;
    if (index == p.range_count || offset >= p.ranges[index].length) {
        const u32 successor = index == p.range_count ? 0u : index + 1u;  // 1083-1127
        d.status = successor < p.range_count && range_overlaps(p.ranges[successor], a, bytes)
                       ? kUnsupported : kBypass;
        return d;
    }
    const DevRange& r = p.ranges[index];
    // access_supported (hbf_device.cuh:843-862) and media_descriptor
    // (929-944).  Registration guarantees base + length and file_offset +
    // length do not overflow, so with offset < length the reference's
    // overflow checks reduce to bytes <= length - offset, and r.timing holds
    // the operations a timing range allows.
    if (op > 1 || ((r.timing >> op) & 1u) == 0 || bytes > r.length - offset) return d;
    const u64 page_mask = (u64{1} << r.reserved) - 1;
    if ((offset & page_mask) + bytes > page_mask + 1) return d;   // one page only
    const u32 u = static_cast<u32>((r.file_offset + offset) >> p.stripe_shift);
    u32 g;
    if (p.pow2) {
        g = (u >> p.chan_shift) & p.chan_mask;
        d.die = (u >> p.die_shift) & p.die_mask;
        d.local = g >> p.shard_shift;
        d.status = (g & p.shard_mask) == p.shard_rank ? kModeled : kForeign;
    } else {
        const u32 uc = fastdiv_q(u, p.chan_stride);
        g = uc - fastdiv_q(uc, p.radix[0]) * p.radix[0].d;
        const u32 ud = fastdiv_q(u, p.die_stride);
        d.die = ud - fastdiv_q(ud, p.radix[2]) * p.radix[2].d;
        const u32 lq = fastdiv_q(g, p.shard_div);
        d.local = lq;
        d.status = p.shard_count > 1 && g - lq * p.shard_div.d != p.shard_rank ? kForeign
                                                                                 : kModeled;
    }
    return d;
}

// The same classification for a context with one registered range, its
// record passed by value in the kernel arguments.
template <bool POW2 = false>
__device__ __forceinline__ TimingDecoded classify_single(const SingleRange& r,
                                                         const DecodeParams& p, u64 a,
                                                         u32 bytes, u32 op)
{
    TimingDecoded d{kUnsupported, 0, 0};
    if (bytes == 0) return d;                                  // hbf_device.cu:997-1003
    const u64 offset = a - r.base;  // wraps when a < base
    if (offset >= r.length) {
        // below the range: unsupported if it straddles into it; else bypass
        d.status = a < r.base && a <= ~u64{0} - bytes && r.base < a + bytes ? kUnsupported
                                                                           : kBypass;
        return d;
    }
    if (op > 1 || ((r.allowed >> op) & 1u) == 0 || bytes > r.length - offset) return d;
    if ((offset & r.page_mask) + bytes > r.page_mask + 1) return d;
    const u32 u = static_cast<u32>((r.file_offset + offset) >> p.stripe_shift);
    u32 g;
    if (POW2 || p.pow2) {
        g = (u >> p.chan_shift) & p.chan_mask;
        d.die = (u >> p.die_shift) & p.die_mask;
        d.local = g >> p.shard_shift;
        d.status = (g & p.shard_mask) == p.shard_rank ? kModeled : kForeign;
    } else {
        const u32 uc = fastdiv_q(u, p.chan_stride);
        g = uc - fastdiv_q(uc, p.radix[0]) * p.radix[0].d;
        const u32 ud = fastdiv_q(u, p.die_stride);
        d.die = ud - fastdiv_q(ud, p.radix[2]) * p.radix[2].d;
        const u32 lq = fastdiv_q(g, p.shard_div);
        d.local = lq;
        d.status = p.shard_count > 1 && g - lq * p.shard_div.d != p.shard_rank ? kForeign
                                                                                 : kModeled;
    }
    return d;
}

// The exact sequential walk with the reference's saturating unsigned
// arithmetic, for one local channel c: the batch in order, the accesses of
// channel c timed, the untimed ones written by channel 0's thread.
template <int MODEL>
__device__ void sequential_walk(const DecodeParams& dp, const TimingParams& tp,
                                const u64* address, const u32* bytes, const u8* op,
                                const u64* arrival, u64* done_out, u64* latency, u8* status,
                                u64 n, u32 K, const u64* state_in, u64* state_out,
                                u64* last_arrival, DevCounters* counters, u32 c)
{
    struct {
        const DecodeParams& dp;
        const TimingParams& tp;
        const u64* address;
        const u32* bytes;
        const u8* op;
        const u64* arrival;
        u64* done;
        u64* latency;
        u8* status;
        u64 n;
        u32 K;
        const u64* state_in;
        u64* state_out;
        u64* last_arrival;
        DevCounters* counters;
    } a{dp, tp, address, bytes, op, arrival, done_out, latency, status, n, K, state_in,
        state_out, last_arrival, counters};
    u64 st[17];
    for (u32 k = 0; k < a.K; ++k) st[k] = a.state_in[static_cast<u64>(c) * a.K + k];
    unsigned long long n_mod = 0, n_byp = 0, n_uns = 0, n_for = 0, lat = 0,
                       mx = 0, fast = 0;
    for (u64 i = 0; i < a.n; ++i) {
        const u64 arr = a.arrival[i];
        const Decoded d = classify_decode(a.dp, a.address[i], a.bytes[i], a.op[i],
                                          MODEL == kModelDie);
        const u32 key = MODEL == kModelDie ? d.local : 0u;
        if (d.status != kModeled) {
            if (c == 0) {
                a.done[i] = arr;
                a.latency[i] = 0;
                a.status[i] = static_cast<u8>(d.status);
                if (d.status == kBypass) ++n_byp;
                else if (d.status == kForeign) ++n_for;
                else ++n_uns;
            }
            continue;
        }
        if (key != c) continue;
        u64 done;
        if (MODEL == kModelFast) {
            const u64 x = static_cast<u64>(a.tp.fast_x);  // host: already saturated
            const u64 lat_op = static_cast<u64>(a.op[i] ? a.tp.fast_l_prog : a.tp.fast_l_read);
            const u64 s = st[0] > arr ? st[0] : arr;
            st[0] = sat_add_u64(s, x);
            const u64 lt = sat_add_u64(arr, lat_op);
            done = lt > st[0] ? lt : st[0];
            fast += a.op[i] ? a.tp.fast_service_prog : a.tp.fast_service_read;
        } else {
            const u64 bw = a.tp.chan_bw[c];
            const u64 num = static_cast<u64>(a.bytes[i]) * 1000000000ull;
            const u64 x = sat_mul_u64(num / bw + (num % bw != 0), a.tp.time_scale);
            const u64 top = static_cast<u64>(a.op[i] ? a.tp.chan_t_prog[c] : a.tp.chan_t_read[c]);
            u64 s = arr;
            const u64 admit = static_cast<u64>(a.tp.chan_admit[c]);
            if (admit > s) s = admit;
            if (st[0] > s) s = st[0];
            if (st[1 + d.die] > s) s = st[1 + d.die];
            st[0] = sat_add_u64(s, x);
            st[1 + d.die] = sat_add_u64(st[0], top);
            done = st[1 + d.die];
            if (a.tp.die_read_bytes) {  // this thread owns channel c's dies
                const u64 k = static_cast<u64>(c) * a.tp.dies + d.die;
                if (a.op[i]) a.tp.die_writes[k] += 1;
                else a.tp.die_read_bytes[k] += a.bytes[i];
            }
        }
        a.done[i] = done;
        a.latency[i] = done - arr;
        a.status[i] = kModeled;
        ++n_mod;
        lat += done - arr;
        mx = done > mx ? done : mx;
    }
    for (u32 k = 0; k < a.K; ++k) a.state_out[static_cast<u64>(c) * a.K + k] = st[k];
    atomicAdd(&a.counters->modeled, n_mod);
    if (c == 0) {
        atomicAdd(&a.counters->bypass, n_byp);
        atomicAdd(&a.counters->foreign, n_for);
        atomicAdd(&a.counters->unsupported, n_uns);
        atomicAdd(&a.counters->batches, 1ull);
        if (a.n) *a.last_arrival = a.arrival[a.n - 1];
    }
    atomicAdd(&a.counters->latency_sum, lat);
    atomicAdd(&a.counters->fast_modeled_ns, fast);
    atomicMax(&a.counters->max_done, mx);
}

// ---------------------------------------------------------------- kernels
struct PassArgs {
    DecodeParams dp;
    TimingParams tp;
    const u64* address;
    const u32* bytes;
    const u8* op;
    const u64* arrival;
    u64* done;
    u64* latency;
    u8* status;
    u64 n;
    u32 tiles_per_cta;
    u32 vec;        // all SoA pointers 16-byte aligned: vector loads/stores
    u32 T;          // tile size (multiple of 32 * warps)
    u32 L;          // piece length
    u32 C;          // local channels
    u32 K;          // state words per channel
    u32 group_channels;  // channels per piece-matrix group
    u32 pm_capacity;     // piece slots in shared memory per group
    // shared memory offsets (bytes)
    u32 off_addr, off_arr, off_bytes, off_op, off_ord, off_key, off_rank;
    u32 off_wcnt, off_seg, off_pbase, off_pchan, off_pm, off_pin, off_die;
    u32 off_chan, off_act, off_red, off_ranges;
    u32 off_sarr[2], off_sinfo[2];  // direct kernel: channel-sorted arrays per pass
    u32 off_slot;                   // direct replay: sorted slot of each access
    u32 off_dies[2];                // direct pass 1: die words of the 32-bit chains
    u32 off_xtab;                   // general direct pass 1: transfer ticks of pow2 sizes
    u32 off_mid;                    // halves: each channel's split point (pass 1)
    u32 halves;                     // one tile per CTA, its two halves separate ranges
    // global scratch
    i64* agg;        // [ctas][C][K][K+1]  (pass 1 out)
    i64* incoming;   // [ctas][C][K]       (pass 2 in, carried in place)
    u32* error;      // device error bits of this batch
    const u64* last_arrival;  // last arrival of the previous batch
    const u64* state_in;      // carried state (checked against the tick limit)
    DevCounters* counters;
    u64* state_out;           // direct pass 2: the sequential walk's final state
};

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr u32 kThreadsDie = kThreads;  // stride of the shared die words (rel32_loop)

struct ChanInfo {  // per local channel, staged in shared memory
    i64 t_read;
    i64 t_prog;
    i64 admit;
    u64 bw;
    u32 x_add;     // transfer = (bytes + x_add) >> x_shift, x_add = 2^x_shift - 1,
    u32 x_shift;   // when 1e9 / bw reduces to 1 / 2^x_shift; else x_shift = kXDivide
                   // and x_add holds 1 / bw as an fp32 (the quotient's estimate)
};

constexpr u32 kXDivide = 0xffu;
// per-channel transfer ticks of the power-of-two sizes 2^kXTabMin ..
// 2^(kXTabMin + kXTabSizes - 1), tabulated by the general pass-1 kernel
constexpr u32 kXTabMin = 4, kXTabSizes = 12;

// ceil(bytes * 1e9 / bw) * time_scale for one access of a channel.  An
// access never exceeds its page (access_supported), and the host admits the
// parallel path only when a page's transfer times the scale stays below
// 2^24, so the plain product is exact here.  Per-channel rates are mostly
// 1e9 * 2^k bytes per second (a shift); otherwise the quotient q of
// n = bytes * 1e9 by bw is estimated as n * r in fp64, r = 1 / bw rounded
// to fp32 (relative error 2^-24, plus 2^-52 for the product), so for every
// q below 2^23 the estimate is within 0.6 of the quotient and one step of
// the exact remainder test settles it; larger estimates take the division.
__device__ __noinline__ u64 transfer_ticks_div(u64 n, u64 d) { return ceil_div_u64(n, d); }

__device__ __forceinline__ u64 transfer_ticks(u32 bytes, const ChanInfo& ci, u32 scale)
{
    const uint2 code = *reinterpret_cast<const uint2*>(&ci.x_add);
    if (code.y != kXDivide) {
        const u32 x = static_cast<u32>((static_cast<u64>(bytes) + code.x) >> code.y);
        return static_cast<u64>(x) * scale;
    }
    const u64 n = static_cast<u64>(bytes) * 1000000000ull, d = ci.bw;
    const double r = static_cast<double>(__uint_as_float(code.x));
    u64 q = static_cast<u64>(static_cast<double>(n) * r);
    if (q >= (u64{1} << 23)) return transfer_ticks_div(n, d) * scale;
    if (q * d > n) --q;                 // now q * d <= n
    else if (n - q * d >= d) ++q;       // now n - q * d < d
    return (q + (q * d != n ? 1u : 0u)) * scale;
}

__device__ ChanInfo stage_channel(const TimingParams& tp, u32 c, bool die)
{
    ChanInfo ci{};
    if (!die) return ci;
    ci.t_read = tp.chan_t_read[c];
    ci.t_prog = tp.chan_t_prog[c];
    ci.admit = tp.chan_admit[c];
    ci.bw = tp.chan_bw[c];
    // 1e9 / bw is 1 / 2^s exactly when bw = 1e9 * 2^s
    ci.x_shift = kXDivide;
    ci.x_add = __float_as_uint(ci.bw ? static_cast<float>(1.0 / static_cast<double>(ci.bw))
                                     : 0.0f);
    const u64 den = ci.bw / 1000000000ull;
    if (ci.bw % 1000000000ull == 0 && den != 0 && (den & (den - 1)) == 0 &&
        63 - __clzll(den) < 32) {
        ci.x_shift = 63 - __clzll(den);
        ci.x_add = static_cast<u32>((u64{1} << ci.x_shift) - 1);
    }
    return ci;
}

template <int MODEL>
struct StepModel;

// FAST model, hbf_device.cu:883-910: one tail for the whole device.
//   tail' = max(tail, a) + X ;  done = max(a + L_op, tail')
template <>
struct StepModel<kModelFast> {
    static __device__ __forceinline__ i64 step(i64& chan, i64* /*die*/,
                                               u32 /*stride*/, i64 a, u32 info,
                                               const ChanInfo&,
                                               const TimingParams& tp)
    {
        chan = imax(chan, a) + tp.fast_x;
        const i64 lat = (info >> 28) & 1u ? tp.fast_l_prog : tp.fast_l_read;
        return imax(a + lat, chan);
    }
};

// DIE model (north-star recurrence, builder-fixed details):
//   start = max(a, channel_free, die_free[d]); channel_free = start + X;
//   die_free[d] = channel_free + T_op; done = die_free[d]
template <>
struct StepModel<kModelDie> {
    static __device__ __forceinline__ i64 step(i64& chan, i64* die,
                                               u32 stride, i64 a, u32 info,
                                               const ChanInfo& ci,
                                               const TimingParams&)
    {
        const i64 x = static_cast<i64>(info & 0xffffffu);
        const u32 d = (info >> 24) & 15u;
        const i64 t = (info >> 28) & 1u ? ci.t_prog : ci.t_read;
        i64* slot = die + d * stride;
        const i64 start = imax(imax(a, chan), *slot);
        chan = start + x;
        const i64 done = chan + t;
        *slot = done;
        return done;
    }
};

// The same DIE step with the die state in registers (D known at compile
// time): the die slot is read through a select chain and written with
// predicated moves, so the loop-carried chain never goes through memory.
template <int D>
struct DieRegs {
    i64 chan;
    i64 die[D];
    __device__ __forceinline__ i64 step(i64 a, u32 info, const ChanInfo& ci)
    {
        const i64 x = static_cast<i64>(info & 0xffffffu);
        const u32 d = (info >> 24) & 15u;
        const i64 t = (info >> 28) & 1u ? ci.t_prog : ci.t_read;
        i64 cur = die[0];
#pragma unroll
        for (int j = 1; j < D; ++j) cur = d == static_cast<u32>(j) ? die[j] : cur;
        const i64 start = imax(imax(a, chan), cur);
        chan = start + x;
        const i64 done = chan + t;
#pragma unroll
        for (int j = 0; j < D; ++j)
            if (d == static_cast<u32>(j)) die[j] = done;
        return done;
    }
    // The same step with the arrival at -inf (the unit columns of pass 1):
    // every state word is >= NEG, so max(NEG, chan) is chan.
    __device__ __forceinline__ void step_unit(u32 info, const ChanInfo& ci)
    {
        const i64 x = static_cast<i64>(info & 0xffffffu);
        const u32 d = (info >> 24) & 15u;
        const i64 t = (info >> 28) & 1u ? ci.t_prog : ci.t_read;
        i64 cur = die[0];
#pragma unroll
        for (int j = 1; j < D; ++j) cur = d == static_cast<u32>(j) ? die[j] : cur;
        chan = imax(chan, cur) + x;
        const i64 done = chan + t;
#pragma unroll
        for (int j = 0; j < D; ++j)
            if (d == static_cast<u32>(j)) die[j] = done;
    }
};

// Replay of one channel's shifted segment [first, last) in 32-bit words
// relative to a base B: the same max-plus steps on one-instruction integer
// max and add, so each step's dependency chain is a few cycles instead of
// the 64-bit compare/select sequences.  The D die words live in shared
// memory during the loop (`sd`: word j at sd[j * kThreads], one column per
// thread, so a warp's accesses never share a bank): a step reads and writes
// its die's word directly instead of selecting among D registers.
//   REAL   arrivals from sarr (non-decreasing in a sorted batch); otherwise
//          the arrival is -inf (the unit columns of pass 1).
//   WRITE  each completion tick goes back to sarr[k] (pass 2).
// B = max(first arrival, chan): every max of the segment has an operand
// >= B (an arrival, or chan, which never decreases), so state words below
// B cannot win and are clamped to -1; a word that is still -1 at the end
// was not touched and keeps its 64-bit value.  When the queue runs more
// than 2^30 ahead of the first arrival, the segment's arrivals must all be
// at or below B (then none of them wins and the unit step is exact);
// otherwise the function declines.  Every word stays below
// hi + (n + 1) * step_max, hi the largest starting word or arrival above B
// and step_max a bound on one access's transfer plus die time; when that is
// not below 2^31 the function returns false with `reg` unchanged and the
// caller replays in 64 bits.
template <bool ARR, bool WRITE>
__device__ __forceinline__ void rel32_loop(int& rc, int* sd, i64* sarr, const u32* sinfo,
                                           u32 first, u32 last, i64 B, int t_read, int t_prog)
{
    // operands one step ahead; index `last` <= T + C - 1 stays inside the
    // sorted arrays
    i64 a_next = ARR ? sarr[first] : 0;
    u32 info_next = sinfo[first];
#pragma unroll 4
    for (u32 k = first; k < last; ++k) {
        const i64 a64 = a_next;
        const u32 info = info_next;
        if (ARR) a_next = sarr[k + 1];
        info_next = sinfo[k + 1];
        const int x = static_cast<int>(info & 0xffffffu);
        int* slot = sd + ((info >> 24) & 15u) * kThreadsDie;
        const int t = (info >> 28) & 1u ? t_prog : t_read;
        const int cur = *slot;
        if (ARR) rc = max(max(static_cast<int>(a64 - B), rc), cur) + x;
        else rc = max(rc, cur) + x;
        const int done = rc + t;
        *slot = done;
        if (WRITE) sarr[k] = B + done;
    }
}

// The same steps with the D die words in registers (a select chain reads
// the step's die word, predicated moves write it): more instructions per
// step, but no shared-memory round trip on the loop-carried path.  Pass 2,
// whose chains run on a quarter of the CTA's threads while the rest wait,
// is bound by that path; pass 1, whose chains share the SMs with other
// CTAs' decoding, by instructions.
template <int D, bool ARR, bool WRITE>
__device__ __forceinline__ void rel32_loop_regs(int& rc, int (&rd)[D], i64* sarr,
                                                const u32* sinfo, u32 first, u32 last, i64 B,
                                                int t_read, int t_prog)
{
    i64 a_next = ARR ? sarr[first] : 0;
    u32 info_next = sinfo[first];
#pragma unroll 4
    for (u32 k = first; k < last; ++k) {
        const i64 a64 = a_next;
        const u32 info = info_next;
        if (ARR) a_next = sarr[k + 1];
        info_next = sinfo[k + 1];
        const int x = static_cast<int>(info & 0xffffffu);
        const u32 d = (info >> 24) & 15u;
        const int t = (info >> 28) & 1u ? t_prog : t_read;
        int cur = rd[0];
#pragma unroll
        for (int j = 1; j < D; ++j) cur = d == static_cast<u32>(j) ? rd[j] : cur;
        if (ARR) rc = max(max(static_cast<int>(a64 - B), rc), cur) + x;
        else rc = max(rc, cur) + x;
        const int done = rc + t;
#pragma unroll
        for (int j = 0; j < D; ++j)
            if (d == static_cast<u32>(j)) rd[j] = done;
        if (WRITE) sarr[k] = B + done;
    }
}

// SMEM: the die words in shared memory (rel32_loop) or registers
// (rel32_loop_regs; `sd` unused).
template <int D, bool REAL, bool WRITE, bool SMEM = true>
__device__ __forceinline__ bool replay_rel32(DieRegs<D>& reg, int* sd, i64* sarr,
                                             const u32* sinfo, u32 first, u32 last,
                                             const ChanInfo& ci, i64 step_max)
{
    constexpr i64 kWindow = i64{1} << 30;
    // Unit replay with the channel word at -inf (a die column before any
    // access of its die): B is the smallest finite word instead, so every
    // finite word starts at or above 0, and the -inf words start at
    // kNegWord, far enough below 0 that the segment's steps cannot bring
    // them near it (they stay -inf and keep their 64-bit value).  Nothing
    // to do when every word is -inf.
    constexpr int kNegWord = -(1 << 30);
    const bool neg_chan = !REAL && reg.chan < kNeg / 2;
    bool arrivals = REAL;
    i64 B = reg.chan, hi = 0;
    if (neg_chan) {
        i64 lo = 0;
        bool any = false;
#pragma unroll
        for (int j = 0; j < D; ++j) {
            if (reg.die[j] < kNeg / 2) continue;
            lo = any ? (reg.die[j] < lo ? reg.die[j] : lo) : reg.die[j];
            any = true;
        }
        if (!any) return true;
        if (static_cast<i64>(last - first + 1) * step_max >= (i64{1} << 29)) return false;
        B = lo;
    }
    if (REAL) {
        const i64 a_first = sarr[first], a_last = sarr[last - 1];
        B = imax(a_first, reg.chan);
        if (B - a_first >= kWindow) {
            if (a_last > B) return false;  // the arrivals overtake the queue inside the segment
            arrivals = false;
        }
        hi = a_last - B;
    }
    int rc, rd[D];
    if (neg_chan) {
        rc = kNegWord;
#pragma unroll
        for (int j = 0; j < D; ++j) {
            const bool fin = reg.die[j] >= kNeg / 2;
            const i64 v = fin ? reg.die[j] - B : 0;
            hi = imax(hi, v);
            rd[j] = fin ? static_cast<int>(v) : kNegWord;
        }
    } else {
        {
            const i64 v = reg.chan - B;
            hi = imax(hi, v);
            rc = v < 0 ? -1 : static_cast<int>(v);
        }
#pragma unroll
        for (int j = 0; j < D; ++j) {
            const i64 v = reg.die[j] - B;
            hi = imax(hi, v);
            rd[j] = v < 0 ? -1 : static_cast<int>(v);
        }
    }
    if (hi + static_cast<i64>(last - first + 1) * step_max >= (i64{1} << 31)) return false;
    const int t_read = static_cast<int>(ci.t_read), t_prog = static_cast<int>(ci.t_prog);
    if constexpr (SMEM) {
#pragma unroll
        for (int j = 0; j < D; ++j) sd[j * kThreadsDie] = rd[j];
        if (arrivals) rel32_loop<true, WRITE>(rc, sd, sarr, sinfo, first, last, B, t_read, t_prog);
        else rel32_loop<false, WRITE>(rc, sd, sarr, sinfo, first, last, B, t_read, t_prog);
#pragma unroll
        for (int j = 0; j < D; ++j) rd[j] = sd[j * kThreadsDie];
    } else {
        if (arrivals)
            rel32_loop_regs<D, true, WRITE>(rc, rd, sarr, sinfo, first, last, B, t_read, t_prog);
        else
            rel32_loop_regs<D, false, WRITE>(rc, rd, sarr, sinfo, first, last, B, t_read, t_prog);
    }
    if (rc >= 0 || !neg_chan) reg.chan = B + rc;  // a -inf channel word stays -inf
#pragma unroll
    for (int j = 0; j < D; ++j)
        if (rd[j] >= 0) reg.die[j] = B + rd[j];
    return true;
}

__device__ __forceinline__ u32 lane_id() { return threadIdx.x & 31u; }

// Exclusive scan of `count` u32 values in shared memory by warp 0.
__device__ void warp0_exclusive_scan(u32* v, u32 count, u32* total)
{
    if (threadIdx.x >= 32) return;
    u32 carry = 0;
    for (u32 base = 0; base < count; base += 32) {
        const u32 i = base + lane_id();
        const u32 x = i < count ? v[i] : 0u;
        u32 s = x;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const u32 y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane_id() >= static_cast<u32>(o)) s += y;
        }
        if (i < count) v[i] = carry + s - x;
        carry += __shfl_sync(0xffffffffu, s, 31);
    }
    if (lane_id() == 0 && total) *total = carry;
}

// Shared-memory views of one tile.
struct TileSmem {
    u64* addr;    // -> done
    u64* arr;     // -> latency
    u32* bytes;   // -> packed info (transfer ticks | die << 24 | op << 28)
    u8* op;       // -> status
    u16* ord;     // channel-sorted order of modeled accesses
    u16* key;
    u16* rank;
    u32* wcnt;    // [warps][C+1]
    u32* seg;     // [C+2] segment starts
    ChanInfo* chan;
    unsigned long long* act;  // [C*D][2]
    unsigned long long* red;
    DevRange* ranges;         // staged range table (kSmemRanges entries)
    // Direct kernel: the tile's timed accesses in channel-sorted order, with
    // channel c's segment shifted by c slots (starts at seg[c] + c) so that
    // the lanes of a chain warp, one channel each, spread over the banks.
    i64* sarr;    // max(arrival, admit); pass 2 overwrites it with done
    u32* sinfo;   // packed step info
};

constexpr u32 kSmemRanges = 32;

__device__ __forceinline__ TileSmem tile_views(unsigned char* smem, const PassArgs& A,
                                               int pass = 1)
{
    TileSmem s;
    s.sarr = reinterpret_cast<i64*>(smem + A.off_sarr[pass - 1]);
    s.sinfo = reinterpret_cast<u32*>(smem + A.off_sinfo[pass - 1]);
    s.addr = reinterpret_cast<u64*>(smem + A.off_addr);
    s.arr = reinterpret_cast<u64*>(smem + A.off_arr);
    s.bytes = reinterpret_cast<u32*>(smem + A.off_bytes);
    s.op = smem + A.off_op;
    s.ord = reinterpret_cast<u16*>(smem + A.off_ord);
    s.key = reinterpret_cast<u16*>(smem + A.off_key);
    s.rank = reinterpret_cast<u16*>(smem + A.off_rank);
    s.wcnt = reinterpret_cast<u32*>(smem + A.off_wcnt);
    s.seg = reinterpret_cast<u32*>(smem + A.off_seg);
    s.chan = reinterpret_cast<ChanInfo*>(smem + A.off_chan);
    s.act = reinterpret_cast<unsigned long long*>(smem + A.off_act);
    s.red = reinterpret_cast<unsigned long long*>(smem + A.off_red);
    s.ranges = reinterpret_cast<DevRange*>(smem + A.off_ranges);
    return s;
}

// Pass-2 statistics of one thread.
struct Stats7 {
    unsigned long long modeled = 0, bypass = 0, unsup = 0, foreign = 0, lat = 0,
                       max = 0, fast = 0;
};

// 16-byte global -> shared copies that do not pass through registers: a
// thread issues all of its copies of a tile before it waits for any, so the
// tile costs one memory round trip instead of one per loop iteration.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src)
{
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(gmem_src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all()
{
    asm volatile("cp.async.wait_all;\n" ::: "memory");
}

// Stage one tile, decode it, and build the channel-sorted order in s.ord
// with segment starts in s.seg (stable: warps own contiguous chunks, lanes
// are ranked in index order with __match_any_sync).
// FAST: one registered range, power-of-two geometry, one transfer shift, no
// activity counting and no admission delay, all known when the kernel is
// chosen.
template <int MODEL, int PASS, bool SORTED = false, bool FAST = false>
__device__ __forceinline__ void load_decode_partition(const PassArgs& A, const TileSmem& s,
                                                      u64 start, u32 nt, bool activity,
                                                      Stats7& st)
{
    const u32 tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const u32 T = A.T, C = A.C, D = A.tp.dies;
    if (nt == T && A.vec) {
        const uint4* g_addr = reinterpret_cast<const uint4*>(A.address + start);
        const uint4* g_arr = reinterpret_cast<const uint4*>(A.arrival + start);
        const uint4* g_bytes = reinterpret_cast<const uint4*>(A.bytes + start);
        const uint4* g_op = reinterpret_cast<const uint4*>(A.op + start);
        uint4* d_addr = reinterpret_cast<uint4*>(s.addr);
        uint4* d_arr = reinterpret_cast<uint4*>(s.arr);
        uint4* d_bytes = reinterpret_cast<uint4*>(s.bytes);
        uint4* d_op = reinterpret_cast<uint4*>(s.op);
#pragma unroll 1
        for (u32 k = tid; k < T / 2; k += kThreads) {
            cp_async16(d_addr + k, g_addr + k);
            cp_async16(d_arr + k, g_arr + k);
        }
#pragma unroll 1
        for (u32 k = tid; k < T / 4; k += kThreads) cp_async16(d_bytes + k, g_bytes + k);
        for (u32 k = tid; k < T / 16; k += kThreads) cp_async16(d_op + k, g_op + k);
        cp_async_commit();
        cp_async_wait_all();
    } else {
        for (u32 k = tid; k < nt; k += kThreads) {
            s.addr[k] = A.address[start + k];
            s.arr[k] = A.arrival[start + k];
            s.bytes[k] = A.bytes[start + k];
            s.op[k] = A.op[start + k];
        }
    }
    for (u32 k = tid; k < kWarps * (C + 1); k += kThreads) s.wcnt[k] = 0;
    __syncthreads();

    DecodeParams dp = A.dp;
    if (dp.range_count <= kSmemRanges) dp.ranges = s.ranges;
    const bool single = A.dp.one.valid != 0;
    const u32 chunk = T / kWarps;
    bool unsorted = false;
    u64 arr_max = 0;  // arrivals from 2^59 on take the sequential kernel
    // the arrival before this tile (previous tile, or the previous batch)
    const u64 tile_prev = PASS == 1 && warp == 0 && lane == 0
                              ? (start > 0 ? A.arrival[start - 1] : *A.last_arrival)
                              : 0;
    for (u32 j = 0; j < chunk; j += 32) {
        const u32 e = warp * chunk + j + lane;
        u32 key = C;
        const u64 arr = e < nt ? s.arr[e] : 0;
        if (PASS == 1) {
            // previous arrival: the element before this one in the staged tile
            // (for the tile's first, the arrival before the tile)
            const u64 prev = e > 0 ? (e <= nt ? s.arr[e - 1] : 0) : tile_prev;
            if (e < nt && arr < prev) unsorted = true;
            if (!FAST) arr_max = arr > arr_max ? arr : arr_max;
        }
        if (e < nt) {
            const u64 a = s.addr[e];
            const u32 b = s.bytes[e];
            const u32 o = s.op[e];
            TimingDecoded d;
            if (MODEL == kModelDie) {
                d = FAST ? classify_single<true>(A.dp.one, A.dp, a, b, o)
                    : single ? classify_single(A.dp.one, A.dp, a, b, o)
                             : classify_timing(dp, a, b, o);
            } else {
                const Decoded f = classify_decode(dp, a, b, o, false);
                d = TimingDecoded{f.status, 0u, 0u};
            }
            u32 info = (o & 1u) << 28;
            if (d.status == kModeled) {
                key = MODEL == kModelDie ? d.local : 0u;
                if (MODEL == kModelDie) {
                    const u32 xs = A.tp.x_shift;
                    const u64 x =
                        FAST || xs != kXDivide
                            ? static_cast<u64>(static_cast<u32>(
                                  (static_cast<u64>(b) + ((u64{1} << xs) - 1)) >> xs)) *
                                  A.tp.time_scale
                            : transfer_ticks(b, s.chan[key], A.tp.time_scale);
                    if (x > 0xffffffull) atomicOr(A.error, kErrNeedSeq);
                    info |= static_cast<u32>(x & 0xffffffull) | (d.die << 24);
                    if (!FAST && activity) {
                        if (o) atomicAdd(&s.act[2 * (key * D + d.die) + 1], 1ull);
                        else atomicAdd(&s.act[2 * (key * D + d.die)],
                                       static_cast<unsigned long long>(b));
                    }
                }
                if (PASS == 2) ++st.modeled;
            } else if (PASS == 2) {
                s.addr[e] = arr;  // done = arrival
                s.arr[e] = 0;     // latency 0
                if (d.status == kBypass) ++st.bypass;
                else if (d.status == kForeign) ++st.foreign;
                else ++st.unsup;
            }
            s.bytes[e] = info;
            s.op[e] = static_cast<u8>(d.status);
            s.key[e] = static_cast<u16>(key);
        }
    }
    __syncwarp();
    // rank the warp's chunk 32 accesses at a time, in index order
    for (u32 j = 0; j < chunk; j += 32) {
        const u32 e = warp * chunk + j + lane;
        const u32 key = e < nt ? static_cast<u32>(s.key[e]) : C;
        const u32 peers = __match_any_sync(0xffffffffu, key);
        const u32 before = __popc(peers & ((1u << lane) - 1u));
        const u32 base = s.wcnt[warp * (C + 1) + key];
        __syncwarp();
        if (before == 0) s.wcnt[warp * (C + 1) + key] = base + __popc(peers);
        if (e < nt) s.rank[e] = static_cast<u16>(base + before);
        __syncwarp();
    }
    if (PASS == 1 && unsorted && !A.tp.any_order) atomicOr(A.error, kErrUnsorted);
    // FAST batches must follow the arrival order (or are refused as
    // unsorted), so the tile's last arrival is its largest
    if (FAST && PASS == 1 && tid == 0 && nt > 0) arr_max = s.arr[nt - 1];
    if (PASS == 1 && arr_max >= kArrivalLimit) atomicOr(A.error, kErrNeedSeq);
    __syncthreads();

    // segment offsets: key-major, warp-minor
    for (u32 c = tid; c < C; c += kThreads) {
        u32 total = 0;
        for (u32 w = 0; w < kWarps; ++w) total += s.wcnt[w * (C + 1) + c];
        s.seg[c] = total;
    }
    __syncthreads();
    warp0_exclusive_scan(s.seg, C, &s.seg[C]);
    __syncthreads();
    for (u32 c = tid; c < C; c += kThreads) {
        u32 running = s.seg[c];
        for (u32 w = 0; w < kWarps; ++w) {
            const u32 cnt = s.wcnt[w * (C + 1) + c];
            s.wcnt[w * (C + 1) + c] = running;
            running += cnt;
        }
    }
    __syncthreads();
    for (u32 j = 0; j < chunk; j += 32) {
        const u32 e = warp * chunk + j + lane;
        if (e < nt) {
            const u32 key = s.key[e];
            if (SORTED) {
                // the shifted channel-sorted copy that the chains read, and
                // the access's record for pass 2 (format at record_slot)
                const u32 pos = key < C ? s.wcnt[warp * (C + 1) + key] + s.rank[e] : 0u;
                const u32 info = s.bytes[e];
                if (key < C) {
                    s.sinfo[pos + key] = info;
                    // FAST: every admission tick is 0 and arrivals are below 2^59
                    s.sarr[pos + key] = FAST ? static_cast<i64>(s.arr[e])
                                             : imax(static_cast<i64>(s.arr[e]), s.chan[key].admit);
                }
                __stcs(reinterpret_cast<unsigned long long*>(A.latency + start + e),
                       static_cast<u64>(info) | (static_cast<u64>(pos) << 32) |
                           (static_cast<u64>(s.op[e]) << 48) |
                           (static_cast<u64>(key & 0xffu) << 56));
            } else if (key < C) {
                s.ord[s.wcnt[warp * (C + 1) + key] + s.rank[e]] = static_cast<u16>(e);
            }
        }
    }
    __syncthreads();
}

__device__ __forceinline__ void store_tile(const PassArgs& A, const TileSmem& s, u64 start,
                                           u32 nt)
{
    const u32 tid = threadIdx.x, T = A.T;
    if (nt == T && A.vec) {
        uint4* g_done = reinterpret_cast<uint4*>(A.done + start);
        uint4* g_lat = reinterpret_cast<uint4*>(A.latency + start);
        uint4* g_st = reinterpret_cast<uint4*>(A.status + start);
        const uint4* d_done = reinterpret_cast<const uint4*>(s.addr);
        const uint4* d_lat = reinterpret_cast<const uint4*>(s.arr);
        const uint4* d_st = reinterpret_cast<const uint4*>(s.op);
        for (u32 k = tid; k < T / 2; k += kThreads) {
            __stcs(g_done + k, d_done[k]);
            __stcs(g_lat + k, d_lat[k]);
        }
        for (u32 k = tid; k < T / 16; k += kThreads) __stcs(g_st + k, d_st[k]);
    } else {
        for (u32 k = tid; k < nt; k += kThreads) {
            A.done[start + k] = s.addr[k];
            A.latency[start + k] = s.arr[k];
            A.status[start + k] = s.op[k];
        }
    }
}

// Compact per-access records that pass 1 of the direct kernel leaves for
// pass 2 in the caller's latency buffer (written by the sorted partition in
// load_decode_partition; overwritten by pass 2 with the latency):
//            bits 0-31  packed step info of access j (transfer | die | op),
//            bits 32-47 channel-sorted position of access j,
//            bits 48-55 status of access j,
//            bits 56-63 local channel of access j (C < 256 in direct mode).
// Pass 2 rebuilds the tile's partition from them without decoding again.
__device__ __forceinline__ u32 record_slot(u64 r)
{
    return static_cast<u32>((r >> 32) & 0xffffu) + static_cast<u32>(r >> 56);
}

// Block-reduce the pass-2 statistics and the die activity; one atomic each
// per CTA.
__device__ __forceinline__ void flush_stats(const PassArgs& A, const TileSmem& s,
                                            const Stats7& st, bool activity)
{
    const u32 tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const u32 C = A.C, D = A.tp.dies;
    if (activity) {
        for (u32 k = tid; k < C * D; k += kThreads) {
            if (s.act[2 * k]) atomicAdd(&A.tp.die_read_bytes[k], s.act[2 * k]);
            if (s.act[2 * k + 1]) atomicAdd(&A.tp.die_writes[k], s.act[2 * k + 1]);
        }
    }
    unsigned long long vals[7] = {st.modeled, st.bypass, st.unsup, st.foreign,
                                  st.lat, st.max, st.fast};
#pragma unroll
    for (int k = 0; k < 7; ++k) {
        unsigned long long v = vals[k];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long y = __shfl_down_sync(0xffffffffu, v, o);
            v = k == 5 ? (y > v ? y : v) : v + y;
        }
        if (lane == 0) s.red[k * kWarps + warp] = v;
    }
    __syncthreads();
    if (tid < 7) {
        unsigned long long v = 0;
        for (u32 w = 0; w < kWarps; ++w) {
            const unsigned long long y = s.red[tid * kWarps + w];
            v = tid == 5 ? (y > v ? y : v) : v + y;
        }
        unsigned long long* dst = &A.counters->modeled;
        if (tid == 5) atomicMax(&A.counters->max_done, v);
        else if (v) atomicAdd(tid == 6 ? &A.counters->fast_modeled_ns : dst + tid, v);
    }
}

__device__ __forceinline__ void prologue(const PassArgs& A, const TileSmem& s, bool die,
                                         bool activity, bool stage_ranges = true)
{
    const u32 tid = threadIdx.x, C = A.C, D = A.tp.dies;
    for (u32 c = tid; c < C; c += kThreads) s.chan[c] = stage_channel(A.tp, c, die);
    if (stage_ranges && A.dp.range_count <= kSmemRanges)
        for (u32 k = tid; k < A.dp.range_count; k += kThreads) s.ranges[k] = A.dp.ranges[k];
    if (activity)
        for (u32 k = tid; k < 2 * C * D; k += kThreads) s.act[k] = 0;
    if (blockIdx.x == 0 && A.state_in) {
        // the parallel path needs every carried tick below 2^59
        for (u32 k = tid; k < C * A.K; k += kThreads)
            if (A.state_in[k] >= kArrivalLimit) atomicOr(A.error, kErrNeedSeq);
    }
}

// ---------------------------------------------------------------------------
// Piece kernel: generic K; channel segments are cut into pieces of <= L
// accesses whose max-plus matrices are built by replaying each column.
template <int MODEL, int PASS>
__global__ void __launch_bounds__(kThreads, 2)
timing_pass_kernel(const PassArgs args)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const PassArgs& A = args;
    const u32 tid = threadIdx.x;
    const u32 T = A.T, L = A.L, C = A.C, K = A.K;
    const TileSmem s = tile_views(smem, A);
    u32* s_pbase = reinterpret_cast<u32*>(smem + A.off_pbase); // [C+2]
    u16* s_pchan = reinterpret_cast<u16*>(smem + A.off_pchan);
    i64* s_pm = reinterpret_cast<i64*>(smem + A.off_pm);       // [P][K][K+1]
    i64* s_pin = reinterpret_cast<i64*>(smem + A.off_pin);     // [P][K]
    i64* s_die = reinterpret_cast<i64*>(smem + A.off_die);     // [D][threads]

    if (PASS == 2 && *A.error != 0) return;  // pass 1 refused or rerouted the batch
    const u32 KK = K + 1;
    const bool activity = PASS == 2 && MODEL == kModelDie && A.tp.die_read_bytes != nullptr;
    if (PASS == 1) prologue(A, s, MODEL == kModelDie, false);
    else prologue(A, s, MODEL == kModelDie, activity);

    i64* agg = A.agg + static_cast<u64>(blockIdx.x) * C * K * KK;
    i64* carry = A.incoming + static_cast<u64>(blockIdx.x) * C * K;
    if (PASS == 1) {
        for (u32 k = tid; k < C * K * KK; k += kThreads) {  // identity map
            const u32 col = k % KK, row = (k / KK) % K;
            agg[k] = col == row ? 0 : kNeg;
        }
    }
    __syncthreads();
    Stats7 st;

    const u64 tile_first = static_cast<u64>(blockIdx.x) * A.tiles_per_cta;
    for (u32 tt = 0; tt < A.tiles_per_cta; ++tt) {
        const u64 start = (tile_first + tt) * T;
        if (start >= A.n) break;
        const u32 nt = static_cast<u32>(A.n - start < T ? A.n - start : T);
        load_decode_partition<MODEL, PASS>(A, s, start, nt, activity, st);

        for (u32 c = tid; c < C; c += kThreads) s_pbase[c] = (s.seg[c + 1] - s.seg[c] + L - 1) / L;
        __syncthreads();
        warp0_exclusive_scan(s_pbase, C, &s_pbase[C]);
        __syncthreads();
        for (u32 c = tid; c < C; c += kThreads)
            for (u32 p = s_pbase[c]; p < s_pbase[c + 1]; ++p) s_pchan[p] = static_cast<u16>(c);
        __syncthreads();

        for (u32 cg0 = 0; cg0 < C; cg0 += A.group_channels) {
            const u32 cg1 = cg0 + A.group_channels < C ? cg0 + A.group_channels : C;
            const u32 p0 = s_pbase[cg0];
            const u32 np = s_pbase[cg1] - p0;
            if (np == 0) continue;

            // phase A: column r of piece p = replay from unit state e_r
            for (u32 q = tid; q < np * KK; q += kThreads) {
                const u32 pl = q % np, r = q / np;
                const u32 pg = p0 + pl;
                const u32 c = s_pchan[pg];
                const u32 first = s.seg[c] + (pg - s_pbase[c]) * L;
                const u32 seg_end = s.seg[c + 1];
                const u32 last = first + L < seg_end ? first + L : seg_end;
                const ChanInfo ci = s.chan[c];
                i64 chan = r == 0 ? 0 : kNeg;
                i64* die = s_die + tid;
                for (u32 j = 1; j < K; ++j) die[(j - 1) * kThreads] = r == j ? 0 : kNeg;
                const bool real = r == K;
                for (u32 k = first; k < last; ++k) {
                    const u32 e = s.ord[k];
                    const i64 a = real ? imax(static_cast<i64>(s.arr[e]), ci.admit) : kNeg;
                    StepModel<MODEL>::step(chan, die, kThreads, a, s.bytes[e], ci, A.tp);
                }
                i64* col = s_pm + static_cast<u64>(pl) * K * KK + r;
                col[0] = chan;
                for (u32 j = 1; j < K; ++j) col[j * KK] = die[(j - 1) * kThreads];
            }
            __syncthreads();

            if (PASS == 1) {
                // fold this group's pieces into R_b, one thread per (c, r)
                for (u32 q = tid; q < (cg1 - cg0) * KK; q += kThreads) {
                    const u32 c = cg0 + q / KK, r = q % KK;
                    if (s_pbase[c] == s_pbase[c + 1]) continue;
                    i64 v[17];
                    i64* col = agg + static_cast<u64>(c) * K * KK + r;
                    for (u32 i = 0; i < K; ++i) v[i] = col[i * KK];
                    v[K] = r == K ? 0 : kNeg;
                    for (u32 pg = s_pbase[c]; pg < s_pbase[c + 1]; ++pg) {
                        const i64* M = s_pm + static_cast<u64>(pg - p0) * K * KK;
                        i64 w[16];
                        for (u32 i = 0; i < K; ++i) {
                            i64 best = kNeg;  // clamp: -inf stays -inf
                            for (u32 j = 0; j <= K; ++j) best = imax(best, M[i * KK + j] + v[j]);
                            w[i] = best;
                        }
                        for (u32 i = 0; i < K; ++i) v[i] = w[i];
                    }
                    for (u32 i = 0; i < K; ++i) col[i * KK] = v[i];
                }
                __syncthreads();
            } else {
                // propagate the carried state through the pieces
                for (u32 c = cg0 + tid; c < cg1; c += kThreads) {
                    i64 v[17];
                    i64* cv = carry + static_cast<u64>(c) * K;
                    for (u32 i = 0; i < K; ++i) v[i] = cv[i];
                    v[K] = 0;
                    for (u32 pg = s_pbase[c]; pg < s_pbase[c + 1]; ++pg) {
                        i64* pin = s_pin + static_cast<u64>(pg - p0) * K;
                        for (u32 i = 0; i < K; ++i) pin[i] = v[i];
                        const i64* M = s_pm + static_cast<u64>(pg - p0) * K * KK;
                        i64 w[16];
                        for (u32 i = 0; i < K; ++i) {
                            i64 best = kNeg;
                            for (u32 j = 0; j <= K; ++j) best = imax(best, M[i * KK + j] + v[j]);
                            w[i] = best;
                        }
                        for (u32 i = 0; i < K; ++i) v[i] = w[i];
                    }
                    for (u32 i = 0; i < K; ++i) cv[i] = v[i];
                }
                __syncthreads();
                // phase C: replay every piece from its exact incoming state
                for (u32 pl = tid; pl < np; pl += kThreads) {
                    const u32 pg = p0 + pl;
                    const u32 c = s_pchan[pg];
                    const u32 first = s.seg[c] + (pg - s_pbase[c]) * L;
                    const u32 seg_end = s.seg[c + 1];
                    const u32 last = first + L < seg_end ? first + L : seg_end;
                    const ChanInfo ci = s.chan[c];
                    const i64* pin = s_pin + static_cast<u64>(pl) * K;
                    i64 chan = pin[0];
                    i64* die = s_die + tid;
                    for (u32 j = 1; j < K; ++j) die[(j - 1) * kThreads] = pin[j];
                    for (u32 k = first; k < last; ++k) {
                        const u32 e = s.ord[k];
                        const u32 info = s.bytes[e];
                        const u64 arr = s.arr[e];
                        const i64 a = imax(static_cast<i64>(arr), ci.admit);
                        const i64 done = StepModel<MODEL>::step(chan, die, kThreads, a,
                                                                info, ci, A.tp);
                        const u64 ud = static_cast<u64>(done);
                        s.addr[e] = ud;
                        s.arr[e] = ud - arr;
                        st.lat += ud - arr;
                        st.max = ud > st.max ? ud : st.max;
                        if (MODEL == kModelFast)
                            st.fast += (info >> 28) & 1u ? A.tp.fast_service_prog
                                                         : A.tp.fast_service_read;
                    }
                }
                __syncthreads();
            }
        }
        if (PASS == 2) store_tile(A, s, start, nt);
        __syncthreads();
    }
    if (PASS == 2) flush_stats(A, s, st, activity);
}

// ---------------------------------------------------------------------------
// Direct kernels (die model, D dies known at compile time, enough channels
// for parallelism): no pieces.  Pass 1 is direct_pass_kernel<1, D, FAST>
// (FAST: the decode specialized for one range, power-of-two geometry, one
// transfer shift, no activity counting and no admission delay), pass 2
// direct_replay_kernel<D, NOADMIT> below.
//
// Pass 1: item (r, c) carries column r of channel c's range aggregate.  Items
// are laid out r-major so that a warp holds one kind of column.  Column 0
// (channel unit) and column K (real arrivals) are replayed over the whole
// range.  A die column r = 1..D is replayed only until it couples to column
// 0: equal to it plus one scalar delta in every finite component and -inf
// exactly where column 0 is.  From then on it stays so -- the homogeneous
// max-plus maps of later accesses commute with adding a scalar -- and only
// delta is kept; the warps whose columns have all coupled skip their loops.
__device__ __forceinline__ bool is_neg_inf(i64 v) { return v < kNeg / 2; }

template <int D>
__device__ __forceinline__ bool try_couple(const i64* col0, const DieRegs<D>& v, i64& delta)
{
    bool have = false;
    i64 dl = 0;
#pragma unroll
    for (int i = 0; i <= D; ++i) {
        const i64 a = col0[i];
        const i64 b = i == 0 ? v.chan : v.die[i - 1];
        const bool ia = is_neg_inf(a), ib = is_neg_inf(b);
        if (ia != ib) return false;
        if (ia) continue;
        if (!have) {
            dl = b - a;
            have = true;
        } else if (b - a != dl) {
            return false;
        }
    }
    if (!have) return false;
    delta = dl;
    return true;
}

// Tiles after which the die columns try to couple to column 0: each of the
// first 8 (short ranges couple early), then every 8th.  Coupling may be
// tested at any tile boundary; testing less often only replays more tiles.
__device__ __forceinline__ bool couple_now(u32 tt) { return tt < 8 || (tt & 7u) == 7u; }

// The column items of one CTA's range aggregate (pass 1 of the direct
// path): thread tid holds items q = tid and tid + kThreads of the C x (K+1)
// (r-major) column array.
template <int D>
struct ColumnItems {
    static constexpr int kItems = 2;
    static constexpr u32 K = D + 1, KK = D + 2;
    DieRegs<D> reg[kItems];
    u32 item_c[kItems], item_r[kItems], item_p[kItems];
    bool item_on[kItems], coupled[kItems];
    i64 delta[kItems];

    // parts = 2: each channel's segment is split in the middle (the first
    // half rounded up), and each half is a range of its own (one tile per
    // CTA, 2 C (K+1) <= kThreads items)
    __device__ __forceinline__ void init(u32 C, u32 parts = 1)
    {
#pragma unroll
        for (int it = 0; it < kItems; ++it) {
            const u32 q = threadIdx.x + it * kThreads;
            item_on[it] = q < parts * C * KK;
            item_p[it] = q / (C * KK);
            item_r[it] = q % (C * KK) / C;
            item_c[it] = q % C;
            coupled[it] = false;
            delta[it] = 0;
            if (!item_on[it]) continue;
            // identity column e_r (r == K: no constant yet)
            reg[it].chan = item_r[it] == 0 ? 0 : kNeg;
#pragma unroll
            for (int j = 0; j < D; ++j)
                reg[it].die[j] = item_r[it] == static_cast<u32>(j + 1) ? 0 : kNeg;
        }
    }

    // Replay the tile's channel-sorted segments into the items' columns
    // (`mid`: each channel's split point, with parts = 2).
    __device__ __forceinline__ void replay(const TileSmem& s, int* sd, bool rel32,
                                           i64 step_max, const u32* mid = nullptr)
    {
#pragma unroll
        for (int it = 0; it < kItems; ++it) {
            if (!item_on[it] || coupled[it]) continue;
            const u32 c = item_c[it];
            u32 first = s.seg[c] + c, last = s.seg[c + 1] + c;  // shifted segment
            if (mid) {
                if (item_p[it] == 0) last = mid[c] + c;
                else first = mid[c] + c;
            }
            if (first == last) continue;
            const ChanInfo ci = s.chan[c];
            if (item_r[it] == K) {
                if (rel32 && replay_rel32<D, true, false>(reg[it], sd, s.sarr, s.sinfo, first,
                                                          last, ci, step_max))
                    continue;
#pragma unroll 4
                for (u32 k = first; k < last; ++k) reg[it].step(s.sarr[k], s.sinfo[k], ci);
            } else {
                // unit columns: column 0 and the die columns not yet coupled
                // (a die column whose channel word is still -inf declines)
                if (rel32 && replay_rel32<D, false, false>(reg[it], sd, s.sarr, s.sinfo, first,
                                                           last, ci, step_max))
                    continue;
#pragma unroll 4
                for (u32 k = first; k < last; ++k) reg[it].step_unit(s.sinfo[k], ci);
            }
        }
    }

    // Snapshot column 0 into s_col0, then let the die columns try to couple
    // to it.  Called by every thread (contains barriers).
    __device__ __forceinline__ void couple(i64* s_col0, u32 C)
    {
#pragma unroll
        for (int it = 0; it < kItems; ++it) {
            if (!item_on[it] || item_r[it] != 0) continue;
            i64* v0 = s_col0 + static_cast<u64>(item_p[it] * C + item_c[it]) * K;
            v0[0] = reg[it].chan;
#pragma unroll
            for (int j = 0; j < D; ++j) v0[1 + j] = reg[it].die[j];
        }
        __syncthreads();
#pragma unroll
        for (int it = 0; it < kItems; ++it) {
            if (!item_on[it] || coupled[it] || item_r[it] == 0 || item_r[it] == K) continue;
            coupled[it] = try_couple<D>(
                s_col0 + static_cast<u64>(item_p[it] * C + item_c[it]) * K, reg[it], delta[it]);
        }
        __syncthreads();
    }

    // Write the CTA's range aggregates (agg: the first of them, parts of C
    // channels each); s_col0 holds column 0 after the last tile of the range.
    __device__ __forceinline__ void write(i64* agg, const i64* s_col0, u32 C) const
    {
#pragma unroll
        for (int it = 0; it < kItems; ++it) {
            if (!item_on[it]) continue;
            const u32 c = item_c[it], r = item_r[it], pc = item_p[it] * C + c;
            i64* col = agg + static_cast<u64>(pc) * K * KK + r;
            if (coupled[it]) {
                const i64* v0 = s_col0 + static_cast<u64>(pc) * K;
#pragma unroll
                for (int i = 0; i <= D; ++i)
                    col[i * KK] = is_neg_inf(v0[i]) ? kNeg : v0[i] + delta[it];
            } else {
                col[0] = reg[it].chan;
#pragma unroll
                for (int j = 0; j < D; ++j) col[(j + 1) * KK] = reg[it].die[j];
            }
        }
    }
};

template <int PASS, int D, bool FAST>
__global__ void __launch_bounds__(kThreads, 3)
direct_pass_kernel(const PassArgs args)
{
    static_assert(PASS == 1, "pass 2 of the direct path is direct_replay_kernel");
    extern __shared__ __align__(16) unsigned char smem[];
    const PassArgs& A = args;
    const u32 tid = threadIdx.x;
    constexpr u32 K = D + 1, KK = D + 2;
    const u32 T = A.T, C = A.C;
    const TileSmem s = tile_views(smem, A, 1);
    i64* s_col0 = reinterpret_cast<i64*>(smem + A.off_pm);  // [C][K]
    // activity is counted where the access sizes are decoded (pass 1) and
    // staged until the range scan accepts the batch
    const bool activity = !FAST && A.tp.act_stage != nullptr;
    prologue(A, s, true, activity, true);

    ColumnItems<D> items;
    items.init(C);
    i64* agg = A.agg + static_cast<u64>(blockIdx.x) * C * K * KK;
    int* sd = reinterpret_cast<int*>(smem + A.off_dies[0]) + tid;
    __syncthreads();
    Stats7 st;
    // 32-bit relative chains need arrivals that do not decrease (a batch
    // that must follow the arrival order; pass 1 refuses it otherwise)
    const bool rel32 = !A.tp.any_order && A.tp.step_max > 0;

    const u64 tile_first = static_cast<u64>(blockIdx.x) * A.tiles_per_cta;
    for (u32 tt = 0; tt < A.tiles_per_cta; ++tt) {
        const u64 start = (tile_first + tt) * T;
        if (start >= A.n) break;
        const u32 nt = static_cast<u32>(A.n - start < T ? A.n - start : T);
        load_decode_partition<kModelDie, 1, true, FAST>(A, s, start, nt, activity, st);
        items.replay(s, sd, rel32, A.tp.step_max);
        __syncthreads();
        // at the tiles couple_now picks and after the last: snapshot column 0,
        // then let the die columns try to couple to it
        if (!couple_now(tt) && tt + 1 < A.tiles_per_cta && start + T < A.n) continue;
        items.couple(s_col0, C);
    }
    items.write(agg, s_col0, C);
    if (activity)
        for (u32 k = tid; k < 2 * C * D; k += kThreads)
            if (s.act[k]) atomicAdd(&A.tp.act_stage[k], s.act[k]);
}

// ---------------------------------------------------------------------------
// Pass 1 of the direct path for the common case -- one registered range,
// power-of-two geometry, one transfer shift, no activity counting and no
// admission delay (the conditions of direct_pass_kernel's FAST instantiation)
// -- restructured around the issue rate, which bounds that kernel:
//   * the tile size is a compile-time 2048 (8 rounds of 32 accesses per
//     warp), so every per-access loop unrolls and its shared-memory loads
//     issue together instead of one round trip per iteration;
//   * decode and warp ranking are one loop, and each access's channel, rank
//     and status stay in registers until the sorted copy (no key / rank
//     arrays in shared memory; the step info overwrites the staged size);
//   * the segment offsets take two barriers (warp-shuffle scan of the
//     per-channel totals) instead of four;
//   * the channel-sorted copy has buffers of its own (layout_fast), so the
//     next tile's inputs stream into the staging buffers while the chains
//     run;
//   * the decode drops what the host has proven for this context: a page's
//     transfer times the scale fits the 24-bit field (the host sends the
//     batch to the sequential kernel otherwise), and every admission tick
//     is 0.
// Outputs and aggregates are identical to direct_pass_kernel's, and so is
// every record field pass 2 reads (the step info of an untimed access is 0
// here).
constexpr u32 kFastTile = 2048;
constexpr u32 kFastRounds = kFastTile / kThreads;  // rounds of 32 per warp

template <int D, bool GENERAL = false>
__global__ void __launch_bounds__(kThreads, 3)
direct_fast_kernel(const PassArgs args)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const PassArgs& A = args;
    const u32 tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    constexpr u32 K = D + 1, KK = D + 2, T = kFastTile;
    const u32 C = A.C;
    const TileSmem s = tile_views(smem, A, 1);
    i64* s_col0 = reinterpret_cast<i64*>(smem + A.off_pm);  // [C][K]
    u32* s_part = reinterpret_cast<u32*>(s.red);            // per-warp channel totals
    // Stage tile [start, start + nt): full aligned tiles by cp.async (all
    // copies in flight before any wait), others by plain copies.
    auto stage = [&](u64 start, u32 nt) {
        if (nt == T && A.vec) {
            const uint4* g_addr = reinterpret_cast<const uint4*>(A.address + start);
            const uint4* g_arr = reinterpret_cast<const uint4*>(A.arrival + start);
            const uint4* g_bytes = reinterpret_cast<const uint4*>(A.bytes + start);
            const uint4* g_op = reinterpret_cast<const uint4*>(A.op + start);
#pragma unroll
            for (u32 k = tid; k < T / 2; k += kThreads) {
                cp_async16(reinterpret_cast<uint4*>(s.addr) + k, g_addr + k);
                cp_async16(reinterpret_cast<uint4*>(s.arr) + k, g_arr + k);
            }
#pragma unroll
            for (u32 k = tid; k < T / 4; k += kThreads)
                cp_async16(reinterpret_cast<uint4*>(s.bytes) + k, g_bytes + k);
            if (tid < T / 16) cp_async16(reinterpret_cast<uint4*>(s.op) + tid, g_op + tid);
            cp_async_commit();
        } else {
            for (u32 k = tid; k < nt; k += kThreads) {
                s.addr[k] = A.address[start + k];
                s.arr[k] = A.arrival[start + k];
                s.bytes[k] = A.bytes[start + k];
                s.op[k] = A.op[start + k];
            }
        }
    };
    auto tile_size = [&](u64 start) -> u32 {
        return static_cast<u32>(A.n - start < T ? A.n - start : T);
    };
    // the CTA's first tile streams in while the prologue runs
    const u64 tile_first = static_cast<u64>(blockIdx.x) * A.tiles_per_cta;
    if (tile_first * T < A.n) stage(tile_first * T, tile_size(tile_first * T));
    // GENERAL with several ranges: the range records in shared memory
    // (layout_fast reserves them when the batch has at most kSmemRanges)
    const bool smem_ranges = GENERAL && A.off_ranges != 0;
    prologue(A, s, true, false, smem_ranges);
    DecodeParams dpl = A.dp;
    if (smem_ranges) dpl.ranges = s.ranges;
    // GENERAL: the activity of this tile (layout_fast puts it beside the
    // per-warp counts), flushed to the staging counters per tile
    const bool activity = GENERAL && A.tp.act_stage != nullptr;
    unsigned long long* act = reinterpret_cast<unsigned long long*>(smem + A.off_act);

    // halves: one tile per CTA, two ranges (the tile's halves) per CTA
    const u32 parts = A.halves ? 2u : 1u;
    u32* s_mid = A.halves ? reinterpret_cast<u32*>(smem + A.off_mid) : nullptr;
    ColumnItems<D> items;
    items.init(C, parts);
    i64* agg = A.agg + static_cast<u64>(blockIdx.x) * parts * C * K * KK;
    const bool rel32 = !A.tp.any_order && A.tp.step_max > 0;
    const SingleRange rg = A.dp.one;
    const u32 lanes_below = (1u << lane) - 1u;
    int* sd = reinterpret_cast<int*>(smem + A.off_dies[0]) + tid;
    u32* wc = s.wcnt + warp * (C + 1);
    __syncthreads();
    // GENERAL at odd channel rates: each channel's transfer ticks of the
    // power-of-two access sizes, so that those take no division
    u32* xtab = GENERAL && A.off_xtab && A.tp.x_shift == kXDivide
                    ? reinterpret_cast<u32*>(smem + A.off_xtab) : nullptr;
    if (xtab) {
        for (u32 k = tid; k < C * kXTabSizes; k += kThreads) {
            const u64 x = transfer_ticks(1u << (kXTabMin + k % kXTabSizes), s.chan[k / kXTabSizes],
                                         A.tp.time_scale);
            xtab[k] = x > 0xffffffffull ? 0xffffffffu : static_cast<u32>(x);
        }
        __syncthreads();
    }

    for (u32 tt = 0; tt < A.tiles_per_cta; ++tt) {
        const u64 start = (tile_first + tt) * T;
        if (start >= A.n) break;
        const u32 nt = tile_size(start);
        // GENERAL: the chains' die words overlay the staged addresses, so
        // later tiles are staged here, not during the previous chains
        if (GENERAL && tt > 0) stage(start, nt);
        for (u32 k = lane; k <= C; k += 32) wc[k] = 0;
        if (activity)
            for (u32 k = tid; k < 2 * C * D; k += kThreads) act[k] = 0;
        const u64 tile_prev = tid == 0 ? (start > 0 ? A.arrival[start - 1] : *A.last_arrival) : 0;
        cp_async_wait_all();
        __syncthreads();

        // ---- decode and rank, 8 rounds of 32 accesses per warp
        u32 kr[kFastRounds];   // channel key | status << 8 | rank in warp << 16
        bool unsorted = false;
#pragma unroll
        for (u32 j = 0; j < kFastRounds; ++j) {
            const u32 e = warp * (T / kWarps) + j * 32 + lane;
            u32 key = C, status = kUnsupported, info = 0;
            u32 act_slot = 0xffffffffu, act_add = 0;  // GENERAL: activity counter, amount
            if (e < nt) {
                const u64 a = s.addr[e];
                const u64 arr = s.arr[e];
                const u64 prev = e > 0 ? s.arr[e - 1] : tile_prev;
                unsorted |= arr < prev;
                const u32 b = s.bytes[e];
                const u32 o = s.op[e];
                if (GENERAL) {
                    // the general classification (ranges read through the
                    // cache), the channel's own transfer rate, activity
                    const TimingDecoded d = rg.valid ? classify_single(rg, A.dp, a, b, o)
                                                     : classify_timing(dpl, a, b, o);
                    status = d.status;
                    if (d.status == kModeled) {
                        key = d.local;
                        const u32 xs = A.tp.x_shift;
                        const u32 k = __ffs(b) - 1 - kXTabMin;  // a power-of-two size's slot
                        const u64 x = xs != kXDivide
                                          ? static_cast<u64>(static_cast<u32>(
                                                (static_cast<u64>(b) + ((u64{1} << xs) - 1)) >> xs)) *
                                                A.tp.time_scale
                                      : xtab && (b & (b - 1)) == 0 && k < kXTabSizes
                                          ? static_cast<u64>(xtab[key * kXTabSizes + k])
                                          : transfer_ticks(b, s.chan[key], A.tp.time_scale);
                        if (x > 0xffffffull) atomicOr(A.error, kErrNeedSeq);
                        info = static_cast<u32>(x & 0xffffffull) | d.die << 24 | (o & 1u) << 28;
                        act_slot = 2 * (key * D + d.die) + (o & 1u);
                        act_add = o & 1u ? 1u : b;
                    }
                } else {
                    const u64 off = a - rg.base;  // wraps when a < base
                    if (b == 0) {                 // hbf_device.cu:997-1003
                    } else if (off >= rg.length) {
                        // below the range: unsupported if it straddles into it
                        status = a < rg.base && a <= ~u64{0} - b && rg.base < a + b
                                     ? kUnsupported : kBypass;
                    } else if (o <= 1 && ((rg.allowed >> o) & 1u) && b <= rg.length - off &&
                               (off & rg.page_mask) + b <= rg.page_mask + 1) {
                        const u32 u =
                            static_cast<u32>((rg.file_offset + off) >> A.dp.stripe_shift);
                        const u32 g = (u >> A.dp.chan_shift) & A.dp.chan_mask;
                        if ((g & A.dp.shard_mask) == A.dp.shard_rank) {
                            status = kModeled;
                            key = g >> A.dp.shard_shift;
                            const u32 xs = A.tp.x_shift;
                            info = ((b + ((1u << xs) - 1u)) >> xs) * A.tp.time_scale |
                                   ((u >> A.dp.die_shift) & A.dp.die_mask) << 24 | (o & 1u) << 28;
                        } else {
                            status = kForeign;
                        }
                    }
                }
            }
            if (activity) {
                // one shared-memory atomic per group of lanes with the same
                // counter (runs of accesses to one die would otherwise
                // serialize on it), carrying the group's sum (a page's
                // bytes times 32 at most: no overflow)
                const u64 tag = static_cast<u64>(act_add) << 32 | act_slot;
                const u32 same = __match_any_sync(0xffffffffu, tag);
                if (act_slot != 0xffffffffu && (same & lanes_below) == 0)
                    atomicAdd(&act[act_slot], static_cast<unsigned long long>(act_add) *
                                                   static_cast<unsigned long long>(__popc(same)));
            }
            const u32 peers = __match_any_sync(0xffffffffu, key);
            const u32 before = __popc(peers & lanes_below);
            const u32 base = wc[key];
            __syncwarp();
            if (before == 0) wc[key] = base + __popc(peers);
            __syncwarp();
            kr[j] = key | status << 8 | (base + before) << 16;
            if (e < nt) s.bytes[e] = info;  // step info (transfer | die << 24 | op << 28)
        }
        if (unsorted && !A.tp.any_order) atomicOr(A.error, kErrUnsorted);
        if (tid == 0 && s.arr[nt - 1] >= kArrivalLimit) atomicOr(A.error, kErrNeedSeq);
        __syncthreads();

        // ---- segment offsets: channel c's segment starts after every
        // smaller channel's accesses; within it, warp w's accesses follow
        // the earlier warps'.
        {
            const u32 c = tid;
            u32 tot = 0;
            u32 pre[kWarps];
            if (c < C) {
#pragma unroll
                for (u32 w = 0; w < kWarps; ++w) {
                    pre[w] = tot;
                    tot += s.wcnt[w * (C + 1) + c];
                }
            }
            u32 incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const u32 y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= static_cast<u32>(o)) incl += y;
            }
            if (lane == 31) s_part[warp] = incl;
            __syncthreads();
            if (c < C) {
                u32 offset = incl - tot;
                for (u32 w = 0; w < warp; ++w) offset += s_part[w];
#pragma unroll
                for (u32 w = 0; w < kWarps; ++w) s.wcnt[w * (C + 1) + c] = offset + pre[w];
                s.seg[c] = offset;
                if (c == C - 1) s.seg[C] = offset + tot;
                // the split point: the middle of the channel's segment
                if (s_mid) s_mid[c] = offset + (tot + 1) / 2;
            }
            __syncthreads();
        }

        // ---- channel-sorted copy (segment c shifted by c slots) and the
        // per-access records for pass 2 (format at record_slot)
#pragma unroll
        for (u32 j = 0; j < kFastRounds; ++j) {
            const u32 e = warp * (T / kWarps) + j * 32 + lane;
            if (e >= nt) continue;
            const u32 key = kr[j] & 0xffu;
            const u32 info = s.bytes[e];
            u32 pos = 0;
            if (key < C) {
                pos = wc[key] + (kr[j] >> 16);
                s.sinfo[pos + key] = info;
                s.sarr[pos + key] = GENERAL ? imax(static_cast<i64>(s.arr[e]), s.chan[key].admit)
                                            : static_cast<i64>(s.arr[e]);
            }
            __stcs(reinterpret_cast<unsigned long long*>(A.latency + start + e),
                   static_cast<u64>(info) | static_cast<u64>(pos) << 32 |
                       static_cast<u64>((kr[j] >> 8) & 0xffu) << 48 |
                       static_cast<u64>(key) << 56);
        }
        __syncthreads();

        // ---- the staging buffers are free: stream the next tile in while
        // the chains run
        const u64 next = start + T;
        if (!GENERAL && tt + 1 < A.tiles_per_cta && next < A.n) stage(next, tile_size(next));
        if (activity)
            for (u32 k = tid; k < 2 * C * D; k += kThreads)
                if (act[k]) atomicAdd(&A.tp.act_stage[k], act[k]);
        items.replay(s, sd, rel32, A.tp.step_max, s_mid);
        __syncthreads();
        if (!couple_now(tt) && tt + 1 < A.tiles_per_cta && start + T < A.n) continue;
        items.couple(s_col0, C);
    }
    items.write(agg, s_col0, C);
}

// ---------------------------------------------------------------------------
// Direct replay (pass 2 of the direct kernel), streamed.  Thread c < C
// carries channel c's exact state through the CTA's tiles.  Per tile: the
// staged records and arrivals are unpacked into the shifted channel-sorted
// copy (and each access's slot in it); statuses and the outputs of untimed
// accesses go straight out.  Then -- while the chains run and the outputs are
// written -- the next tile's records and arrivals stream into the staging
// buffers with cp.async.  The outputs of timed accesses are written in access
// order (coalesced), their arrival re-read from global memory (in L2).

// Stage tile [start, start + nt) (records from the latency buffer, arrivals):
// asynchronously when the tile is full and the buffers are 16-byte aligned.
__device__ __forceinline__ void stage_records(const PassArgs& A, const TileSmem& s, u64 start,
                                              u32 nt)
{
    const u32 tid = threadIdx.x, T = A.T;
    const u64* rec = A.latency + start;
    if (nt == T && A.vec) {
        const uint4* g_arr = reinterpret_cast<const uint4*>(A.arrival + start);
        const uint4* g_rec = reinterpret_cast<const uint4*>(rec);
        uint4* d_arr = reinterpret_cast<uint4*>(s.arr);
        uint4* d_rec = reinterpret_cast<uint4*>(s.addr);
        for (u32 k = tid; k < T / 2; k += kThreads) {
            cp_async16(d_arr + k, g_arr + k);
            cp_async16(d_rec + k, g_rec + k);
        }
        cp_async_commit();
    } else {
        for (u32 k = tid; k < nt; k += kThreads) {
            s.arr[k] = A.arrival[start + k];
            s.addr[k] = rec[k];
        }
    }
}

constexpr u32 kOutBatch = 8;  // tiles hold at most 2048 = 8 x kThreads accesses

template <int D, bool NOADMIT, bool HALVES = false, bool WALK = false>
__global__ void __launch_bounds__(kThreads, 3)
direct_replay_kernel(const PassArgs args)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const PassArgs& A = args;
    const u32 tid = threadIdx.x;
    constexpr u32 K = D + 1;
    const u32 T = A.T, C = A.C;
    const TileSmem s = tile_views(smem, A, 2);
    u16* slot_of = reinterpret_cast<u16*>(smem + A.off_slot);  // access -> sorted slot
    int* sd = nullptr;  // pass 2 keeps its chains' die words in registers
    if (const u32 err = *A.error) {
        // pass 1 refused the batch, or rerouted it to the exact sequential
        // walk; WALK (small batches, where a launch of its own costs as much
        // as the pass): CTA 0 runs that walk here, one thread per channel
        if (WALK && !(err & kErrUnsorted) && (err & kErrNeedSeq) && blockIdx.x == 0 && tid < C)
            sequential_walk<kModelDie>(A.dp, A.tp, A.address, A.bytes, A.op, A.arrival, A.done,
                                       A.latency, A.status, A.n, K, A.state_in, A.state_out,
                                       const_cast<u64*>(A.last_arrival), A.counters, tid);
        return;
    }
    prologue(A, s, true, false, false);

    // halves: threads c and C + c replay the first and second half of
    // channel c's segment of the (one) tile, each from its own incoming state
    constexpr u32 parts = HALVES ? 2u : 1u;
    DieRegs<D> reg;
    const bool chain = tid < parts * C;
    if (chain) {
        const i64* cv = A.incoming + (static_cast<u64>(blockIdx.x) * parts * C + tid) * K;
        reg.chan = cv[0];
#pragma unroll
        for (int j = 0; j < D; ++j) reg.die[j] = cv[1 + j];
    }
    Stats7 st;
    const bool rel32 = !A.tp.any_order && A.tp.step_max > 0;  // see direct_pass_kernel
    const u64 tile_first = static_cast<u64>(blockIdx.x) * A.tiles_per_cta;
    auto tile_size = [&](u64 start) -> u32 {
        return static_cast<u32>(A.n - start < T ? A.n - start : T);
    };
    if (tile_first * T < A.n) stage_records(A, s, tile_first * T, tile_size(tile_first * T));
    for (u32 tt = 0; tt < A.tiles_per_cta; ++tt) {
        const u64 start = (tile_first + tt) * T;
        if (start >= A.n) break;
        const u32 nt = tile_size(start);
        cp_async_wait_all();
        for (u32 c = tid; c <= C; c += kThreads) s.seg[c] = 0;
        __syncthreads();
        // unpack: sorted copy, access -> slot, statuses, untimed outputs
        for (u32 j = tid; j < nt; j += kThreads) {
            const u64 r = s.addr[j];
            const u64 arr = s.arr[j];
            const u32 status = static_cast<u32>(r >> 48) & 0xffu;
            A.status[start + j] = static_cast<u8>(status);
            if (status == kModeled) {
                const u32 k = record_slot(r);
                s.sinfo[k] = static_cast<u32>(r);
                // NOADMIT: every admission tick is 0 (arrivals are below 2^59)
                s.sarr[k] = NOADMIT ? static_cast<i64>(arr)
                                    : imax(static_cast<i64>(arr), s.chan[r >> 56].admit);
                slot_of[j] = static_cast<u16>(k);
                atomicAdd(&s.seg[r >> 56], 1u);
                ++st.modeled;
            } else {
                slot_of[j] = 0xffffu;
                __stcs(reinterpret_cast<unsigned long long*>(A.done + start + j), arr);
                __stcs(reinterpret_cast<unsigned long long*>(A.latency + start + j), 0ull);
                if (status == kBypass) ++st.bypass;
                else if (status == kForeign) ++st.foreign;
                else ++st.unsup;
            }
        }
        __syncthreads();
        warp0_exclusive_scan(s.seg, C, &s.seg[C]);
        __syncthreads();
        // the staging buffers are free: stream the next tile in
        const u64 next = start + T;
        if (tt + 1 < A.tiles_per_cta && next < A.n) stage_records(A, s, next, tile_size(next));
        const u32 c = HALVES ? tid % C : tid, part = HALVES ? tid / C : 0u;
        u32 first = chain ? s.seg[c] + c : 0u, last = chain ? s.seg[c + 1] + c : 0u;
        if (HALVES && chain) {
            // the middle of the channel's segment, as pass 1 split it
            const u32 mid = s.seg[c] + (s.seg[c + 1] - s.seg[c] + 1) / 2 + c;
            if (part == 0) last = mid;
            else first = mid;
        }
        const ChanInfo ci = chain ? s.chan[c] : ChanInfo{};
        if (first < last &&
            !(rel32 && replay_rel32<D, true, true, false>(reg, sd, s.sarr, s.sinfo, first, last, ci,
                                                   A.tp.step_max))) {
            // operands one step ahead; index `last` <= T + C - 1 stays inside
            // the sorted arrays
            i64 a_next = s.sarr[first];
            u32 info_next = s.sinfo[first];
#pragma unroll 4
            for (u32 k = first; k < last; ++k) {
                const i64 a = a_next;
                const u32 info = info_next;
                a_next = s.sarr[k + 1];
                info_next = s.sinfo[k + 1];
                s.sarr[k] = reg.step(a, info, ci);
            }
        }
        __syncthreads();
        // outputs of the timed accesses, in access order.  Their arrivals
        // come from L2 (the staging buffer already holds the next tile): a
        // thread loads a batch of them before it stores anything, so the
        // loads overlap instead of each waiting behind the previous stores.
        for (u32 j0 = tid; j0 < nt; j0 += kOutBatch * kThreads) {
            u64 arr[kOutBatch];
            u32 slot[kOutBatch];
#pragma unroll
            for (u32 i = 0; i < kOutBatch; ++i) {
                const u32 j = j0 + i * kThreads;
                slot[i] = j < nt ? slot_of[j] : 0xffffu;
                arr[i] = slot[i] != 0xffffu
                             ? __ldcg(reinterpret_cast<const unsigned long long*>(A.arrival) +
                                      start + j)
                             : 0ull;
            }
#pragma unroll
            for (u32 i = 0; i < kOutBatch; ++i) {
                if (slot[i] == 0xffffu) continue;
                const u32 j = j0 + i * kThreads;
                const u64 done = static_cast<u64>(s.sarr[slot[i]]);
                const u64 lat = done - arr[i];
                __stcs(reinterpret_cast<unsigned long long*>(A.done + start + j), done);
                __stcs(reinterpret_cast<unsigned long long*>(A.latency + start + j), lat);
                st.lat += lat;
                st.max = done > st.max ? done : st.max;
            }
        }
        // the next iteration's barrier keeps the sorted copy until this is done
    }
    flush_stats(A, s, st, false);
}

// Range scan: incoming_b = R_{b-1} ... R_0 (state), one CTA per local
// channel (channels are independent); range_scan_lb_kernel below replaces
// it whenever a channel's ranges fit 32 groups of 32.  Each range aggregate
// R is a max-plus affine map x -> max(R[:, :K] + x, R[:, K]) (K state
// words).  The CTA's 32 warps split the ranges into 32 groups, one each:
//   A  each warp composes its group into one map (one lane per entry,
//      clamping sums below -2^61 back to NEG so that they cannot overflow);
//   B  warp 0 applies the 32 group maps to the carried state, giving each
//      group its incoming state (and the batch's final state);
//   C  each warp walks its group from that state (lane i = state word i,
//      shuffles), writing every range's incoming state.
// Aggregates are staged per warp in chunks of `chunk` with coalesced loads.
// When the batch is accepted the CTA also adds the activity pass 1 staged
// for its channel to the die counters.
struct ScanArgs {
    const i64* agg;     // [ctas][C][K][K+1]
    i64* incoming;      // [ctas][C][K]
    const u64* state_in;
    u64* state_out;
    const u32* error;
    u64* last_arrival;
    const u64* arrival;
    u64 n;
    u32 ctas, C, K;
    u32 chunk;          // aggregates staged per warp per round
    u32 dies;
    DevCounters* counters;
    const unsigned long long* act_stage;  // [C*D][2] or null
    unsigned long long* die_read_bytes;
    unsigned long long* die_writes;
};

constexpr u32 kScanWarps = 32;

// 8-byte global -> shared copy (cp.async.ca; both addresses 8-byte aligned).
__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gmem_src)
{
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst), "l"(gmem_src));
}

// A warp stages nb consecutive range aggregates of channel c.  The copies
// do not pass through registers, so all of them are in flight before the
// one wait (a load-then-store loop waits one memory round trip per
// iteration: the compiler cannot move a load above the previous store).
__device__ __forceinline__ void stage_aggregates(const ScanArgs& a, u32 c, u32 b0, u32 nb,
                                                 u32 per, i64* stage)
{
    const u32 lane = threadIdx.x & 31u;
    for (u32 b = 0; b < nb; ++b) {
        const i64* src = a.agg + (static_cast<u64>(b0 + b) * a.C + c) * per;
        for (u32 w = lane; w < per; w += 32) cp_async8(stage + b * per + w, src + w);
    }
    cp_async_commit();
    cp_async_wait_all();
    __syncwarp();
}

__global__ void __launch_bounds__(kScanWarps * 32) range_scan_kernel(const ScanArgs a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const u32 tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const u32 c = blockIdx.x, K = a.K, KK = K + 1, per = K * KK;
    const u32 err = *a.error;
    if (!(err & kErrUnsorted) && (err & kErrNeedSeq)) return;  // sequential path
    const u64 row0 = static_cast<u64>(c) * K;
    if (err & kErrUnsorted) {  // refused: keep the state
        for (u32 k = tid; k < K; k += blockDim.x) a.state_out[row0 + k] = a.state_in[row0 + k];
        if (c == 0 && tid == 0) {
            atomicAdd(&a.counters->errors, 1ull);
            atomicOr(&a.counters->error_code, static_cast<unsigned long long>(err));
        }
        return;
    }
    const u32 n = a.ctas, span = a.chunk * per + per;
    i64* stage = reinterpret_cast<i64*>(smem) + static_cast<u64>(warp) * span;
    i64* comp = stage + static_cast<u64>(a.chunk) * per;  // the group's composite
    i64* gin = reinterpret_cast<i64*>(smem) + static_cast<u64>(kScanWarps) * span;  // [warps][K]
    const u32 g0 = static_cast<u32>(static_cast<u64>(n) * warp / kScanWarps);
    const u32 g1 = static_cast<u32>(static_cast<u64>(n) * (warp + 1) / kScanWarps);

    // A: comp = R_{g1-1} o ... o R_{g0}
    for (u32 b0 = g0; b0 < g1; b0 += a.chunk) {
        const u32 nb = g1 - b0 < a.chunk ? g1 - b0 : a.chunk;
        stage_aggregates(a, c, b0, nb, per, stage);
        for (u32 b = 0; b < nb; ++b) {
            const i64* R = stage + static_cast<u64>(b) * per;
            if (b0 == g0 && b == 0) {
                for (u32 e = lane; e < per; e += 32) comp[e] = R[e];
                __syncwarp();
                continue;
            }
            i64 v[9];
#pragma unroll
            for (u32 t = 0; t < 9; ++t) {
                const u32 e = lane + 32 * t;
                if (e >= per) break;
                const u32 i = e / KK, j = e - i * KK;
                const i64* Ri = R + static_cast<u64>(i) * KK;
                i64 best = j == K ? Ri[K] : kNeg;
                for (u32 k = 0; k < K; ++k) best = imax(best, Ri[k] + comp[k * KK + j]);
                v[t] = best < kNeg / 2 ? kNeg : best;
            }
            __syncwarp();
#pragma unroll
            for (u32 t = 0; t < 9; ++t) {
                const u32 e = lane + 32 * t;
                if (e >= per) break;
                comp[e] = v[t];
            }
            __syncwarp();
        }
    }
    __syncthreads();

    // B: incoming state of every group, and the batch's final state
    const u32 my_row = lane < K ? lane : 0u;
    if (warp == 0) {
        i64 x = lane < K ? static_cast<i64>(a.state_in[row0 + lane]) : 0;
        for (u32 w = 0; w < kScanWarps; ++w) {
            if (lane < K) gin[w * K + lane] = x;
            const u32 s0 = static_cast<u32>(static_cast<u64>(n) * w / kScanWarps);
            const u32 s1 = static_cast<u32>(static_cast<u64>(n) * (w + 1) / kScanWarps);
            if (s0 == s1) continue;
            const i64* G = reinterpret_cast<i64*>(smem) + static_cast<u64>(w) * span +
                           static_cast<u64>(a.chunk) * per + static_cast<u64>(my_row) * KK;
            i64 best = G[K];
            for (u32 j = 0; j < K; ++j) best = imax(best, G[j] + __shfl_sync(0xffffffffu, x, j));
            if (lane < K) x = best;
        }
        if (lane < K) a.state_out[row0 + lane] = static_cast<u64>(x);
    }
    __syncthreads();

    // C: every range's incoming state
    i64 x = lane < K ? gin[warp * K + lane] : 0;
    for (u32 b0 = g0; b0 < g1; b0 += a.chunk) {
        const u32 nb = g1 - b0 < a.chunk ? g1 - b0 : a.chunk;
        __syncwarp();  // the previous chunk is consumed
        stage_aggregates(a, c, b0, nb, per, stage);
        for (u32 b = 0; b < nb; ++b) {
            if (lane < K) a.incoming[(static_cast<u64>(b0 + b) * a.C + c) * K + lane] = x;
            const i64* row = stage + static_cast<u64>(b) * per + static_cast<u64>(my_row) * KK;
            i64 best = row[K];
            for (u32 j = 0; j < K; ++j) best = imax(best, row[j] + __shfl_sync(0xffffffffu, x, j));
            if (lane < K) x = best;
        }
    }
    if (a.act_stage) {
        const u32 D = a.dies;
        for (u32 d = tid; d < D; d += blockDim.x) {
            const u64 k = static_cast<u64>(c) * D + d;
            a.die_read_bytes[k] += a.act_stage[2 * k];
            a.die_writes[k] += a.act_stage[2 * k + 1];
        }
    }
    if (c == 0 && tid == 0) {
        if (a.n) *a.last_arrival = a.arrival[a.n - 1];
        atomicAdd(&a.counters->batches, 1ull);
    }
}

// ---------------------------------------------------------------------------
// Range scan over several CTAs per channel (decoupled look-back).  CTA
// (group g, channel c) -- taken in ticket order, so every group it waits on
// is already running -- owns ranges [g R, (g + 1) R) of channel c, R =
// kLbWarps * m, m per warp:
//   A  each warp composes its m range maps (kept staged for C);
//   P  the warps' maps form an inclusive prefix (Hillis-Steele, 3 rounds);
//      the last is the group's map, published as an aggregate (flag 1);
//   L  warp 0 reads the flags of the preceding groups of channel c at once
//      (one lane per group, at most 31), starts from the nearest group that
//      published its outgoing state (flag 2; before group 0, the carried
//      state) and applies the published maps of the groups after it, fetched
//      together: the group's incoming state; it publishes its own outgoing
//      state (flag 2);
//   C  each warp applies the prefix of the warps before it and walks its
//      ranges, writing every range's incoming state.
// Flags live at a fixed address and are cleared by the last CTA to finish;
// waits are bounded (a wait error is counted and the scan goes on).
constexpr u32 kLbWarps = 8;
constexpr u32 kLbRangesPerWarp = 4;
constexpr u32 kLbRanges = kLbWarps * kLbRangesPerWarp;  // ranges per group
constexpr u32 kLbSpins = 1u << 22;
constexpr u32 kLbMaxGroups = 32;  // groups of one channel (the look-back window)

struct LbScanArgs {
    i64* gmap;     // [groups][C][K][K+1] published group maps
    i64* gstate;   // [groups][C][K] published outgoing states
    u32* ctr;      // ticket and done counters, then the flags [groups][C]: 0, 1 map,
    u32 groups;    //   2 outgoing state (zero between scans)
};

// Out = Post o Pre (Pre first) for maps x -> max(M[:, :K] + x, M[:, K]),
// one warp, entries strided over the lanes; sums below -2^61 clamp to NEG.
__device__ __forceinline__ void compose_maps(i64* out, const i64* post, const i64* pre, u32 K)
{
    const u32 lane = threadIdx.x & 31u, KK = K + 1, per = K * KK;
    i64 v[3];
#pragma unroll
    for (u32 t = 0; t < 3; ++t) {
        const u32 e = lane + 32 * t;
        v[t] = 0;
        if (e >= per) continue;
        const u32 i = e / KK, j = e - i * KK;
        const i64* Pi = post + static_cast<u64>(i) * KK;
        i64 best = j == K ? Pi[K] : kNeg;
        for (u32 k = 0; k < K; ++k) best = imax(best, Pi[k] + pre[k * KK + j]);
        v[t] = best < kNeg / 2 ? kNeg : best;
    }
    __syncwarp();
#pragma unroll
    for (u32 t = 0; t < 3; ++t) {
        const u32 e = lane + 32 * t;
        if (e < per) out[e] = v[t];
    }
    __syncwarp();
}

// x -> M(x), lane i < K holding word i (all lanes call)
__device__ __forceinline__ i64 apply_map(const i64* M, i64 x, u32 K)
{
    const u32 lane = threadIdx.x & 31u, row = lane < K ? lane : 0u;
    const i64* r = M + static_cast<u64>(row) * (K + 1);
    i64 best = r[K];
    for (u32 j = 0; j < K; ++j) best = imax(best, r[j] + __shfl_sync(0xffffffffu, x, j));
    return lane < K ? best : x;
}

__device__ __forceinline__ void identity_map(i64* M, u32 K)
{
    const u32 lane = threadIdx.x & 31u, KK = K + 1;
    for (u32 e = lane; e < K * KK; e += 32) {
        const u32 i = e / KK, j = e - i * KK;
        M[e] = i == j ? 0 : kNeg;
    }
    __syncwarp();
}

__global__ void __launch_bounds__(kLbWarps * 32) range_scan_lb_kernel(const ScanArgs a,
                                                                      const LbScanArgs b)
{
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ u32 s_ticket, s_last;
    const u32 tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const u32 K = a.K, KK = K + 1, per = K * KK, C = a.C;
    const u32 err = *a.error;
    if (!(err & kErrUnsorted) && (err & kErrNeedSeq)) return;  // sequential path
    if (err & kErrUnsorted) {  // refused: keep the state
        for (u32 c = blockIdx.x; c < C; c += gridDim.x)
            for (u32 k = tid; k < K; k += blockDim.x)
                a.state_out[static_cast<u64>(c) * K + k] = a.state_in[static_cast<u64>(c) * K + k];
        if (blockIdx.x == 0 && tid == 0) {
            atomicAdd(&a.counters->errors, 1ull);
            atomicOr(&a.counters->error_code, static_cast<unsigned long long>(err));
        }
        return;
    }
    u32* ticket = b.ctr;
    u32* flags = b.ctr + 2;
    if (tid == 0) s_ticket = atomicAdd(ticket, 1u);
    __syncthreads();
    const u32 t = s_ticket;
    const u32 g = t / C, c = t % C;
    i64* stage = reinterpret_cast<i64*>(smem) + static_cast<u64>(warp) * kLbRangesPerWarp * per;
    i64* pm = reinterpret_cast<i64*>(smem) + static_cast<u64>(kLbWarps) * kLbRangesPerWarp * per;
    i64* pm2 = pm + static_cast<u64>(kLbWarps) * per;        // prefix double buffer
    i64* maps = pm2 + static_cast<u64>(kLbWarps) * per;      // look-back: fetched maps
    i64* gin = maps + static_cast<u64>(kLbMaxGroups - 1) * per;  // [warps][K] incoming states
    const u32 n = a.ctas;
    const u32 w0 = g * kLbRanges + warp * kLbRangesPerWarp;
    const u32 w1 = w0 + kLbRangesPerWarp < n ? w0 + kLbRangesPerWarp : n;
    const u32 nb = w0 < n ? w1 - w0 : 0u;
    bool failed = false;

    // A: the warp's map R_{w1-1} o ... o R_{w0}
    if (nb) stage_aggregates(a, c, w0, nb, per, stage);
    i64* mine = pm + static_cast<u64>(warp) * per;
    if (nb == 0) {
        identity_map(mine, K);
    } else {
        for (u32 e = lane; e < per; e += 32) mine[e] = stage[e];
        __syncwarp();
        for (u32 k = 1; k < nb; ++k) compose_maps(mine, stage + static_cast<u64>(k) * per, mine, K);
    }
    __syncthreads();
    // P: inclusive prefix over the warps
    i64 *cur = pm, *nxt = pm2;
    for (u32 d = 1; d < kLbWarps; d <<= 1) {
        i64* o = nxt + static_cast<u64>(warp) * per;
        const i64* m = cur + static_cast<u64>(warp) * per;
        if (warp >= d) {
            compose_maps(o, m, cur + static_cast<u64>(warp - d) * per, K);
        } else {
            for (u32 e = lane; e < per; e += 32) o[e] = m[e];
            __syncwarp();
        }
        __syncthreads();
        i64* sw = cur;
        cur = nxt;
        nxt = sw;
    }
    const i64* group_map = cur + static_cast<u64>(kLbWarps - 1) * per;
    u32* my_flag = flags + g * C + c;
    // L: the group's incoming state
    if (warp == 0) {
        i64 x = 0;
        if (g == 0) {
            x = lane < K ? static_cast<i64>(a.state_in[static_cast<u64>(c) * K + lane]) : 0;
        } else {
            i64* slot = b.gmap + (static_cast<u64>(g) * C + c) * per;
            for (u32 e = lane; e < per; e += 32) slot[e] = group_map[e];
            __syncwarp();
            if (lane == 0) {
                __threadfence();
                atomicExch(my_flag, 1u);
            }
            // the window of preceding groups (at most 31): lane k watches
            // group g - 1 - k, and a lane before group 0 stands for the
            // carried state; the nearest group that published its
            // outgoing state starts the walk, the maps of the groups after
            // it are fetched at once and applied in order
            const int j = static_cast<int>(g) - 1 - static_cast<int>(lane);
            u32 fv = 2;
            if (j >= 0) {
                const volatile u32* f = flags + static_cast<u32>(j) * C + c;
                fv = *f;
                for (u32 spins = 0; fv == 0 && spins < kLbSpins; ++spins) {
                    __nanosleep(32);
                    fv = *f;
                }
            }
            __threadfence();  // the published words after the flags
            failed = __any_sync(0xffffffffu, fv == 0);
            const u32 have = __ballot_sync(0xffffffffu, fv == 2);
            const u32 kstar = failed ? 31u : static_cast<u32>(__ffs(have)) - 1u;
            const int jstar = failed ? -1 : static_cast<int>(g) - 1 - static_cast<int>(kstar);
            if (lane < K)
                x = jstar >= 0 ? __ldcg(b.gstate + (static_cast<u64>(jstar) * C + c) * K + lane)
                               : static_cast<i64>(a.state_in[static_cast<u64>(c) * K + lane]);
            const u32 count = failed ? 0u : kstar;  // groups jstar + 1 .. g - 1
            // all of their maps in flight before one wait: one L2 round trip
            // instead of one per word the lane copies, which had made this
            // fetch the slowest step of the scan's late groups.  16-byte
            // copies (a map is K (K + 1) words, an even count) when the maps
            // start on a 16-byte boundary; the static entry's scratch may put
            // them 8 bytes off it, and plain loads take that case.
            if ((reinterpret_cast<std::uintptr_t>(b.gmap) & 15u) == 0) {
                const u32 halves = per / 2;
                for (u32 w = lane; w < count * halves; w += 32) {
                    const u32 q = w / halves, e = 2 * (w - q * halves);
                    cp_async16(maps + static_cast<u64>(q) * per + e,
                               b.gmap + ((static_cast<u64>(jstar) + 1 + q) * C + c) * per + e);
                }
                cp_async_commit();
                cp_async_wait_all();
            } else {
                for (u32 w = lane; w < count * per; w += 32) {
                    const u32 q = w / per, e = w - q * per;
                    maps[w] = __ldcg(b.gmap + ((static_cast<u64>(jstar) + 1 + q) * C + c) * per + e);
                }
            }
            __syncwarp();
            for (u32 q = 0; q < count; ++q) x = apply_map(maps + static_cast<u64>(q) * per, x, K);
        }
        if (lane < K) gin[lane] = x;
        // outgoing state of the group
        const i64 out = apply_map(group_map, x, K);
        if (lane < K) b.gstate[(static_cast<u64>(g) * C + c) * K + lane] = out;
        __syncwarp();
        if (lane == 0) {
            __threadfence();
            atomicExch(my_flag, 2u);
        }
        if ((g + 1) * kLbRanges >= n && lane < K) a.state_out[static_cast<u64>(c) * K + lane] = out;
        if (failed && lane == 0) {
            atomicAdd(&a.counters->errors, 1ull);
            atomicOr(&a.counters->error_code, static_cast<unsigned long long>(kErrWait));
        }
    }
    __syncthreads();
    // C: every range's incoming state
    {
        i64 x = lane < K ? gin[lane] : 0;
        if (warp > 0) x = apply_map(cur + static_cast<u64>(warp - 1) * per, x, K);
        for (u32 k = 0; k < nb; ++k) {
            if (lane < K) a.incoming[(static_cast<u64>(w0 + k) * C + c) * K + lane] = x;
            x = apply_map(stage + static_cast<u64>(k) * per, x, K);
        }
    }
    if (g == 0 && a.act_stage) {
        const u32 D = a.dies;
        for (u32 d = tid; d < D; d += blockDim.x) {
            const u64 k = static_cast<u64>(c) * D + d;
            a.die_read_bytes[k] += a.act_stage[2 * k];
            a.die_writes[k] += a.act_stage[2 * k + 1];
        }
    }
    if (t == 0 && tid == 0) {
        if (a.n) *a.last_arrival = a.arrival[a.n - 1];
        atomicAdd(&a.counters->batches, 1ull);
    }
    // the last CTA to finish clears the flags and counters for the next scan
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(ticket + 1, 1u) == b.groups * C - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (s_last) {
        for (u32 k = tid; k < b.groups * C; k += blockDim.x) flags[k] = 0;
        if (tid == 0) {
            ticket[0] = 0;
            ticket[1] = 0;
        }
    }
}

// Exact sequential fallback with the reference's saturating unsigned
// arithmetic, for batches whose ticks may approach 2^64.  One thread per
// local channel walks the whole batch in order.
struct SeqArgs {
    DecodeParams dp;
    TimingParams tp;
    const u64* address;
    const u32* bytes;
    const u8* op;
    const u64* arrival;
    u64* done;
    u64* latency;
    u8* status;
    u64 n;
    u32 C, K;
    const u64* state_in;
    u64* state_out;
    u32* error;
    u64* last_arrival;
    DevCounters* counters;
};

template <int MODEL>
__global__ void sequential_kernel(const SeqArgs a)
{
    const u32 c = blockIdx.x * blockDim.x + threadIdx.x;
    const u32 flags = *a.error;
    if ((flags & kErrUnsorted) || !(flags & kErrNeedSeq) || c >= a.C) return;
    sequential_walk<MODEL>(a.dp, a.tp, a.address, a.bytes, a.op, a.arrival, a.done, a.latency,
                           a.status, a.n, a.K, a.state_in, a.state_out, a.last_arrival,
                           a.counters, c);
}

// Decode-only kernel (A1 + A2), one thread per access.
struct DecodeOut {
    u64 media_address;
    u64 page;
    u32 status;
    u32 range_index;
    u32 stack;
    u32 channel;
    u32 die;
    u32 plane;
};
static_assert(sizeof(DecodeOut) == 40, "decoded record layout");

__global__ void decode_kernel(const DecodeParams p, const u64* address,
                              const u32* bytes, const u8* op, u64 n,
                              DecodeOut* out)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const Decoded d = classify_decode(p, address[i], bytes[i], op[i], true);
    DecodeOut o{};
    o.status = d.status;
    o.range_index = d.range_index;
    o.media_address = d.media;
    if (d.status == kModeled || d.status == kForeign) {
        o.page = d.page;
        o.stack = d.stack;
        o.channel = d.channel;
        o.die = d.die;
        o.plane = d.plane;
    }
    out[i] = o;
}

// ---------------------------------------------------------------- host side
struct Launch {
    PassArgs pass;
    u32 ctas;
    u32 smem_bytes;
};

static u32 align_up(u32 v, u32 a) { return (v + a - 1) / a * a; }

// Shared-memory layout for a tile of T accesses with C channels, K words.
// Piece mode: one layout for both passes.  Direct mode: a common part
// (staged inputs / outputs, status, segments, channel table, reduction
// slots) and a tail that pass 1 fills with its partition and column arrays
// and pass 2 with its channel-sorted copy.  In pass 1 the sorted arrivals
// overlay the staged addresses, which are dead once the tile is decoded.
static u32 layout(PassArgs& a, u32 T, u32 L, u32 C, u32 K, u32 dies,
                  u32 group_channels, bool direct)
{
    u32 off = 0;
    auto take = [&](u32 bytes) {
        off = align_up(off, 16);
        const u32 at = off;
        off += bytes;
        return at;
    };
    const u32 pm_capacity = direct ? 0 : T / L + group_channels;
    a.T = T;
    a.L = L;
    a.C = C;
    a.K = K;
    a.group_channels = group_channels;
    a.pm_capacity = pm_capacity;
    const u32 D = dies ? dies : 1;
    if (direct) {
        a.off_addr = take(8 * (T + C));
        a.off_arr = take(8 * T);
        a.off_op = take(T);
        a.off_seg = take(4 * (C + 2));
        a.off_chan = take(static_cast<u32>(sizeof(ChanInfo)) * C);
        a.off_red = take(8 * 8 * kWarps);
        const u32 tail = align_up(off, 16);
        // pass 1
        a.off_bytes = take(4 * T);
        a.off_key = take(2 * T);
        a.off_rank = take(2 * T);
        // the chains' die words (below) overlay the key and rank arrays;
        // short tiles leave them less room than the words need
        const u32 dies_bytes = 4 * (K - 1) * kThreadsDie;
        if (4 * T < dies_bytes) take(dies_bytes - 4 * T);
        a.off_wcnt = take(4 * kWarps * (C + 1));
        a.off_act = take(16 * C * D);
        a.off_ranges = take(static_cast<u32>(sizeof(DevRange)) * kSmemRanges);
        a.off_pm = take(8 * C * K);  // column-0 snapshot
        a.off_sinfo[0] = take(4 * (T + C));
        a.off_sarr[0] = a.off_addr;
        a.off_ord = 0;
        // the chains' die words overlay the key and rank arrays, which are
        // dead once the sorted copy is written
        a.off_dies[0] = a.off_key;
        const u32 end1 = align_up(off, 16);
        // pass 2
        off = tail;
        a.off_sarr[1] = take(8 * (T + C));
        a.off_sinfo[1] = take(4 * (T + C));
        a.off_slot = take(2 * T);
        a.off_dies[1] = 0;
        const u32 end2 = align_up(off, 16);
        return end1 > end2 ? end1 : end2;
    }
    a.off_addr = take(8 * T);
    a.off_arr = take(8 * T);
    a.off_bytes = take(4 * T);
    a.off_op = take(T);
    a.off_ord = take(2 * T);
    a.off_key = take(2 * T);
    a.off_rank = take(2 * T);
    a.off_seg = take(4 * (C + 2));
    a.off_wcnt = take(4 * kWarps * (C + 1));
    a.off_chan = take(static_cast<u32>(sizeof(ChanInfo)) * C);
    a.off_act = take(16 * C * D);
    a.off_red = take(8 * 8 * kWarps);
    a.off_ranges = take(static_cast<u32>(sizeof(DevRange)) * kSmemRanges);
    a.off_pbase = take(4 * (C + 2));
    a.off_pchan = take(2 * (T / L + C + 1));
    a.off_pm = take(8 * pm_capacity * K * (K + 1));
    a.off_pin = take(8 * pm_capacity * K);
    a.off_die = take(8 * D * kThreads);
    a.off_sarr[0] = a.off_sarr[1] = 0;
    a.off_sinfo[0] = a.off_sinfo[1] = 0;
    return align_up(off, 16);
}

// Shared-memory layout of direct_fast_kernel (tile kFastTile): the staged
// inputs, the channel-sorted copy in buffers of its own (so that the next
// tile's inputs can stream in while the chains read the sorted copy),
// per-warp counts, segment starts, the channel table, the column-0 snapshot.
// dynamic shared memory of a pass-1 CTA that leaves room for 3 per SM
constexpr u32 kFastSmemBudget = 76800;

static u32 layout_fast(PassArgs& a, u32 C, u32 K, bool general = false, u32 ranges = 0,
                       bool halves = false)
{
    u32 off = 0;
    auto take = [&](u32 bytes) {
        off = align_up(off, 16);
        const u32 at = off;
        off += bytes;
        return at;
    };
    const u32 T = kFastTile;
    a.off_addr = take(8 * T);
    a.off_arr = take(8 * T);
    a.off_bytes = take(4 * T);
    a.off_op = take(T);
    a.off_sarr[0] = take(8 * (T + C));
    a.off_sinfo[0] = take(4 * (T + C));
    a.off_seg = take(4 * (C + 2));
    a.off_chan = take(static_cast<u32>(sizeof(ChanInfo)) * C);
    // per-warp counts, the segment scan's warp totals and the column-0
    // snapshot, with the chains' die words over them (the counts and totals
    // are dead once the sorted copy is written, the snapshot is taken after
    // the chains)
    const u32 wc_bytes = align_up(4 * kWarps * (C + 1), 16);
    const u32 red_bytes = 8 * 8 * kWarps;
    const u32 dies_bytes = 4 * (K - 1) * kThreads;
    const u32 col0_bytes = 8 * C * K * (halves ? 2 : 1);  // a snapshot per range
    a.off_key = a.off_rank = a.off_ord = a.off_act = a.off_ranges = 0;
    a.off_mid = halves ? take(4 * C) : 0;
    if (general) {
        // no prefetch: the die words overlay the staged addresses (dead once
        // decoded); the tile's activity (flushed before the chains) and the
        // column-0 snapshot (taken after them) share a slot
        const u32 pm_bytes = align_up(col0_bytes, 16), act_bytes = 16 * C * (K - 1);
        a.off_wcnt = take(wc_bytes + red_bytes + (pm_bytes > act_bytes ? pm_bytes : act_bytes));
        a.off_red = a.off_wcnt + wc_bytes;
        a.off_pm = a.off_red + red_bytes;
        a.off_act = a.off_pm;
        a.off_dies[0] = a.off_addr;
        if (ranges > 1 && ranges <= kSmemRanges)
            a.off_ranges = take(static_cast<u32>(sizeof(DevRange)) * ranges);
        // the transfer table, where it leaves room for 3 CTAs per SM
        a.off_xtab = 0;
        if (align_up(off, 16) + 4 * C * kXTabSizes <= kFastSmemBudget)
            a.off_xtab = take(4 * C * kXTabSizes);
        return align_up(off, 16);
    }
    const u32 shared = wc_bytes + red_bytes + col0_bytes;
    a.off_wcnt = take(shared > dies_bytes ? shared : dies_bytes);
    a.off_red = a.off_wcnt + wc_bytes;
    a.off_pm = a.off_red + red_bytes;
    a.off_dies[0] = a.off_wcnt;
    return align_up(off, 16);
}

}  // namespace hbfb

// ---------------------------------------------------------------- C++ entry
// (called by context.cu; not part of the C ABI)
namespace hbfb {

// Direct mode: pass 1 holds two column items per thread, pass 2 one channel.
static bool direct_supported(u32 C, u32 K, u32 dies)
{
    const bool d_ok = dies == 1 || dies == 2 || dies == 4 || dies == 8;
    return dies > 0 && d_ok && K == dies + 1 && C * (K + 1) <= 2 * kThreads && C <= kThreads;
}

int plan_batch(u64 n, u32 C, u32 K, u32 dies, int sm_count, BatchPlan* plan)
{
    PassArgs probe{};
    const bool direct = direct_supported(C, K, dies);
    u32 T = 2048, L = 32, group = C;
    const u32 per_sm = direct ? 3 : 2;
    const u32 smem_limit = (direct ? 74 : 110) * 1024;  // 3 or 2 CTAs per SM
    if (direct) {
        L = T;
        while (layout(probe, T, L, C, K, dies, group, true) > smem_limit) {
            if (T <= 512) return -1;
            T /= 2;
            L = T;
        }
    } else {
        for (;;) {
            const u32 bytes = layout(probe, T, L, C, K, dies, group, false);
            if (bytes <= smem_limit) break;
            if (group > 8) group = (group + 1) / 2;
            else if (T > 512) T /= 2;
            else return -1;
        }
    }
    // small batches: shorter tiles (down to 256 accesses, one per thread),
    // so that at least one runs per SM (a tile's time is latency-bound;
    // media-action pieces are a few thousand accesses)
    while (T > 256 && (n + T - 1) / T < static_cast<u64>(sm_count)) {
        T /= 2;
        if (direct) L = T;
    }
    const u64 tiles = (n + T - 1) / T;
    const u64 max_ctas = static_cast<u64>(sm_count) * per_sm;
    u64 ctas = tiles < max_ctas ? tiles : max_ctas;
    if (ctas == 0) ctas = 1;
    const u64 per = (tiles + ctas - 1) / ctas;
    ctas = (tiles + per - 1) / per;
    if (ctas == 0) ctas = 1;
    plan->T = T;
    plan->L = L;
    plan->C = C;
    plan->K = K;
    plan->group_channels = group;
    plan->ctas = static_cast<u32>(ctas);
    plan->tiles_per_cta = static_cast<u32>(per ? per : 1);
    plan->smem_bytes = layout(probe, T, L, C, K, dies, group, direct);
    plan->direct = direct ? 1u : 0u;
    plan->dies = dies;
    return 0;
}

static_assert(kErrNeedSeq < 256u, "the sequential flag is set by a one-byte memset");

// Launch sequence of one batch: pass 1, range scan, pass 2, then the
// sequential kernel, which returns at once unless the error word asks for it
// (set by the host when its tick bound fails, or by pass 1 on the device).
using PassKernel = void (*)(const PassArgs);

// The pass-2 instantiation for admit-free batches (z), tile halves and the
// walk in pass 2.
template <int D>
static PassKernel pick_replay(bool z, bool halves, bool walk)
{
    if (walk)
        return z ? (halves ? direct_replay_kernel<D, true, true, true>
                           : direct_replay_kernel<D, true, false, true>)
                 : (halves ? direct_replay_kernel<D, false, true, true>
                           : direct_replay_kernel<D, false, false, true>);
    return z ? (halves ? direct_replay_kernel<D, true, true> : direct_replay_kernel<D, true>)
             : (halves ? direct_replay_kernel<D, false, true> : direct_replay_kernel<D, false>);
}

cudaError_t launch_batch(const DecodeParams& dp, const TimingParams& tp,
                         const BatchIO& io, const BatchPlan& plan,
                         const BatchScratch& s, bool force_sequential,
                         cudaStream_t stream, const LaunchHooks& hooks)
{
    const u32 initial = force_sequential ? kErrNeedSeq : 0u;
    cudaError_t err = cudaMemsetAsync(s.error, 0, sizeof(u32), stream);
    if (err != cudaSuccess) return err;
    if (tp.act_stage && !force_sequential) {
        err = cudaMemsetAsync(tp.act_stage, 0, 16ull * plan.C * (tp.dies ? tp.dies : 1), stream);
        if (err != cudaSuccess) return err;
    }
    if (initial) {
        // the word is zero: setting its low byte (little-endian) gives
        // kErrNeedSeq without a copy from host memory, so the sequence stays
        // valid inside a stream capture
        err = cudaMemsetAsync(s.error, static_cast<int>(kErrNeedSeq), 1, stream);
        if (err != cudaSuccess) return err;
    }
    bool walk = false;
    if (!force_sequential) {
        PassArgs a{};
        layout(a, plan.T, plan.L, plan.C, plan.K, tp.dies, plan.group_channels,
               plan.direct != 0);
        a.dp = dp;
        a.tp = tp;
        a.address = io.address;
        a.bytes = io.bytes;
        a.op = io.op;
        a.arrival = io.arrival;
        a.done = io.done;
        a.latency = io.latency;
        a.status = io.status;
        a.n = io.n;
        a.tiles_per_cta = plan.tiles_per_cta;
        a.vec = io.aligned ? 1u : 0u;
        a.agg = s.agg;
        a.incoming = s.incoming;
        a.error = s.error;
        a.last_arrival = s.last_arrival;
        a.state_in = s.state_in;
        a.counters = s.counters;
        a.state_out = s.state_out;
        const bool fast = tp.model == kModelFast;
        using Kernel = void (*)(const PassArgs);
        Kernel p1 = fast ? timing_pass_kernel<kModelFast, 1> : timing_pass_kernel<kModelDie, 1>;
        Kernel p2 = fast ? timing_pass_kernel<kModelFast, 2> : timing_pass_kernel<kModelDie, 2>;
        bool fast_p1 = false, general_p1 = false;
        if (plan.direct) {
            // the specialized decode: one range, power-of-two geometry, one
            // transfer shift, no activity counting
            const bool f = dp.one.valid && dp.pow2 && tp.x_shift != kXDivide && !tp.act_stage &&
                           tp.admit_zero;
            const bool f2 = f && plan.T == kFastTile;  // direct_fast_kernel's fixed tile
            // its general instantiation: any ranges, activity, admission
            // delays and per-channel rates, for batches in arrival order
            const bool g2 = !f2 && plan.T == kFastTile && !tp.any_order;
            fast_p1 = f2 || g2;
            general_p1 = g2;
            const bool z = tp.admit_zero != 0;
            switch (plan.dies) {
            case 1:
                p1 = f2  ? direct_fast_kernel<1>
                     : g2 ? direct_fast_kernel<1, true>
                     : f ? direct_pass_kernel<1, 1, true> : direct_pass_kernel<1, 1, false>;
                p2 = z ? direct_replay_kernel<1, true> : direct_replay_kernel<1, false>;
                break;
            case 2:
                p1 = f2  ? direct_fast_kernel<2>
                     : g2 ? direct_fast_kernel<2, true>
                     : f ? direct_pass_kernel<1, 2, true> : direct_pass_kernel<1, 2, false>;
                p2 = z ? direct_replay_kernel<2, true> : direct_replay_kernel<2, false>;
                break;
            case 4:
                p1 = f2  ? direct_fast_kernel<4>
                     : g2 ? direct_fast_kernel<4, true>
                     : f ? direct_pass_kernel<1, 4, true> : direct_pass_kernel<1, 4, false>;
                p2 = z ? direct_replay_kernel<4, true> : direct_replay_kernel<4, false>;
                break;
            default:
                p1 = f2  ? direct_fast_kernel<8>
                     : g2 ? direct_fast_kernel<8, true>
                     : f ? direct_pass_kernel<1, 8, true> : direct_pass_kernel<1, 8, false>;
                p2 = z ? direct_replay_kernel<8, true> : direct_replay_kernel<8, false>;
                break;
            }
        }
        // One tile per CTA and few column items: each channel's segment is
        // timed as two ranges (its halves), so that twice the items and
        // chains (pass 1 and pass 2) each walk half a segment.
        const bool halves = fast_p1 && plan.tiles_per_cta == 1 &&
                            2 * plan.C * (plan.K + 1) <= static_cast<u32>(kThreads) &&
                            s.ranges_capacity >= 2ull * plan.ctas;
        a.halves = halves ? 1u : 0u;
        // small batches: pass 2 also runs the sequential walk when it is
        // needed, instead of a separate launch after it
        walk = plan.direct && plan.tiles_per_cta == 1;
        if (plan.direct) {
            const bool z = tp.admit_zero != 0;
            switch (plan.dies) {
            case 1: p2 = pick_replay<1>(z, halves, walk); break;
            case 2: p2 = pick_replay<2>(z, halves, walk); break;
            case 4: p2 = pick_replay<4>(z, halves, walk); break;
            default: p2 = pick_replay<8>(z, halves, walk); break;
            }
        }
        // direct_fast_kernel runs on a layout of its own
        PassArgs a1 = a;
        u32 smem1 = plan.smem_bytes;
        if (fast_p1)
            smem1 = layout_fast(a1, plan.C, plan.K, general_p1,
                                dp.one.valid ? 0u : dp.range_count, halves);
        err = cudaFuncSetAttribute(p1, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(smem1));
        if (err != cudaSuccess) return err;
        err = cudaFuncSetAttribute(p2, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(plan.smem_bytes));
        if (err != cudaSuccess) return err;
        hooks(kSlotPass1, 0, stream);
        p1<<<plan.ctas, kThreads, smem1, stream>>>(a1);
        hooks(kSlotPass1, 1, stream);
        ScanArgs sa{};
        sa.agg = s.agg;
        sa.incoming = s.incoming;
        sa.state_in = s.state_in;
        sa.state_out = s.state_out;
        sa.error = s.error;
        sa.last_arrival = s.last_arrival;
        sa.arrival = io.arrival;
        sa.n = io.n;
        sa.ctas = halves ? 2 * plan.ctas : plan.ctas;  // ranges
        sa.C = plan.C;
        sa.K = plan.K;
        sa.counters = s.counters;
        sa.dies = tp.dies;
        sa.act_stage = tp.act_stage;
        sa.die_read_bytes = tp.die_read_bytes;
        sa.die_writes = tp.die_writes;
        // per warp: `chunk` staged aggregates and the group's composite
        const u32 per = plan.K * (plan.K + 1);
        const u32 group = (sa.ctas + kScanWarps - 1) / kScanWarps;
        const u32 room = (96u * 1024u / 8u) / kScanWarps - per;
        sa.chunk = std::max(1u, std::min(group, room / per));
        const u32 groups = (sa.ctas + kLbRanges - 1) / kLbRanges;
        if (s.scan_lb && s.scan_groups && groups <= kLbMaxGroups &&
            static_cast<u64>(groups) * plan.C <= kLbFlagWords) {
            // several CTAs per channel, chained by look-back
            LbScanArgs lb{};
            lb.gmap = s.scan_groups;
            lb.gstate = s.scan_groups + static_cast<u64>(groups) * plan.C * per;
            lb.ctr = s.scan_lb;
            lb.groups = groups;
            const u32 lb_smem =
                8u * (kLbWarps * kLbRangesPerWarp * per + 2 * kLbWarps * per +
                      (kLbMaxGroups - 1) * per + kLbWarps * plan.K);
            err = cudaFuncSetAttribute(range_scan_lb_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(lb_smem));
            if (err != cudaSuccess) return err;
            hooks(kSlotScan, 0, stream);
            range_scan_lb_kernel<<<groups * plan.C, kLbWarps * 32, lb_smem, stream>>>(sa, lb);
            hooks(kSlotScan, 1, stream);
        } else {
            const u32 scan_smem =
                8u * (kScanWarps * (sa.chunk * per + per) + kScanWarps * plan.K);
            err = cudaFuncSetAttribute(range_scan_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(scan_smem));
            if (err != cudaSuccess) return err;
            hooks(kSlotScan, 0, stream);
            range_scan_kernel<<<plan.C, kScanWarps * 32, scan_smem, stream>>>(sa);
            hooks(kSlotScan, 1, stream);
        }
        hooks(kSlotPass2, 0, stream);
        p2<<<plan.ctas, kThreads, plan.smem_bytes, stream>>>(a);
        hooks(kSlotPass2, 1, stream);
    }
    // the direct pass 2 runs the sequential walk itself when the batch needs
    // it; the other paths launch it (it returns at once unless needed)
    if (walk) return cudaGetLastError();
    SeqArgs q{};
    q.dp = dp;
    q.tp = tp;
    q.address = io.address;
    q.bytes = io.bytes;
    q.op = io.op;
    q.arrival = io.arrival;
    q.done = io.done;
    q.latency = io.latency;
    q.status = io.status;
    q.n = io.n;
    q.C = plan.C;
    q.K = plan.K;
    q.state_in = s.state_in;
    q.state_out = s.state_out;
    q.error = s.error;
    q.last_arrival = s.last_arrival;
    q.counters = s.counters;
    const u32 threads = 64;
    const u32 blocks = (plan.C + threads - 1) / threads;
    hooks(kSlotSequential, 0, stream);
    if (tp.model == kModelFast)
        sequential_kernel<kModelFast><<<blocks, threads, 0, stream>>>(q);
    else
        sequential_kernel<kModelDie><<<blocks, threads, 0, stream>>>(q);
    hooks(kSlotSequential, 1, stream);
    return cudaGetLastError();
}

cudaError_t launch_decode(const DecodeParams& dp, const u64* address,
                          const u32* bytes, const u8* op, u64 n, void* out,
                          cudaStream_t stream, const LaunchHooks& hooks)
{
    if (n == 0) return cudaSuccess;
    const u32 threads = 256;
    const u64 blocks = (n + threads - 1) / threads;
    hooks(kSlotDecode, 0, stream);
    decode_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        dp, address, bytes, op, n, static_cast<DecodeOut*>(out));
    hooks(kSlotDecode, 1, stream);
    return cudaGetLastError();
}

}  // namespace hbfb

// ---------------------------------------------------------------------------
// Hybrid sampler bit (A7).  The reference numbers every access that reaches
// resolve_fast_or_hybrid (hbf_device.cu:779-788) with a device-wide counter
// and sends it to the reference model when hybrid_reference_sample
// (hbf_device.cuh:738-744) says so, keyed by
// media address ^ range_id << 32 ^ op.  Here the counter is the context's
// running count of timed accesses in batch order: each CTA counts its
// contiguous share, a one-block scan turns the counts into starting numbers,
// and the write pass numbers the accesses in order.
namespace hbfb {
namespace {

constexpr u32 kSampleThreads = 256;
constexpr u32 kSampleItems = 8;  // contiguous accesses per thread per round

// splitmix64 finalizer (Steele, Lea & Flood, "Fast splittable pseudorandom
// number generators", 2014), the mix the reference sampler uses
__device__ __forceinline__ u64 sample_mix(u64 v)
{
    v += 0x9e3779b97f4a7c15ull;
    v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
    v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
    return v ^ (v >> 31);
}

__device__ __forceinline__ u64 sample_key(const DecodeParams& p, const Decoded& d, u32 op)
{
    return d.media ^ (static_cast<u64>(p.ranges[d.range_index].range_id) << 32) ^ op;
}

__global__ void __launch_bounds__(kSampleThreads)
sample_count_kernel(const DecodeParams p, const u64* address, const u32* bytes, const u8* op,
                    u64 n, u64 per, u64* counts)
{
    const u64 lo = blockIdx.x * per, hi = lo + per < n ? lo + per : n;
    u32 mine = 0;
    for (u64 i = lo + threadIdx.x; i < hi; i += kSampleThreads)
        mine += classify_decode(p, address[i], bytes[i], op[i], false).status == kModeled;
    __shared__ u32 red[kSampleThreads / 32];
    for (int o = 16; o > 0; o >>= 1) mine += __shfl_down_sync(0xffffffffu, mine, o);
    if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = mine;
    __syncthreads();
    if (threadIdx.x == 0) {
        u64 total = 0;
        for (u32 w = 0; w < kSampleThreads / 32; ++w) total += red[w];
        counts[blockIdx.x] = total;
    }
}

// counts -> starting sequence numbers; the context counter moves past them
__global__ void sample_scan_kernel(u64* counts, u32 ctas, u64* seq)
{
    if (threadIdx.x != 0) return;
    u64 run = *seq;
    for (u32 b = 0; b < ctas; ++b) {
        const u64 c = counts[b];
        counts[b] = run;
        run += c;
    }
    *seq = run;
}

__global__ void __launch_bounds__(kSampleThreads)
sample_write_kernel(const DecodeParams p, const u64* address, const u32* bytes, const u8* op,
                    u64 n, u64 per, const u64* starts, u32 warmup, u64 threshold, u8* sample)
{
    const u64 lo = blockIdx.x * per, hi = lo + per < n ? lo + per : n;
    __shared__ u32 warp_sum[kSampleThreads / 32];
    __shared__ u32 round_total;
    const u32 lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    u64 next = starts[blockIdx.x];
    for (u64 base = lo; base < hi; base += static_cast<u64>(kSampleThreads) * kSampleItems) {
        const u64 first = base + static_cast<u64>(threadIdx.x) * kSampleItems;
        Decoded d[kSampleItems];
        u32 count = 0;
#pragma unroll
        for (u32 k = 0; k < kSampleItems; ++k) {
            const u64 i = first + k;
            d[k].status = 0;
            if (i < hi) {
                d[k] = classify_decode(p, address[i], bytes[i], op[i], false);
                count += d[k].status == kModeled;
            }
        }
        // block exclusive scan of the per-thread counts (index order)
        u32 incl = count;
        for (int o = 1; o < 32; o <<= 1) {
            const u32 y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= static_cast<u32>(o)) incl += y;
        }
        if (lane == 31) warp_sum[warp] = incl;
        __syncthreads();
        if (threadIdx.x == 0) {
            u32 run = 0;
            for (u32 w = 0; w < kSampleThreads / 32; ++w) {
                const u32 s = warp_sum[w];
                warp_sum[w] = run;
                run += s;
            }
            round_total = run;
        }
        __syncthreads();
        u64 seq = next + warp_sum[warp] + incl - count;
#pragma unroll
        for (u32 k = 0; k < kSampleItems; ++k) {
            const u64 i = first + k;
            if (i >= hi) break;
            u8 bit = 0;
            if (d[k].status == kModeled) {
                bit = seq < warmup ||
                      (threshold != 0 && sample_mix(seq ^ sample_key(p, d[k], op[i])) <= threshold);
                ++seq;
            }
            sample[i] = bit;
        }
        next += round_total;
        __syncthreads();
    }
}

}  // namespace

cudaError_t launch_sample(const DecodeParams& dp, const u64* address, const u32* bytes,
                          const u8* op, u64 n, u8* sample, u32 warmup, u64 threshold,
                          u64* seq, u64* counts, u32 max_ctas, cudaStream_t stream,
                          const LaunchHooks& hooks)
{
    if (n == 0) return cudaSuccess;
    const u64 min_per = static_cast<u64>(kSampleThreads) * kSampleItems;
    u64 ctas = (n + min_per - 1) / min_per;
    if (ctas > max_ctas) ctas = max_ctas;
    const u64 per = (n + ctas - 1) / ctas;
    ctas = (n + per - 1) / per;
    hooks(kSlotOther, 0, stream);
    sample_count_kernel<<<static_cast<unsigned>(ctas), kSampleThreads, 0, stream>>>(
        dp, address, bytes, op, n, per, counts);
    sample_scan_kernel<<<1, 32, 0, stream>>>(counts, static_cast<u32>(ctas), seq);
    sample_write_kernel<<<static_cast<unsigned>(ctas), kSampleThreads, 0, stream>>>(
        dp, address, bytes, op, n, per, counts, warmup, threshold, sample);
    hooks(kSlotOther, 1, stream);
    return cudaGetLastError();
}

}  // namespace hbfb

// ---------------------------------------------------------------------------
// Chained media actions (Capacity mode).  A read that refills a page after a
// dirty victim's program arrives at max(arrival, program completion)
// (request_dispatcher.cpp:294-298).  The batch is timed in pieces that each
// start at such a read; before a piece runs, its first read's arrival is
// raised to the completion of its program, which an earlier piece produced.
namespace hbfb {
namespace {

__global__ void chain_fixup_kernel(u64* arrival, const u64* done, const u32* chain, u64 index)
{
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        const u32 src = chain[index];
        if (src != 0xffffffffu && done[src] > arrival[index]) arrival[index] = done[src];
    }
}

// Exact fallback for media-action batches with more chained reads than the
// piece path takes: one thread walks every action in batch order with the
// saturating die model.
__global__ void chain_sequential_kernel(const DecodeParams dp, const TimingParams tp,
                                        const u64* address, const u32* bytes, const u8* op,
                                        u64* arrival, const u32* chain, u64 n, u32 K,
                                        const u64* state_in, u64* state_out, u64* done,
                                        u64* latency, u8* status, u64 words)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    for (u64 k = 0; k < words; ++k) state_out[k] = state_in[k];
    for (u64 i = 0; i < n; ++i) {
        u64 a = arrival[i];
        if (chain[i] != 0xffffffffu && done[chain[i]] > a) a = done[chain[i]];
        arrival[i] = a;
        const Decoded d = classify_decode(dp, address[i], bytes[i], op[i], true);
        status[i] = static_cast<u8>(d.status);
        if (d.status != kModeled) {
            done[i] = a;
            latency[i] = 0;
            continue;
        }
        const u32 c = d.local;
        u64* st = state_out + static_cast<u64>(c) * K;
        const u64 bw = tp.chan_bw[c];
        const u64 num = static_cast<u64>(bytes[i]) * 1000000000ull;
        const u64 x = sat_mul_u64(num / bw + (num % bw != 0), tp.time_scale);
        const u64 top = static_cast<u64>(op[i] ? tp.chan_t_prog[c] : tp.chan_t_read[c]);
        u64 s = a;
        const u64 admit = static_cast<u64>(tp.chan_admit[c]);
        if (admit > s) s = admit;
        if (st[0] > s) s = st[0];
        if (st[1 + d.die] > s) s = st[1 + d.die];
        st[0] = sat_add_u64(s, x);
        st[1 + d.die] = sat_add_u64(st[0], top);
        done[i] = st[1 + d.die];
        latency[i] = done[i] - a;
        if (tp.die_read_bytes) {
            const u64 k = static_cast<u64>(c) * tp.dies + d.die;
            if (op[i]) tp.die_writes[k] += 1;
            else tp.die_read_bytes[k] += bytes[i];
        }
    }
}

}  // namespace

cudaError_t launch_chain_fixup(u64* arrival, const u64* done, const u32* chain, u64 index,
                               cudaStream_t stream)
{
    chain_fixup_kernel<<<1, 32, 0, stream>>>(arrival, done, chain, index);
    return cudaGetLastError();
}

cudaError_t launch_chain_sequential(const DecodeParams& dp, const TimingParams& tp,
                                    const u64* address, const u32* bytes, const u8* op,
                                    u64* arrival, const u32* chain, u64 n, u32 K,
                                    const u64* state_in, u64* state_out, u64 words, u64* done,
                                    u64* latency, u8* status, cudaStream_t stream)
{
    chain_sequential_kernel<<<1, 32, 0, stream>>>(dp, tp, address, bytes, op, arrival, chain, n,
                                                  K, state_in, state_out, done, latency, status,
                                                  words);
    return cudaGetLastError();
}

}  // namespace hbfb
