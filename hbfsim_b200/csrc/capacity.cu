// capacity.cu -- Capacity mode: exact LRU over HBM frames, batch-parallel.
//
// Reference: CapacityPageService::resolve
// (src/host_service/capacity_page_service.cpp:97-210) keeps pages of
// CAPACITY ranges in HBM frames and, on a miss, reads the page from HBF after
// programming a dirty victim (request_dispatcher.cpp:107-126); the exact-LRU
// policy is the reference's offline LruCache
// (adapters/vllm_capacity/placement_policy.py:68-93).  The reference runtime
// decides one request at a time under a mutex.
//
// B200 design.  LRU decisions follow from reuse distances, so a whole batch
// is decided at once.  The batch is prefixed with the resident list (oldest
// first, as if those pages had just been accessed in that order), giving a
// sequence S of m accesses.  Then, for access i with previous access p of
// the same page (prev(i), found by a stable radix sort on the page):
//
//   hit(i)  <=>  p exists and  distinct pages in (p, i)  <  F   (F = frames)
//   distinct pages in (p, i) = (i - p - 1) - #{u < i : prev(u) > p}
//
// and the count is one query on a wavelet matrix over prev(.) (each level a
// stable one-bit partition: ballots and prefix counts).  A miss evicts when
// F distinct pages are already resident.  Entry j leaves the cache exactly
// when its page's next access is a miss (or never comes), and entries leave
// in order of j: so the k-th evicting miss evicts the page of the k-th such
// entry.  A victim is dirty when a write hit its page since the miss that
// brought it in (segmented OR over the page-sorted order).  The new resident
// list is the newest F last-occurrences of pages, oldest first.
#include "context.h"

#include <algorithm>
#include <vector>

namespace hbfb {

constexpr u32 kNone = 0xffffffffu;

struct CapacityState {
    std::uint64_t frames = 0;        // F
    std::uint32_t page_shift = 12;   // LRU page = 2^page_shift bytes
    std::uint64_t resident = 0;      // entries in the resident list
    std::uint64_t capacity_m = 0;    // scratch size (sequence entries)
    // resident list, oldest first (device)
    u32* res_page = nullptr;
    u8* res_dirty = nullptr;
    // sequence and scratch
    u32 *key = nullptr, *w = nullptr, *bidx = nullptr;
    u32 *sk = nullptr, *si = nullptr, *tk = nullptr, *ti = nullptr;
    u32 *prev = nullptr, *next = nullptr, *cur = nullptr, *nxt = nullptr;
    uint2* levels = nullptr;         // wavelet levels [32][m/32 + 1]
    u32 *hit = nullptr, *a = nullptr, *b = nullptr, *c = nullptr, *d = nullptr;
    u32* tile_sums = nullptr;
    std::uint64_t tile_sums_words = 0;
    u32* valid = nullptr;            // per batch access: 1 = capacity access
    u32* status = nullptr;
    // per batch access (batch order): LRU page and decisions, action slot
    u32 *apage = nullptr, *ahit = nullptr, *avictim = nullptr, *adirty = nullptr;
    u32 *anact = nullptr, *apos = nullptr;
    // media actions (program of a dirty victim, read of a missed page)
    std::uint64_t act_capacity = 0;
    u64* act_addr = nullptr;
    u32* act_bytes = nullptr;
    u8* act_op = nullptr;
    u64* act_arr = nullptr;
    u32* act_chain = nullptr;        // program feeding a chained read, or kNone
    u64* act_done = nullptr;
    u64* act_lat = nullptr;
    u8* act_status = nullptr;
    u32* chained = nullptr;          // indices of the chained reads
    u32* chained_flag = nullptr;
    u32* chained_pos = nullptr;
    DevRange* media_range = nullptr; // identity range: media address -> itself
    u32* counts = nullptr;           // small device results
    // what one timing batch of the media actions changes besides its
    // outputs (counters, last arrival, die activity), saved before the
    // fixed-point rounds and put back before each repeat
    unsigned char* snap = nullptr;
    std::uint64_t snap_bytes = 0;
    std::uint32_t rounds_last = 0;   // rounds the last batch's fixed point took
    std::uint32_t walked_last = 0;   // 1: it took the one-thread walk instead
    std::uint64_t pieces_last = 0;   // pieces it ran in (0: settled in rounds)
    // CLOCK policy (the reference runtime's HbmCache): per frame its page,
    // reference and dirty byte; page -> frame table; [hand, frames in use]
    std::uint32_t policy = 0;        // HBFSIM_CAPACITY_POLICY_*
    std::uint64_t table_pages = 0;   // entries of clk_table
    u32* clk_table = nullptr;
    u32* clk_page = nullptr;
    u8* clk_ref = nullptr;
    u8* clk_dirty = nullptr;
    u64* clk_state = nullptr;
    // single-pass scans (look-back): per tile a tagged status word, the
    // tile ticket counter and an error word; the tag of the current scan
    unsigned long long* lb_state = nullptr;
    std::uint64_t lb_tiles = 0;
    u32* lb_misc = nullptr;          // [0] ticket counter, [1] error
    std::uint32_t lb_tag = 0;
    // counters (host)
    std::uint64_t calls = 0, accesses = 0, hits = 0, misses = 0, evictions = 0,
                  dirty_evictions = 0;
};

namespace {

constexpr u32 kT = 256;          // threads per CTA
constexpr u32 kItems = 8;        // elements per thread in scans
constexpr u32 kTile = kT * kItems;

template <typename T>
cudaError_t grow(T** p, std::uint64_t n)
{
    if (*p) cudaFree(*p);
    *p = nullptr;
    return cudaMalloc(reinterpret_cast<void**>(p), sizeof(T) * (n ? n : 1));
}

__device__ __forceinline__ u32 lane() { return threadIdx.x & 31u; }

// ---------------------------------------------------------------- scans
struct AddOp {
    static __device__ __forceinline__ u32 f(u32 a, u32 b) { return a + b; }
    static constexpr u32 id = 0;
};
struct MaxOp {
    static __device__ __forceinline__ u32 f(u32 a, u32 b) { return a > b ? a : b; }
    static constexpr u32 id = 0;
};

// Block-wide exclusive scan of one value per thread; returns the exclusive
// prefix and writes the block total to *total (all threads).
template <class Op>
__device__ __forceinline__ u32 block_scan(u32 v, u32* total)
{
    __shared__ u32 warp_tot[kT / 32];
    u32 incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const u32 y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane() >= static_cast<u32>(o)) incl = Op::f(incl, y);
    }
    const u32 w = threadIdx.x >> 5;
    if (lane() == 31) warp_tot[w] = incl;
    __syncthreads();
    if (threadIdx.x < 32) {
        u32 x = threadIdx.x < kT / 32 ? warp_tot[threadIdx.x] : Op::id;
        u32 xi = x;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const u32 y = __shfl_up_sync(0xffffffffu, xi, o);
            if (lane() >= static_cast<u32>(o)) xi = Op::f(xi, y);
        }
        if (threadIdx.x < kT / 32) warp_tot[threadIdx.x] = xi;  // inclusive
    }
    __syncthreads();
    const u32 before = w ? warp_tot[w - 1] : Op::id;
    const u32 excl_in_warp = __shfl_up_sync(0xffffffffu, incl, 1);
    const u32 excl = lane() ? Op::f(before, excl_in_warp) : before;
    *total = warp_tot[kT / 32 - 1];
    __syncthreads();
    return excl;
}

// ---------------------------------------------------------------- look-back
// Single-pass scans (decoupled look-back, Merrill & Garland, "Single-pass
// Parallel Prefix Scan with Decoupled Look-back", 2016).  Each CTA takes the
// next tile ticket (so a tile only waits on tiles that already run), scans
// its tile, publishes its aggregate, then walks back over its predecessors'
// published words -- adding aggregates until it meets an inclusive prefix --
// and publishes its own inclusive prefix.  A status word is
//   tag << 34 | kind << 32 | value    (kind 1 aggregate, 2 inclusive)
// with the scan's tag, so that words of earlier scans never match and the
// array needs no clearing.  Every wait is bounded: after kLookbackSpins
// polls the CTA records an error (the host reports it) and goes on.
struct LookBack {
    unsigned long long* state;
    u32* misc;   // [0] ticket counter (reset by the last ticket), [1] error
    u32 tag;
    u32 tiles;
};

constexpr u32 kLookbackSpins = 1u << 22;

__device__ __forceinline__ void lb_publish(const LookBack& lb, u32 tile, u32 kind, u32 value)
{
    const unsigned long long w = static_cast<unsigned long long>(lb.tag) << 34 |
                                 static_cast<unsigned long long>(kind) << 32 | value;
    atomicExch(lb.state + tile, w);
}

// Exclusive prefix of `tile` under Op, called by one whole warp (the result
// in every lane).  The warp reads a window of the 32 preceding status words
// at once, lane k the word of tile - 1 - k; once all are published it folds
// the aggregates up to the nearest inclusive prefix, or all 32 and moves the
// window back.
template <class Op>
__device__ __forceinline__ u32 lb_prefix(const LookBack& lb, u32 tile)
{
    u32 prefix = Op::id;
    int j = static_cast<int>(tile) - 1;
    bool failed = false;
    while (j >= 0) {
        const int idx = j - static_cast<int>(lane());
        u32 kind = 2u, value = Op::id;  // before tile 0: the identity, inclusive
        if (idx >= 0) {
            const volatile unsigned long long* w =
                reinterpret_cast<volatile unsigned long long*>(lb.state + idx);
            unsigned long long x = *w;
            u32 spins = 0;
            while (!((x >> 34) == lb.tag && ((x >> 32) & 3u) != 0)) {
                if (++spins >= kLookbackSpins) {
                    failed = true;
                    break;
                }
                __nanosleep(32);
                x = *w;
            }
            kind = failed ? 2u : static_cast<u32>((x >> 32) & 3u);
            value = failed ? Op::id : static_cast<u32>(x);
        }
        const u32 incl = __ballot_sync(0xffffffffu, kind == 2u);
        const u32 last = incl ? static_cast<u32>(__ffs(incl)) - 1u : 31u;
        u32 v = lane() <= last ? value : Op::id;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = Op::f(v, __shfl_xor_sync(0xffffffffu, v, o));
        prefix = Op::f(v, prefix);
        if (incl) break;
        j -= 32;
    }
    if (__any_sync(0xffffffffu, failed) && lane() == 0) atomicExch(&lb.misc[1], 1u);
    return prefix;
}

// The tile ticket of this CTA, broadcast through shared memory.  A ticket
// past the last tile (a counter not reset) is recorded as an error; the
// caller's CTA then does nothing.
__device__ __forceinline__ u32 lb_ticket(const LookBack& lb, u32* slot)
{
    if (threadIdx.x == 0) {
        const u32 t = atomicAdd(&lb.misc[0], 1u);
        if (t >= lb.tiles) atomicExch(&lb.misc[1], 1u);
        *slot = t;
    }
    __syncthreads();
    return *slot;
}

__device__ __forceinline__ void lb_done(const LookBack& lb, u32 tile)
{
    if (threadIdx.x == 0 && tile + 1 == lb.tiles) lb.misc[0] = 0;  // every ticket is taken
}

template <class Op>
__global__ void __launch_bounds__(kT) lb_scan_kernel(const u32* in, u32* out, u64 n,
                                                     int inclusive, u32* total, LookBack lb)
{
    __shared__ u32 ticket, prefix_s;
    const u32 tile = lb_ticket(lb, &ticket);
    if (tile >= lb.tiles) return;
    const u64 base = static_cast<u64>(tile) * kTile + threadIdx.x * kItems;
    u32 v[kItems];
    u32 run = Op::id;
#pragma unroll
    for (u32 k = 0; k < kItems; ++k) {
        v[k] = base + k < n ? in[base + k] : Op::id;
        run = Op::f(run, v[k]);
    }
    u32 agg;
    u32 pre = block_scan<Op>(run, &agg);
    if (threadIdx.x < 32) {
        u32 prefix = Op::id;
        if (tile == 0) {
            if (threadIdx.x == 0) lb_publish(lb, 0, 2u, agg);
        } else {
            if (threadIdx.x == 0) lb_publish(lb, tile, 1u, agg);
            prefix = lb_prefix<Op>(lb, tile);
            if (threadIdx.x == 0) lb_publish(lb, tile, 2u, Op::f(prefix, agg));
        }
        if (threadIdx.x == 0) {
            prefix_s = prefix;
            if (total && tile + 1 == lb.tiles) *total = Op::f(prefix, agg);
            lb_done(lb, tile);
        }
    }
    __syncthreads();
    pre = Op::f(prefix_s, pre);
#pragma unroll
    for (u32 k = 0; k < kItems; ++k) {
        const u32 x = v[k];
        if (base + k < n) out[base + k] = inclusive ? Op::f(pre, x) : pre;
        pre = Op::f(pre, x);
    }
}

// ---------------------------------------------------------------- classify
__device__ __forceinline__ u32 find_range(const DevRange* r, u32 count, u64 a)
{
    u32 first = 0, last = count;
    while (first < last) {
        const u32 mid = first + (last - first) / 2;
        if (r[mid].base <= a) first = mid + 1;
        else last = mid;
    }
    return first == 0 ? count : first - 1;
}

// One access of a capacity batch: status, and the LRU page of a capacity
// access (range lookup and checks as access_supported, hbf_device.cuh:843-862,
// on CAPACITY ranges; the access must stay inside one LRU page).
__global__ void cap_classify_kernel(const DevRange* ranges, u32 count, const u64* address,
                                    const u32* bytes, const u8* op, u64 n, u32 shift, u32* page,
                                    u32* valid, u32* status)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const u64 a = address[i];
    const u32 b = bytes[i], o = op[i];
    u32 st = kUnsupported, pg = 0;
    if (b != 0) {
        const u32 idx = find_range(ranges, count, a);
        if (idx == count || a - ranges[idx].base >= ranges[idx].length) {
            const u32 succ = idx == count ? 0u : idx + 1u;
            bool overlap = false;
            if (succ < count) {
                const DevRange& r = ranges[succ];
                overlap = r.length != 0 && r.base <= ~u64{0} - r.length &&
                          a <= ~u64{0} - b && a < r.base + r.length && r.base < a + b;
            }
            st = overlap ? kUnsupported : kBypass;
        } else {
            const DevRange& r = ranges[idx];
            const u64 off = a - r.base;
            if (r.mode == 2 && r.ok && o <= 1 && b <= ~u64{0} - a && a + b <= r.end &&
                (r.permissions & (1u << o)) && (off >> shift) == ((off + b - 1) >> shift)) {
                st = kModeled;
                pg = static_cast<u32>((r.file_offset + off) >> shift);
            }
        }
    }
    page[i] = pg;
    valid[i] = st == kModeled ? 1u : 0u;
    status[i] = st;
}

// Sequence S: the resident list, then the batch's capacity accesses.
__global__ void cap_build_kernel(const u32* res_page, const u8* res_dirty, u64 resident,
                                 const u32* page, const u8* op, const u32* valid,
                                 const u32* pos, u64 n, u32* key, u32* w, u32* bidx)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < resident) {
        key[i] = res_page[i];
        w[i] = res_dirty[i];
        bidx[i] = kNone;
    }
    if (i < n && valid[i]) {
        const u64 j = resident + pos[i];
        key[j] = page[i];
        w[j] = op[i] == 1 ? 1u : 0u;
        bidx[j] = static_cast<u32>(i);
    }
}

// ---------------------------------------------------------------- radix sort
// Stable LSD radix sort of (key, index) by 8-bit digits; one CTA per tile of
// kTile elements.  Histogram layout: digit-major, tile-minor.
__global__ void __launch_bounds__(kT) radix_hist_kernel(const u32* key, u64 m, u32 shift,
                                                        u32* hist, u32 tiles)
{
    __shared__ u32 h[256];
    h[threadIdx.x] = 0;
    __syncthreads();
    const u64 base = static_cast<u64>(blockIdx.x) * kTile;
    for (u32 k = threadIdx.x; k < kTile; k += kT)
        if (base + k < m) atomicAdd(&h[(key[base + k] >> shift) & 255u], 1u);
    __syncthreads();
    hist[static_cast<u64>(threadIdx.x) * tiles + blockIdx.x] = h[threadIdx.x];
}

__global__ void __launch_bounds__(kT) radix_scatter_kernel(const u32* key, const u32* val,
                                                           u64 m, u32 shift, const u32* offsets,
                                                           u32 tiles, u32* key_out,
                                                           u32* val_out)
{
    __shared__ u32 running[256];
    __shared__ u32 warp_count[kT / 32][256];
    running[threadIdx.x] = offsets[static_cast<u64>(threadIdx.x) * tiles + blockIdx.x];
    const u32 wid = threadIdx.x >> 5;
    const u64 base = static_cast<u64>(blockIdx.x) * kTile;
    for (u32 round = 0; round < kItems; ++round) {
        for (u32 k = threadIdx.x; k < (kT / 32) * 256; k += kT) (&warp_count[0][0])[k] = 0;
        __syncthreads();
        const u64 i = base + static_cast<u64>(round) * kT + threadIdx.x;
        const bool on = i < m;
        const u32 kv = on ? key[i] : 0u;
        const u32 d = on ? (kv >> shift) & 255u : 256u;
        const u32 peers = __match_any_sync(0xffffffffu, d);
        const u32 rank = __popc(peers & ((1u << lane()) - 1u));
        if (on && rank == 0) warp_count[wid][d] = __popc(peers);
        __syncthreads();
        if (on) {
            u32 pos = running[d] + rank;
            for (u32 w2 = 0; w2 < wid; ++w2) pos += warp_count[w2][d];
            key_out[pos] = kv;
            val_out[pos] = val[i];
        }
        __syncthreads();
        u32 add = 0;
        for (u32 w2 = 0; w2 < kT / 32; ++w2) add += warp_count[w2][threadIdx.x];
        running[threadIdx.x] += add;
        __syncthreads();
    }
}

__global__ void iota_kernel(u32* v, u64 m)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < m) v[i] = static_cast<u32>(i);
}

__global__ void fill_kernel(u32* v, u64 m, u32 x)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < m) v[i] = x;
}

// prev / next links from the page-sorted order
__global__ void link_kernel(const u32* sk, const u32* si, u64 m, u32* prev, u32* next)
{
    const u64 k = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (k + 1 >= m) return;
    if (sk[k] == sk[k + 1]) {
        next[si[k]] = si[k + 1];
        prev[si[k + 1]] = si[k];
    }
}

// ---------------------------------------------------------------- wavelet
// Values v = prev + 1 (0 = no previous access).  Level l partitions the
// current order stably by bit l (zeros first) and stores, per 32 positions,
// the bits and the number of ones before them.
__global__ void value_kernel(const u32* prev, u64 m, u32* v)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < m) v[i] = prev[i] == kNone ? 0u : prev[i] + 1u;
}

// Zeros of every bit over all values (order-independent: each level's
// total zeros), one pass.
__global__ void __launch_bounds__(kT) wm_bit_zeros_kernel(const u32* v, u64 m, u32 bits,
                                                          u32* zeros)
{
    u32 ones[32];
#pragma unroll
    for (int b = 0; b < 32; ++b) ones[b] = 0;
    u32 seen = 0;
    for (u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x; i < m;
         i += static_cast<u64>(gridDim.x) * blockDim.x) {
        const u32 x = v[i];
        ++seen;
#pragma unroll
        for (int b = 0; b < 32; ++b) ones[b] += (x >> b) & 1u;
    }
#pragma unroll
    for (int b = 0; b < 32; ++b) {
        if (static_cast<u32>(b) >= bits) break;
        u32 z = seen - ones[b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) z += __shfl_down_sync(0xffffffffu, z, o);
        if (lane() == 0 && z) atomicAdd(&zeros[b], z);
    }
}

// One wavelet level in one pass: each CTA (ticket order) loads its tile
// (position base + r*kT + t in round r), takes per warp and round the ballot
// of bit `bit` and ranks the ones inside the tile, gets the zeros before the
// tile by look-back, and splits the tile stably through shared memory: its
// zeros go on after the zeros of earlier tiles, its ones after the level's Z
// zeros and the ones of earlier tiles, both as contiguous runs.  Each 32
// positions get their level word (the bits, the ones before them); the last
// tile writes the rank sentinel at position m when m is a multiple of 32.
__global__ void __launch_bounds__(kT) wm_level_kernel(const u32* v, u64 m, u32 bit,
                                                      const u32* total_zeros, u32* out,
                                                      uint2* level, LookBack lb)
{
    constexpr u32 kW = kT / 32;
    static_assert(kItems * kW == 64, "two (round, warp) counts per lane of warp 0");
    __shared__ u32 ticket, zeros_before_s, tile_zeros_s;
    __shared__ u32 cnt[kItems * kW];  // ones per (round, warp), then their prefix
    __shared__ u32 stage[kTile];
    const u32 tile = lb_ticket(lb, &ticket);
    if (tile >= lb.tiles) return;
    const u64 base = static_cast<u64>(tile) * kTile;
    const u32 valid = static_cast<u32>(m - base < kTile ? m - base : kTile);
    const u32 wid = threadIdx.x >> 5;
    u32 x[kItems], mask[kItems];
#pragma unroll
    for (u32 r = 0; r < kItems; ++r) {
        const u32 k = r * kT + threadIdx.x;
        x[r] = k < valid ? v[base + k] : 0u;
    }
#pragma unroll
    for (u32 r = 0; r < kItems; ++r) {
        const u32 k = r * kT + threadIdx.x;
        mask[r] = __ballot_sync(0xffffffffu, k < valid && ((x[r] >> bit) & 1u));
        if (lane() == 0) cnt[r * kW + wid] = __popc(mask[r]);
    }
    __syncthreads();
    // tile-local exclusive prefix of the 64 counts (round-major: position
    // order) by warp 0, then the zeros before the tile by look-back
    if (wid == 0) {
        const u32 c0 = cnt[2 * lane()], c1 = cnt[2 * lane() + 1];
        u32 incl = c0 + c1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const u32 y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane() >= static_cast<u32>(o)) incl += y;
        }
        const u32 tz = valid - __shfl_sync(0xffffffffu, incl, 31);
        const u32 excl = incl - c0 - c1;
        __syncwarp();
        cnt[2 * lane()] = excl;
        cnt[2 * lane() + 1] = excl + c0;
        u32 before = 0;
        if (tile == 0) {
            if (lane() == 0) lb_publish(lb, 0, 2u, tz);
        } else {
            if (lane() == 0) lb_publish(lb, tile, 1u, tz);
            before = lb_prefix<AddOp>(lb, tile);
            if (lane() == 0) lb_publish(lb, tile, 2u, before + tz);
        }
        if (lane() == 0) {
            zeros_before_s = before;
            tile_zeros_s = tz;
            if (tile + 1 == lb.tiles && (m & 31u) == 0)
                level[m >> 5] = make_uint2(0u, static_cast<u32>(m) - *total_zeros);
            lb_done(lb, tile);
        }
    }
    __syncthreads();
    const u32 tz = tile_zeros_s;
    const u32 ones_before_tile = static_cast<u32>(base) - zeros_before_s;
    // the split tile in shared memory: zeros, then ones, each in order
#pragma unroll
    for (u32 r = 0; r < kItems; ++r) {
        const u32 k = r * kT + threadIdx.x;
        const u32 ob = cnt[r * kW + wid];  // ones of the tile before this warp's 32
        if (k < valid) {
            const u32 one_rank = ob + __popc(mask[r] & ((1u << lane()) - 1u));
            stage[((x[r] >> bit) & 1u) ? tz + one_rank : k - one_rank] = x[r];
            if (lane() == 0) level[(base + k) >> 5] = make_uint2(mask[r], ones_before_tile + ob);
        }
    }
    __syncthreads();
    const u32 Z = *total_zeros;
    const u32 zeros_before = zeros_before_s;
#pragma unroll
    for (u32 r = 0; r < kItems; ++r) {
        const u32 k = r * kT + threadIdx.x;
        if (k < valid)
            out[k < tz ? zeros_before + k : Z + ones_before_tile + (k - tz)] = stage[k];
    }
}

__device__ __forceinline__ u32 rank1(const uint2* level, u32 x)
{
    const uint2 wv = level[x >> 5];
    return wv.y + __popc(wv.x & ((1u << (x & 31u)) - 1u));
}

// #{u < hi : value(u) > v} on the wavelet matrix (levels bits-1 .. 0)
__device__ __forceinline__ u32 count_greater(const uint2* levels, u64 words, u32 bits,
                                             const u32* zeros, u32 v, u32 hi)
{
    u32 lo = 0, cnt = 0;
    for (int l = static_cast<int>(bits) - 1; l >= 0; --l) {
        const uint2* L = levels + static_cast<u64>(l) * words;
        const u32 r_lo = rank1(L, lo), r_hi = rank1(L, hi);
        if (((v >> l) & 1u) == 0) {
            cnt += r_hi - r_lo;
            lo -= r_lo;
            hi -= r_hi;
        } else {
            lo = zeros[l] + r_lo;
            hi = zeros[l] + r_hi;
        }
    }
    return cnt;
}

// hit(i) and first-occurrence flags
__global__ void hit_kernel(const u32* prev, u64 m, u64 resident, u64 frames,
                           const uint2* levels, u64 words, u32 bits, const u32* zeros,
                           u32* hit, u32* first)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const u32 p = prev[i];
    first[i] = p == kNone ? 1u : 0u;
    u32 h = 0;
    if (i >= resident && p != kNone) {
        const u64 w = i - p - 1;  // accesses strictly between
        if (w < frames) {
            h = 1;
        } else {
            const u32 r = count_greater(levels, words, bits, zeros, p + 1, static_cast<u32>(i));
            h = w - r < frames ? 1u : 0u;  // distinct pages in between
        }
    }
    hit[i] = h;
}

__global__ void evict_kernel(const u32* hit, const u32* distinct_before, u64 m, u64 resident,
                             u64 frames, u32* evict)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= m) return;
    evict[i] = i >= resident && frames > 0 && !hit[i] && distinct_before[i] >= frames ? 1u : 0u;
}

// entry j leaves the cache (in order of j) when its page's next access misses
__global__ void leave_kernel(const u32* next, const u32* hit, u64 m, u32* leave)
{
    const u64 j = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= m) return;
    const u32 nx = next[j];
    leave[j] = nx == kNone || !hit[nx] ? 1u : 0u;
}

__global__ void compact_kernel(const u32* flag, const u32* pos, u64 m, u32* out)
{
    const u64 j = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j < m && flag[j]) out[pos[j]] = static_cast<u32>(j);
}

// residency starts (misses) and writes, as position+1 in page-sorted order
__global__ void dirty_marks_kernel(const u32* sk, const u32* si, const u32* hit, const u32* w,
                                   u64 m, u32* start_mark, u32* write_mark)
{
    const u64 k = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (k >= m) return;
    const u32 j = si[k];
    const bool start = k == 0 || sk[k - 1] != sk[k] || !hit[j];
    start_mark[k] = start ? static_cast<u32>(k) + 1u : 0u;
    write_mark[k] = w[j] ? static_cast<u32>(k) + 1u : 0u;
}

__global__ void dirty_kernel(const u32* si, const u32* last_start, const u32* last_write, u64 m,
                             u32* dirty)
{
    const u64 k = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (k < m) dirty[si[k]] = last_write[k] >= last_start[k] ? 1u : 0u;
}

struct OutArgs {
    const u32* key;
    const u32* bidx;
    const u32* hit;
    const u32* evict;
    const u32* evict_rank;
    const u32* leave_list;
    const u32* dirty;
    const u32* leave_total;
    u64 m;
    u8* out_hit;
    u64* out_victim;
    u8* out_dirty;
    u32* in_hit;     // the same decisions for the media-action pass
    u32* in_victim;
    u32* in_dirty;
    u32* counters;  // [0] hits, [1] dirty evictions
};

__global__ void output_kernel(OutArgs a)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= a.m) return;
    const u32 b = a.bidx[i];
    if (b == kNone) return;
    u64 victim = ~u64{0};
    u32 vd = 0;
    if (a.evict[i] && a.evict_rank[i] < *a.leave_total) {
        const u32 j = a.leave_list[a.evict_rank[i]];
        victim = a.key[j];
        vd = a.dirty[j];
        if (vd) atomicAdd(&a.counters[1], 1u);
    }
    if (a.hit[i]) atomicAdd(&a.counters[0], 1u);
    if (a.out_hit) a.out_hit[b] = static_cast<u8>(a.hit[i]);
    if (a.out_victim) a.out_victim[b] = victim;
    if (a.out_dirty) a.out_dirty[b] = static_cast<u8>(vd);
    a.in_hit[b] = a.hit[i];
    a.in_victim[b] = victim == ~u64{0} ? kNone : static_cast<u32>(victim);
    a.in_dirty[b] = vd;
}

__global__ void status_kernel(const u32* st, u64 n, u8* out)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = static_cast<u8>(st[i]);
}

// the last `keep` of the L last occurrences, oldest first
__global__ void resident_kernel(const u32* next, const u32* live_pos, const u32* key,
                                const u32* dirty, u64 m, u32 live_total, u32 keep,
                                u32* res_page, u8* res_dirty)
{
    const u64 j = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= m || next[j] != kNone) return;
    const u32 r = live_pos[j];
    if (r + keep >= live_total) {
        const u32 slot = r - (live_total - keep);
        res_page[slot] = key[j];
        res_dirty[slot] = static_cast<u8>(dirty[j]);
    }
}

__global__ void live_kernel(const u32* next, u64 m, u32* live)
{
    const u64 j = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j < m) live[j] = next[j] == kNone ? 1u : 0u;
}

// ---------------------------------------------------------------- actions
// Media actions of the misses (request_dispatcher.cpp:107-126): the program
// of a dirty victim's page, then the read of the missed page, each one LRU
// page at its media address; the read after a program is chained to it.
__global__ void act_count_kernel(const u32* status, const u32* hit, const u32* dirty, u64 n,
                                 u32* nact)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) nact[i] = status[i] == kModeled && !hit[i] ? 1u + (dirty[i] ? 1u : 0u) : 0u;
}

__global__ void act_build_kernel(const u32* status, const u32* hit, const u32* victim,
                                 const u32* dirty, const u32* page, const u32* pos,
                                 const u64* arrival, u64 n, u32 shift, u32 page_bytes,
                                 u64* addr, u32* bytes, u8* op, u64* arr, u32* chain)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n || status[i] != kModeled || hit[i]) return;
    u64 k = pos[i];
    const u64 a = arrival[i];
    u32 feed = kNone;
    if (dirty[i]) {
        addr[k] = static_cast<u64>(victim[i]) << shift;
        bytes[k] = page_bytes;
        op[k] = 1;
        arr[k] = a;
        chain[k] = kNone;
        feed = static_cast<u32>(k);
        ++k;
    }
    addr[k] = static_cast<u64>(page[i]) << shift;
    bytes[k] = page_bytes;
    op[k] = 0;
    arr[k] = a;
    chain[k] = feed;
}

__global__ void chained_flag_kernel(const u32* chain, u64 count, u32* flag)
{
    const u64 k = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (k < count) flag[k] = chain[k] != kNone ? 1u : 0u;
}

// One fixed-point round: each chained read starts no earlier than its
// program's completion.  Raises only ever increase an arrival (completions
// are monotone in the arrivals), so max(current, completion) is the read's
// arrival max(access arrival, completion).
__global__ void raise_kernel(const u32* chained, u64 count, const u32* chain, const u64* done,
                             u64* arrival, u32* changed)
{
    const u64 q = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (q >= count) return;
    const u32 k = chained[q];
    const u64 need = done[chain[k]];
    if (need > arrival[k]) {
        arrival[k] = need;
        *changed = 1u;
    }
}

// completion of each access: its read, or its arrival when served from HBM
// (hit) or not a capacity access
__global__ void act_result_kernel(const u32* status, const u32* hit, const u32* dirty,
                                  const u32* pos, const u64* arrival, const u64* act_done,
                                  u64 n, u64* done, u64* latency)
{
    const u64 i = static_cast<u64>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const u64 a = arrival[i];
    u64 d = a;
    if (status[i] == kModeled && !hit[i]) d = act_done[pos[i] + (dirty[i] ? 1u : 0u)];
    if (done) done[i] = d;
    if (latency) latency[i] = d - a;
}

// ---------------------------------------------------------------- CLOCK
// Second-chance CLOCK, the reference runtime's policy: HbmCache
// (src/cuda_runtime/hbm_cache.cpp) as CapacityPageService::resolve
// (capacity_page_service.cpp:97-210) drives it, one page reference at a
// time.  A resident page is a hit: its reference bit is set (resolve,
// 41-52), and a write sets its dirty bit (mark_dirty, 80-94).  A miss takes
// the lowest free frame (free_frame, 101-110); once every frame holds a
// page, begin_eviction_locked (131-175) walks the hand over the frames,
// clearing set reference bits, and evicts the first frame whose bit is
// clear, leaving the hand one past it.  publish (21-39) places the new page
// referenced and clean; a write marks it dirty.
//
// The policy is sequential by definition (each eviction depends on every
// reference bit the earlier accesses left), so one warp walks the batch in
// order, with its 32 lanes hiding the memory latency:
//   * the page -> frame lookups of 32 accesses are loaded at once, and each
//     decision updates the lanes whose page it placed or evicted;
//   * the lanes hold a window of 32 consecutive frames (reference bit,
//     page, dirty bit) from the hand on: a hand walk is a ballot over the
//     window, and a run of misses consumes the window without new loads;
//   * stores go straight out (the warp reads back only what it wrote after
//     a __syncwarp).
struct ClockArgs {
    const u32* valid;   // per access: 1 = capacity access
    const u32* page;    // per access: LRU page
    const u8* op;
    u64 n;
    u64 frames;
    u32* table;         // page -> frame, kNone = not resident
    u32* fpage;         // frame -> page
    u8* ref;
    u8* dirty;
    u64* state;         // [0] hand, [1] frames in use
    u32* ahit;          // per access decisions (media-action pass)
    u32* avictim;
    u32* adirty;
    u8* out_hit;
    u64* out_victim;
    u8* out_dirty;
    u32* counters;      // [0] hits, [1] dirty evictions, [2] evictions, [3] error,
                        // [4] capacity accesses
};

__global__ void __launch_bounds__(32) clock_kernel(const ClockArgs a)
{
    const u32 lane = threadIdx.x;
    const u64 F = a.frames;
    u64 hand = a.state[0], used = a.state[1];
    u32 hits = 0, dirty_ev = 0, evictions = 0, seen = 0;
    // the window: frames w0 + lane (mod F) for lanes below wn
    bool window = false;
    u64 w0 = 0;
    u32 wn = 0;
    u32 wref = 0, wpage = 0, wdirty = 0;
    auto in_window = [&](u64 f, u32& slot) {
        if (!window) return false;
        const u64 d = f >= w0 ? f - w0 : f + F - w0;
        slot = static_cast<u32>(d);
        return d < wn;
    };
    for (u64 i0 = 0; i0 < a.n; i0 += 32) {
        const u64 i = i0 + lane;
        const bool live = i < a.n && a.valid[i];
        const u32 my_page = live ? a.page[i] : kNone;
        const u32 my_w = live ? a.op[i] : 0u;
        u32 my_frame = live ? a.table[my_page] : kNone;
        const u32 count = static_cast<u32>(a.n - i0 < 32 ? a.n - i0 : 32);
        for (u32 j = 0; j < count; ++j) {
            const u32 p = __shfl_sync(0xffffffffu, my_page, j);
            if (p == kNone) continue;  // not a capacity access (uniform)
            ++seen;
            const u32 w = __shfl_sync(0xffffffffu, my_w, j);
            const u32 f = __shfl_sync(0xffffffffu, my_frame, j);
            const u64 idx = i0 + j;
            u32 slot;
            if (f != kNone) {  // hit
                if (lane == 0) {
                    a.ref[f] = 1;
                    if (w) a.dirty[f] = 1;
                    a.ahit[idx] = 1;
                    a.avictim[idx] = kNone;
                    a.adirty[idx] = 0;
                    if (a.out_hit) a.out_hit[idx] = 1;
                    if (a.out_victim) a.out_victim[idx] = ~u64{0};
                    if (a.out_dirty) a.out_dirty[idx] = 0;
                }
                if (in_window(f, slot) && lane == slot) {
                    wref = 1;
                    if (w) wdirty = 1;
                }
                ++hits;
                continue;
            }
            u64 target;
            u32 victim = kNone, vd = 0;
            if (used < F) {
                target = used++;
            } else {
                // the hand walk ends within two sweeps (the first clears
                // every reference bit it passes); the cap only guards it
                const u64 cap = 2 * (F / 32 + 2);
                for (u64 step = 0;; ++step) {
                    u32 at;
                    if (!in_window(hand, at)) {
                        __syncwarp();
                        w0 = hand;
                        wn = static_cast<u32>(F < 32 ? F : 32);
                        const u64 fl = (w0 + lane) % F;
                        wref = lane < wn ? a.ref[fl] : 1u;
                        wpage = lane < wn ? a.fpage[fl] : kNone;
                        wdirty = lane < wn ? a.dirty[fl] : 0u;
                        window = true;
                        at = 0;
                    }
                    const u32 clear = __ballot_sync(0xffffffffu, lane >= at && lane < wn &&
                                                                     wref == 0);
                    if (clear) {
                        const u32 z = __ffs(clear) - 1;
                        if (lane >= at && lane < z && wref) {  // second chances spent
                            wref = 0;
                            a.ref[(w0 + lane) % F] = 0;
                        }
                        target = (w0 + z) % F;
                        victim = __shfl_sync(0xffffffffu, wpage, z);
                        vd = __shfl_sync(0xffffffffu, wdirty, z);
                        hand = (target + 1) % F;
                        break;
                    }
                    if (lane >= at && lane < wn && wref) {
                        wref = 0;
                        a.ref[(w0 + lane) % F] = 0;
                    }
                    hand = (w0 + wn) % F;
                    window = false;
                    if (step > cap) {  // cannot happen: record it, take the hand's frame
                        if (lane == 0) a.counters[3] = 1;
                        target = hand;
                        victim = a.fpage[hand];
                        vd = a.dirty[hand];
                        hand = (hand + 1) % F;
                        break;
                    }
                }
                ++evictions;
                if (vd) ++dirty_ev;
                if (lane == 0) a.table[victim] = kNone;
                if (my_page == victim) my_frame = kNone;
            }
            if (lane == 0) {
                a.fpage[target] = p;
                a.ref[target] = 1;
                a.dirty[target] = w ? 1 : 0;
                a.table[p] = static_cast<u32>(target);
                a.ahit[idx] = 0;
                a.avictim[idx] = victim;
                a.adirty[idx] = vd;
                if (a.out_hit) a.out_hit[idx] = 0;
                if (a.out_victim) a.out_victim[idx] = victim == kNone ? ~u64{0} : victim;
                if (a.out_dirty) a.out_dirty[idx] = static_cast<u8>(vd);
            }
            if (in_window(target, slot) && lane == slot) {
                wref = 1;
                wpage = p;
                wdirty = w ? 1 : 0;
            }
            if (my_page == p) my_frame = static_cast<u32>(target);
        }
        __syncwarp();
    }
    if (lane == 0) {
        a.state[0] = hand;
        a.state[1] = used;
        a.counters[0] = hits;
        a.counters[1] = dirty_ev;
        a.counters[2] = evictions;
        a.counters[4] = seen;
    }
}

inline unsigned blocks(u64 n) { return static_cast<unsigned>((n + kT - 1) / kT); }

}  // namespace

void capacity_destroy(CapacityState* c)
{
    if (!c) return;
    void* ptrs[] = {c->res_page, c->res_dirty, c->key, c->w, c->bidx, c->sk, c->si, c->tk,
                    c->ti, c->prev, c->next, c->cur, c->nxt, c->levels, c->hit, c->a,
                    c->b, c->c, c->d, c->tile_sums, c->valid, c->status, c->counts,
                    c->apage, c->ahit, c->avictim, c->adirty, c->anact, c->apos,
                    c->act_addr, c->act_bytes, c->act_op, c->act_arr, c->act_chain,
                    c->act_done, c->act_lat, c->act_status, c->chained, c->chained_flag,
                    c->chained_pos, c->media_range, c->clk_table, c->clk_page, c->clk_ref,
                    c->clk_dirty, c->clk_state, c->snap, c->lb_state, c->lb_misc};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    delete c;
}

}  // namespace hbfb

using namespace hbfb;

namespace {

constexpr std::uint32_t kCapCounts = 64;  // device result words

struct CGuard {
    explicit CGuard(hbfsim_context* c) : lock(c->mu) { cudaSetDevice(c->device); }
    std::lock_guard<std::mutex> lock;
};

std::uint32_t bits_for(std::uint64_t v)
{
    std::uint32_t b = 1;
    while (b < 32 && (std::uint64_t{1} << b) <= v) ++b;
    return b;
}

int ensure_scratch(CapacityState* s, std::uint64_t need)
{
    if (need <= s->capacity_m) return HBFSIM_OK;
    // headroom: batches of a run grow slowly (appends), and regrowing costs
    // a free and an allocation of every array
    const std::uint64_t m = std::max<std::uint64_t>(need + need / 4, 1 << 16);
    const std::uint64_t words = m / 32 + 2;
    const std::uint64_t tiles = (m + kTile - 1) / kTile;
    if (grow(&s->key, m) || grow(&s->w, m) || grow(&s->bidx, m) || grow(&s->sk, m) ||
        grow(&s->si, m) || grow(&s->tk, m) || grow(&s->ti, m) || grow(&s->prev, m) ||
        grow(&s->next, m) || grow(&s->cur, m) || grow(&s->nxt, m) ||
        grow(&s->levels, 32 * words) || grow(&s->hit, m) || grow(&s->a, m) ||
        grow(&s->b, m) || grow(&s->c, m) || grow(&s->d, m) || grow(&s->valid, m) ||
        grow(&s->status, m) || grow(&s->tile_sums, 256 * tiles) ||
        grow(&s->apage, m) || grow(&s->ahit, m) || grow(&s->avictim, m) ||
        grow(&s->adirty, m) || grow(&s->anact, m) || grow(&s->apos, m))
        return HBFSIM_CUDA_ERROR;
    s->tile_sums_words = 256 * tiles;
    // look-back status words: the longest scan is over m values
    if (grow(&s->lb_state, tiles + 1) || grow(&s->lb_misc, 4) ||
        cudaMemset(s->lb_state, 0, 8 * (tiles + 1)) != cudaSuccess ||
        cudaMemset(s->lb_misc, 0, 16) != cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    s->lb_tiles = tiles + 1;
    s->lb_tag = 0;
    s->capacity_m = m;
    return HBFSIM_OK;
}

// Single-pass scan of n values (exclusive or inclusive, in place allowed);
// the total goes to *total_dev when given.
template <class Op>
cudaError_t lb_scan(CapacityState* s, const u32* in, u32* out, u64 n, bool inclusive,
                    u32* total_dev, cudaStream_t st)
{
    if (n == 0) {
        if (total_dev) return cudaMemsetAsync(total_dev, 0, 4, st);
        return cudaSuccess;
    }
    const u64 tiles = (n + kTile - 1) / kTile;
    if (tiles > s->lb_tiles) return cudaErrorInvalidValue;
    if (++s->lb_tag >= (1u << 30)) {  // tags are 30 bits: start over on clean words
        const cudaError_t e = cudaMemsetAsync(s->lb_state, 0, 8 * s->lb_tiles, st);
        if (e != cudaSuccess) return e;
        s->lb_tag = 1;
    }
    const LookBack lb{s->lb_state, s->lb_misc, s->lb_tag, static_cast<u32>(tiles)};
    lb_scan_kernel<Op><<<static_cast<unsigned>(tiles), kT, 0, st>>>(in, out, n,
                                                                   inclusive ? 1 : 0,
                                                                   total_dev, lb);
    return cudaGetLastError();
}

LookBack next_lookback(CapacityState* s, u64 tiles, cudaStream_t st)
{
    if (++s->lb_tag >= (1u << 30)) {
        cudaMemsetAsync(s->lb_state, 0, 8 * s->lb_tiles, st);
        s->lb_tag = 1;
    }
    return LookBack{s->lb_state, s->lb_misc, s->lb_tag, static_cast<u32>(tiles)};
}

// Reads device words to the host after the stream's work, with the
// look-back error word (set when a wait gave up): HBFSIM_TIMEOUT then.
int sync_read(CapacityState* s, void* dst, const void* src, std::size_t bytes, cudaStream_t st)
{
    u32 err = 0;
    if (bytes) cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(&err, s->lb_misc + 1, 4, cudaMemcpyDeviceToHost, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) return HBFSIM_CUDA_ERROR;
    return err ? HBFSIM_TIMEOUT : HBFSIM_OK;
}

// exclusive (or inclusive) add-scan with the total written to *total_dev
cudaError_t scan_add(CapacityState* s, const u32* in, u32* out, u64 n, bool inclusive,
                     u32* total_dev, cudaStream_t st)
{
    return lb_scan<AddOp>(s, in, out, n, inclusive, total_dev, st);
}

bool aligned16(const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

// Times the media actions of the batch's misses with the context's die
// model, in batch order, and writes each access's completion: one timing
// batch of all actions per fixed-point round (below).
int time_actions(hbfsim_context* ctx, const hbfsim_capacity_batch_v1* b, cudaStream_t st)
{
    CapacityState* s = ctx->capacity;
    const std::uint64_t n = b->count;
    u32* cnt = s->counts;
    act_count_kernel<<<blocks(n), kT, 0, st>>>(s->status, s->ahit, s->adirty, n, s->anact);
    scan_add(s, s->anact, s->apos, n, false, cnt + 8, st);
    std::uint32_t actions = 0;
    if (const int rc = sync_read(s, &actions, cnt + 8, 4, st)) return rc;
    if (actions > 2 * n) return HBFSIM_CUDA_ERROR;  // a read, after a dirty victim's program
    if (actions > s->act_capacity) {
        const std::uint64_t cap = actions + actions / 4 + 1024;
        if (grow(&s->act_addr, cap) || grow(&s->act_bytes, cap) || grow(&s->act_op, cap) ||
            grow(&s->act_arr, cap) || grow(&s->act_chain, cap) || grow(&s->act_done, cap) ||
            grow(&s->act_lat, cap) || grow(&s->act_status, cap) || grow(&s->chained, cap) ||
            grow(&s->chained_flag, cap) || grow(&s->chained_pos, cap)) {
            s->act_capacity = 0;
            return HBFSIM_CUDA_ERROR;
        }
        s->act_capacity = cap;
    }
    if (actions) {
        act_build_kernel<<<blocks(n), kT, 0, st>>>(s->status, s->ahit, s->avictim, s->adirty,
                                                    s->apage, s->apos, b->arrival_ns, n,
                                                    s->page_shift, 1u << s->page_shift,
                                                    s->act_addr, s->act_bytes, s->act_op,
                                                    s->act_arr, s->act_chain);
        chained_flag_kernel<<<blocks(actions), kT, 0, st>>>(s->act_chain, actions,
                                                             s->chained_flag);
        scan_add(s, s->chained_flag, s->chained_pos, actions, false, cnt + 9, st);
        compact_kernel<<<blocks(actions), kT, 0, st>>>(s->chained_flag, s->chained_pos, actions,
                                                       s->chained);
        std::uint32_t q = 0;
        if (const int rc = sync_read(s, &q, cnt + 9, 4, st)) return rc;
        if (q > actions) return HBFSIM_CUDA_ERROR;
        BatchIO io{};
        io.address = s->act_addr;
        io.bytes = s->act_bytes;
        io.op = s->act_op;
        io.arrival = s->act_arr;
        io.done = s->act_done;
        io.latency = s->act_lat;
        io.status = s->act_status;
        io.n = actions;
        io.aligned = aligned16(io.address) && aligned16(io.bytes) && aligned16(io.op) &&
                     aligned16(io.arrival) && aligned16(io.done) && aligned16(io.latency) &&
                     aligned16(io.status);
        // Fixed point: time every action with the chained reads' current
        // arrivals, raise each chained read to its program's completion,
        // and repeat until no arrival moves.  Each round starts from the
        // batch's initial die state (the timing kernels read one state
        // buffer and write the other) and from the saved counters, last
        // arrival and die activity, so the final round counts once.  The
        // rounds converge to the one-at-a-time walk of the actions in batch
        // order (every action depends only on earlier ones), but a raise
        // can delay later programs of its channel and so move later chained
        // reads: under a deep queue each round settles little more than one
        // program.  After kMaxRounds the batch is timed in pieces instead:
        // every chained read starts a piece, its arrival raised to its
        // program's completion (computed by an earlier piece) just before
        // the piece runs -- pieces in batch order, each in parallel.
        constexpr std::uint32_t kMaxRounds = 3;
        constexpr std::uint32_t kMaxPieces = 1u << 20;
        const int cur0 = ctx->cur;
        const std::uint64_t act_words = ctx->d_die_read_bytes ? 2ull * ctx->C * ctx->D : 0;
        const std::uint64_t need = sizeof(DevCounters) + 8 + 8 * act_words;
        if (need > s->snap_bytes) {
            if (s->snap) cudaFree(s->snap);
            s->snap = nullptr;
            s->snap_bytes = 0;
            if (cudaMalloc(&s->snap, need) != cudaSuccess) return HBFSIM_CUDA_ERROR;
            s->snap_bytes = need;
        }
        unsigned char* snap_counters = s->snap;
        unsigned char* snap_last = snap_counters + sizeof(DevCounters);
        unsigned char* snap_act = snap_last + 8;
        auto save = [&](bool restore) {
            auto copy = [&](void* a, void* b, std::uint64_t bytes) {
                cudaMemcpyAsync(restore ? a : b, restore ? b : a, bytes,
                                cudaMemcpyDeviceToDevice, st);
            };
            copy(ctx->d_counters, snap_counters, sizeof(DevCounters));
            copy(ctx->d_last_arrival, snap_last, 8);
            if (act_words) {
                copy(ctx->d_die_read_bytes, snap_act, 4 * act_words);
                copy(ctx->d_die_writes, snap_act + 4 * act_words, 4 * act_words);
            }
        };
        if (q) save(false);
        bool converged = q == 0;
        std::uint32_t round = 0;
        for (; round < (q ? kMaxRounds : 1u); ++round) {
            if (round) {
                save(true);
                ctx->cur = cur0;
            }
            const int rc = run_media_batch(ctx, io, s->media_range, 1, st);
            if (rc != HBFSIM_OK) return rc;
            if (!q) break;
            cudaMemsetAsync(cnt + 10, 0, 4, st);
            raise_kernel<<<blocks(q), kT, 0, st>>>(s->chained, q, s->act_chain, s->act_done,
                                                   s->act_arr, cnt + 10);
            std::uint32_t changed = 0;
            cudaMemcpyAsync(&changed, cnt + 10, 4, cudaMemcpyDeviceToHost, st);
            if (cudaStreamSynchronize(st) != cudaSuccess) return HBFSIM_CUDA_ERROR;
            if (!changed) {
                converged = true;
                ++round;
                break;
            }
        }
        s->rounds_last = round;
        s->walked_last = 0;
        s->pieces_last = 0;
        if (!converged && q <= kMaxPieces) {
            save(true);
            ctx->cur = cur0;
            std::vector<std::uint32_t> starts(q);
            if (cudaMemcpy(starts.data(), s->chained, 4ull * q, cudaMemcpyDeviceToHost) !=
                cudaSuccess)
                return HBFSIM_CUDA_ERROR;
            std::vector<std::uint64_t> cuts{0};
            for (std::uint32_t v : starts)
                if (v != 0) cuts.push_back(v);
            cuts.push_back(actions);
            for (std::size_t k = 0; k + 1 < cuts.size(); ++k) {
                const std::uint64_t lo = cuts[k], hi = cuts[k + 1];
                if (hi <= lo) continue;
                if (launch_chain_fixup(s->act_arr, s->act_done, s->act_chain, lo, st) !=
                    cudaSuccess)
                    return HBFSIM_CUDA_ERROR;
                BatchIO piece = io;
                piece.address = s->act_addr + lo;
                piece.bytes = s->act_bytes + lo;
                piece.op = s->act_op + lo;
                piece.arrival = s->act_arr + lo;
                piece.done = s->act_done + lo;
                piece.latency = s->act_lat + lo;
                piece.status = s->act_status + lo;
                piece.n = hi - lo;
                piece.aligned = aligned16(piece.address) && aligned16(piece.bytes) &&
                                aligned16(piece.op) && aligned16(piece.arrival) &&
                                aligned16(piece.done) && aligned16(piece.latency) &&
                                aligned16(piece.status);
                const int rc = run_media_batch(ctx, piece, s->media_range, 1, st);
                if (rc != HBFSIM_OK) return rc;
                ++s->pieces_last;
            }
            converged = true;
        }
        if (!converged) {
            s->walked_last = 1;
            save(true);
            ctx->cur = cur0;
            const DecodeParams dp = media_decode_params(ctx, s->media_range, 1);
            const std::uint64_t words = static_cast<std::uint64_t>(ctx->C) * ctx->K;
            if (launch_chain_sequential(dp, context_timing_params(ctx), s->act_addr,
                                        s->act_bytes, s->act_op, s->act_arr, s->act_chain,
                                        actions, ctx->K, ctx->d_state[ctx->cur],
                                        ctx->d_state[1 - ctx->cur], words, s->act_done,
                                        s->act_lat, s->act_status, st) != cudaSuccess)
                return HBFSIM_CUDA_ERROR;
            ctx->cur = 1 - ctx->cur;
        }
    }
    act_result_kernel<<<blocks(n), kT, 0, st>>>(s->status, s->ahit, s->adirty, s->apos,
                                                 b->arrival_ns, s->act_done, n, b->done_ns,
                                                 b->latency_ns);
    return cudaStreamSynchronize(st) == cudaSuccess ? HBFSIM_OK : HBFSIM_CUDA_ERROR;
}

// CLOCK decisions of one batch (clock_kernel), then the media actions.
int run_clock(hbfsim_context* ctx, const hbfsim_capacity_batch_v1* b, cudaStream_t st)
{
    CapacityState* s = ctx->capacity;
    const std::uint64_t n = b->count;
    if (ensure_scratch(s, n) != HBFSIM_OK) return HBFSIM_CUDA_ERROR;
    u32* cnt = s->counts;
    cudaMemsetAsync(cnt, 0, 4 * kCapCounts, st);
    cap_classify_kernel<<<blocks(n), kT, 0, st>>>(ctx->d_ranges,
                                                   static_cast<u32>(ctx->ranges.size()),
                                                   b->address, b->bytes, b->operation, n,
                                                   s->page_shift, s->apage, s->valid, s->status);
    if (b->status) status_kernel<<<blocks(n), kT, 0, st>>>(s->status, n, b->status);
    if (b->hit) cudaMemsetAsync(b->hit, 0, n, st);
    if (b->victim_page) cudaMemsetAsync(b->victim_page, 0xff, 8 * n, st);
    if (b->victim_dirty) cudaMemsetAsync(b->victim_dirty, 0, n, st);
    ClockArgs a{};
    a.valid = s->valid;
    a.page = s->apage;
    a.op = b->operation;
    a.n = n;
    a.frames = s->frames;
    a.table = s->clk_table;
    a.fpage = s->clk_page;
    a.ref = s->clk_ref;
    a.dirty = s->clk_dirty;
    a.state = s->clk_state;
    a.ahit = s->ahit;
    a.avictim = s->avictim;
    a.adirty = s->adirty;
    a.out_hit = b->hit;
    a.out_victim = b->victim_page;
    a.out_dirty = b->victim_dirty;
    a.counters = cnt;
    clock_kernel<<<1, 32, 0, st>>>(a);
    std::uint32_t host_cnt[5] = {0, 0, 0, 0, 0};
    std::uint64_t used = 0;
    cudaMemcpyAsync(host_cnt, cnt, sizeof host_cnt, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(&used, s->clk_state + 1, 8, cudaMemcpyDeviceToHost, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) return HBFSIM_CUDA_ERROR;
    if (host_cnt[3]) return HBFSIM_CUDA_ERROR;
    s->resident = used;
    if (b->done_ns || b->latency_ns) {
        const int rc = time_actions(ctx, b, st);
        if (rc != HBFSIM_OK) return rc;
    }
    ++s->calls;
    s->accesses += host_cnt[4];
    s->hits += host_cnt[0];
    s->misses += host_cnt[4] - host_cnt[0];
    s->dirty_evictions += host_cnt[1];
    s->evictions += host_cnt[2];
    return cudaGetLastError() == cudaSuccess ? HBFSIM_OK : HBFSIM_CUDA_ERROR;
}

int run_capacity(hbfsim_context* ctx, const hbfsim_capacity_batch_v1* b, cudaStream_t st)
{
    CapacityState* s = ctx->capacity;
    if (s->policy == HBFSIM_CAPACITY_POLICY_CLOCK) return run_clock(ctx, b, st);
    const std::uint64_t n = b->count;
    const std::uint64_t resident = s->resident;
    if (ensure_scratch(s, resident + n) != HBFSIM_OK) return HBFSIM_CUDA_ERROR;
    u32* cnt = s->counts;  // [0] valid total, [1] hits, [2] dirty ev, [3] Z, [4] distinct,
                           // [5] evictions, [6] leave total, [7] live total, [8..] zeros/level
    cudaMemsetAsync(cnt, 0, 4 * kCapCounts, st);
    // 1. classify the batch; capacity accesses get sequence positions
    cap_classify_kernel<<<blocks(n), kT, 0, st>>>(ctx->d_ranges,
                                                   static_cast<u32>(ctx->ranges.size()),
                                                   b->address, b->bytes, b->operation, n,
                                                   s->page_shift, s->apage, s->valid, s->status);
    scan_add(s, s->valid, s->a, n, false, cnt + 0, st);
    std::uint32_t valid_total = 0;
    if (const int rc = sync_read(s, &valid_total, cnt + 0, 4, st)) return rc;
    if (valid_total > n) return HBFSIM_CUDA_ERROR;
    const std::uint64_t m = resident + valid_total;
    if (b->status) status_kernel<<<blocks(n), kT, 0, st>>>(s->status, n, b->status);
    // 2. the sequence: resident list, then the capacity accesses
    cap_build_kernel<<<blocks(std::max(n, resident)), kT, 0, st>>>(
        s->res_page, s->res_dirty, resident, s->apage, b->operation, s->valid, s->a, n, s->key,
        s->w, s->bidx);
    if (m == 0) {
        if (b->hit) cudaMemsetAsync(b->hit, 0, n, st);
        if (b->victim_page) cudaMemsetAsync(b->victim_page, 0xff, 8 * n, st);
        if (b->victim_dirty) cudaMemsetAsync(b->victim_dirty, 0, n, st);
        if (b->done_ns || b->latency_ns)  // nothing cached: every access keeps its arrival
            act_result_kernel<<<blocks(n), kT, 0, st>>>(s->status, s->ahit, s->adirty,
                                                         s->apos, b->arrival_ns, nullptr, n,
                                                         b->done_ns, b->latency_ns);
        return cudaStreamSynchronize(st) == cudaSuccess ? HBFSIM_OK : HBFSIM_CUDA_ERROR;
    }
    // 3. stable radix sort of (page, position)
    const std::uint64_t max_page = ctx->profile.capacity_bytes >> s->page_shift;
    const std::uint32_t key_bits = bits_for(max_page);
    const u32 tiles = static_cast<u32>((m + kTile - 1) / kTile);
    cudaMemcpyAsync(s->sk, s->key, 4 * m, cudaMemcpyDeviceToDevice, st);
    iota_kernel<<<blocks(m), kT, 0, st>>>(s->si, m);
    u32 *ik = s->sk, *iv = s->si, *ok = s->tk, *ov = s->ti;
    u32* hist = s->tile_sums;  // radix histograms [256][tiles]
    for (std::uint32_t shift = 0; shift < key_bits; shift += 8) {
        radix_hist_kernel<<<tiles, kT, 0, st>>>(ik, m, shift, hist, tiles);
        lb_scan<AddOp>(s, hist, hist, 256ull * tiles, false, nullptr, st);
        radix_scatter_kernel<<<tiles, kT, 0, st>>>(ik, iv, m, shift, hist, tiles, ok, ov);
        std::swap(ik, ok);
        std::swap(iv, ov);
    }
    // 4. previous / next access of the same page
    fill_kernel<<<blocks(m), kT, 0, st>>>(s->prev, m, kNone);
    fill_kernel<<<blocks(m), kT, 0, st>>>(s->next, m, kNone);
    link_kernel<<<blocks(m), kT, 0, st>>>(ik, iv, m, s->prev, s->next);
    // 5. wavelet matrix over prev + 1
    const std::uint32_t vbits = bits_for(m);
    const std::uint64_t words = m / 32 + 2;
    value_kernel<<<blocks(m), kT, 0, st>>>(s->prev, m, s->cur);
    u32* zeros_dev = cnt + 16;  // per level
    u32 *wc = s->cur, *wn = s->nxt;
    wm_bit_zeros_kernel<<<std::min<u32>(tiles, 4 * 148), kT, 0, st>>>(wc, m, vbits, zeros_dev);
    for (int l = static_cast<int>(vbits) - 1; l >= 0; --l) {
        uint2* level = s->levels + static_cast<std::uint64_t>(l) * words;
        wm_level_kernel<<<tiles, kT, 0, st>>>(wc, m, static_cast<u32>(l), zeros_dev + l, wn,
                                              level, next_lookback(s, tiles, st));
        std::swap(wc, wn);
    }
    // 6. hits, distinct pages before each access, evicting misses
    hit_kernel<<<blocks(m), kT, 0, st>>>(s->prev, m, resident, s->frames, s->levels, words,
                                         vbits, zeros_dev, s->hit, s->a);
    scan_add(s, s->a, s->b, m, false, cnt + 4, st);            // distinct before i
    evict_kernel<<<blocks(m), kT, 0, st>>>(s->hit, s->b, m, resident, s->frames, s->c);
    scan_add(s, s->c, s->d, m, false, cnt + 5, st);            // eviction rank
    // 7. entries that leave the cache, in order
    leave_kernel<<<blocks(m), kT, 0, st>>>(s->next, s->hit, m, s->a);
    scan_add(s, s->a, s->cur, m, false, cnt + 6, st);
    compact_kernel<<<blocks(m), kT, 0, st>>>(s->a, s->cur, m, s->nxt);
    // 8. dirty bits (page-sorted order; ik/iv hold the sorted pairs)
    u32* start_mark = ok;   // the sort's other buffers are free now
    u32* write_mark = ov;
    dirty_marks_kernel<<<blocks(m), kT, 0, st>>>(ik, iv, s->hit, s->w, m, start_mark,
                                                 write_mark);
    lb_scan<MaxOp>(s, start_mark, start_mark, m, true, nullptr, st);
    lb_scan<MaxOp>(s, write_mark, write_mark, m, true, nullptr, st);
    dirty_kernel<<<blocks(m), kT, 0, st>>>(iv, start_mark, write_mark, m, s->b);
    // 9. per-access outputs
    OutArgs oa{};
    oa.key = s->key;
    oa.bidx = s->bidx;
    oa.hit = s->hit;
    oa.evict = s->c;
    oa.evict_rank = s->d;
    oa.leave_list = s->nxt;
    oa.dirty = s->b;
    oa.leave_total = cnt + 6;
    oa.m = m;
    oa.out_hit = b->hit;
    oa.out_victim = b->victim_page;
    oa.out_dirty = b->victim_dirty;
    oa.in_hit = s->ahit;
    oa.in_victim = s->avictim;
    oa.in_dirty = s->adirty;
    oa.counters = cnt + 1;
    if (b->hit) cudaMemsetAsync(b->hit, 0, n, st);
    if (b->victim_page) cudaMemsetAsync(b->victim_page, 0xff, 8 * n, st);
    if (b->victim_dirty) cudaMemsetAsync(b->victim_dirty, 0, n, st);
    output_kernel<<<blocks(m), kT, 0, st>>>(oa);
    // 10. the new resident list
    live_kernel<<<blocks(m), kT, 0, st>>>(s->next, m, s->a);
    scan_add(s, s->a, s->cur, m, false, cnt + 7, st);
    std::uint32_t host_cnt[kCapCounts];
    if (const int rc = sync_read(s, host_cnt, cnt, 4 * kCapCounts, st)) return rc;
    if (host_cnt[7] > m) return HBFSIM_CUDA_ERROR;
    const std::uint32_t live_total = host_cnt[7];
    const std::uint32_t keep =
        static_cast<std::uint32_t>(std::min<std::uint64_t>(live_total, s->frames));
    resident_kernel<<<blocks(m), kT, 0, st>>>(s->next, s->cur, s->key, s->b, m, live_total,
                                              keep, s->res_page, s->res_dirty);
    if (cudaStreamSynchronize(st) != cudaSuccess) return HBFSIM_CUDA_ERROR;
    s->resident = keep;
    if (b->done_ns || b->latency_ns) {
        const int rc = time_actions(ctx, b, st);
        if (rc != HBFSIM_OK) return rc;
    }
    ++s->calls;
    s->accesses += valid_total;
    s->hits += host_cnt[1];
    s->misses += valid_total - host_cnt[1];
    s->evictions += host_cnt[5];
    s->dirty_evictions += host_cnt[2];
    return cudaGetLastError() == cudaSuccess ? HBFSIM_OK : HBFSIM_CUDA_ERROR;
}

}  // namespace

extern "C" {

int hbfsim_capacity_configure_v1(hbfsim_context* c, uint64_t frames, uint32_t page_bytes)
{
    if (!c) return HBFSIM_INVALID_ARGUMENT;
    CGuard g(c);
    if (page_bytes == 0) page_bytes = 4096;
    if (page_bytes < 512 || (page_bytes & (page_bytes - 1)) != 0 ||
        page_bytes > c->profile.page_bytes)
        return HBFSIM_INVALID_ARGUMENT;
    std::uint32_t shift = 0;
    while ((1u << shift) < page_bytes) ++shift;
    if ((c->profile.capacity_bytes >> shift) >= 0xffffffffull ||
        frames >= 0x7fffffffull)
        return HBFSIM_UNSUPPORTED;  // page ids and positions are 32-bit
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    if (c->capacity) capacity_destroy(c->capacity);
    auto* s = new CapacityState();
    c->capacity = s;
    s->frames = frames;
    s->page_shift = shift;
    DevRange media{};
    media.base = 0;
    media.length = c->profile.capacity_bytes;
    media.file_offset = 0;
    media.page_bytes = c->profile.page_bytes;
    media.mode = HBFSIM_RANGE_MODE_TIMING;
    media.permissions = 3;
    std::uint32_t page_log = 0;
    while ((std::uint64_t{1} << page_log) < c->profile.page_bytes) ++page_log;
    media.reserved = page_log;
    media.end = media.base + media.length;
    media.ok = 1;
    media.timing = 3;  // reads and writes
    if (grow(&s->res_page, frames) || grow(&s->res_dirty, frames) ||
        grow(&s->counts, kCapCounts) || grow(&s->media_range, 1) ||
        cudaMemcpy(s->media_range, &media, sizeof media, cudaMemcpyHostToDevice) != cudaSuccess) {
        capacity_destroy(s);
        c->capacity = nullptr;
        return HBFSIM_CUDA_ERROR;
    }
    return HBFSIM_OK;
}

int hbfsim_capacity_policy_v1(hbfsim_context* c, uint32_t policy)
{
    if (!c) return HBFSIM_INVALID_ARGUMENT;
    CGuard g(c);
    CapacityState* s = c->capacity;
    if (!s || (policy != HBFSIM_CAPACITY_POLICY_LRU && policy != HBFSIM_CAPACITY_POLICY_CLOCK))
        return HBFSIM_INVALID_ARGUMENT;
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    s->resident = 0;
    s->policy = policy;
    if (policy == HBFSIM_CAPACITY_POLICY_LRU) return HBFSIM_OK;
    if (s->frames == 0) return HBFSIM_INVALID_ARGUMENT;  // the reference cache needs a frame
    const std::uint64_t pages = (c->profile.capacity_bytes >> s->page_shift) + 1;
    if (grow(&s->clk_table, pages) || grow(&s->clk_page, s->frames) ||
        grow(&s->clk_ref, s->frames) || grow(&s->clk_dirty, s->frames) ||
        grow(&s->clk_state, 2) ||
        cudaMemset(s->clk_table, 0xff, 4 * pages) != cudaSuccess ||
        cudaMemset(s->clk_ref, 0, s->frames) != cudaSuccess ||
        cudaMemset(s->clk_dirty, 0, s->frames) != cudaSuccess ||
        cudaMemset(s->clk_state, 0, 16) != cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    s->table_pages = pages;
    return HBFSIM_OK;
}

int hbfsim_submit_capacity_batch_v1(hbfsim_context* c, const hbfsim_capacity_batch_v1* b,
                                    void* stream)
{
    if (!c || !b || b->struct_size != sizeof(hbfsim_capacity_batch_v1) ||
        b->version != HBFSIM_CAPACITY_BATCH_V1_VERSION)
        return HBFSIM_INVALID_ARGUMENT;
    if (b->count && (!b->address || !b->bytes || !b->operation)) return HBFSIM_INVALID_ARGUMENT;
    CGuard g(c);
    if (!c->capacity) return HBFSIM_INVALID_ARGUMENT;
    if (c->capacity->resident + b->count >= 0x7fffffffull) return HBFSIM_UNSUPPORTED;
    if (b->done_ns || b->latency_ns) {
        // the media actions are timed with the per-die model of one shard
        if (!b->arrival_ns) return HBFSIM_INVALID_ARGUMENT;
        if (c->mode != HBFSIM_MODEL_DIE_V1 || c->shard_count != 1) return HBFSIM_UNSUPPORTED;
    }
    if (b->count == 0) return HBFSIM_OK;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    return run_capacity(c, b, s);
}

int hbfsim_get_capacity_rounds_v1(hbfsim_context* c, uint32_t* rounds, uint64_t* pieces,
                                  uint32_t* walked)
{
    if (!c || !rounds || !pieces || !walked) return HBFSIM_INVALID_ARGUMENT;
    CGuard g(c);
    if (!c->capacity) return HBFSIM_INVALID_ARGUMENT;
    *rounds = c->capacity->rounds_last;
    *pieces = c->capacity->pieces_last;
    *walked = c->capacity->walked_last;
    return HBFSIM_OK;
}

int hbfsim_get_capacity_state_v1(hbfsim_context* c, uint64_t* resident_pages,
                                 uint8_t* resident_dirty, uint64_t count, uint64_t* resident)
{
    if (!c || !resident) return HBFSIM_INVALID_ARGUMENT;
    CGuard g(c);
    CapacityState* s = c->capacity;
    if (!s) return HBFSIM_INVALID_ARGUMENT;
    *resident = s->resident;
    if (!resident_pages && !resident_dirty) return HBFSIM_OK;
    if (count < s->resident) return HBFSIM_INVALID_ARGUMENT;
    std::vector<std::uint32_t> pages(s->resident);
    const bool clock = s->policy == HBFSIM_CAPACITY_POLICY_CLOCK;
    const u32* src_page = clock ? s->clk_page : s->res_page;   // CLOCK: frame order
    const u8* src_dirty = clock ? s->clk_dirty : s->res_dirty;
    if (cudaDeviceSynchronize() != cudaSuccess ||
        (s->resident && cudaMemcpy(pages.data(), src_page, 4 * s->resident,
                                   cudaMemcpyDeviceToHost) != cudaSuccess) ||
        (resident_dirty && s->resident &&
         cudaMemcpy(resident_dirty, src_dirty, s->resident, cudaMemcpyDeviceToHost) !=
             cudaSuccess))
        return HBFSIM_CUDA_ERROR;
    if (resident_pages)
        for (std::uint64_t k = 0; k < s->resident; ++k) resident_pages[k] = pages[k];
    return HBFSIM_OK;
}

}  // extern "C"

namespace hbfb {
void capacity_stats(const CapacityState* s, hbfsim_capacity_stats_v1* out)
{
    out->enabled = 1;
    out->page_bytes = std::uint64_t{1} << s->page_shift;
    out->logical_frame_count = s->frames;
    out->service_resolve_calls = s->accesses;
    out->service_resident_hits = s->hits;
    out->service_misses = s->misses;
    out->successful_backing_read_pages = s->misses;
    out->successful_backing_read_bytes = s->misses << s->page_shift;
    out->successful_resolve_evictions = s->evictions;
    out->successful_d2h_readback_pages = s->dirty_evictions;
    out->successful_d2h_readback_bytes = s->dirty_evictions << s->page_shift;
    out->service_ready_results = s->accesses;
}
}  // namespace hbfb
