// prefetch.cu -- the prefetch model as a sweep on the device: one warp per
// sweep cell.
//
// Reference: src/prefetch/prefetch_model.cpp simulate_prefetch (117-195) and
// include/hbfsim/prefetch_model.hpp.  Per access: compute time passes, the
// prefetcher may fetch a predicted page into a FIFO staging buffer, then the
// demand either takes its page from the buffer (waiting for it to land) or
// pays a media read.  Each cell is a sequential walk; a sweep runs its cells
// side by side, one warp each, all reading the same page stream (L2).
//
// Per warp, in shared memory: the Mersenne Twister state (the predictor's
// std::mt19937_64, twisted by the 32 lanes in two phases) and the staging
// buffer as slots {page, arrival, insertion number} with a stack of free
// slots; one pass of ballots over the live slots finds the predicted page,
// the demanded page and the oldest entry (a warp minimum of the insertion
// numbers), which is dropped before an insertion into a full buffer.  The media servers (prefetch_model.cpp:23-50) all take
// the same read latency and receive reads in non-decreasing issue time, so
// the server that frees first for the j-th read is the one that served read
// j - k: completion_j = max(issue_j, completion_{j-k}) + latency, a ring of
// the last k completions per cell (shared memory up to 256 servers, global
// scratch beyond).  The page stream is read 32 accesses at a time, one page
// per lane, and handed to each step by a shuffle.
#include "../../include/hbfsim/batch_v1.h"
#include "common.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

namespace hbfb {
namespace {

constexpr u32 kFull = 0xffffffffu;
constexpr u32 kMtWords = 312;
constexpr u32 kRingSmem = 256;   // completion rings up to this size live in shared memory
constexpr u64 kWrongPageBase = u64{1} << 60;   // prefetch_model.cpp:18

struct SweepArgs {
    const u64* pages;
    u64 n;
    const hbfsim_prefetch_cell_v1* cells;
    u32 count;
    u32 slots;              // staging slots per warp (multiple of 32)
    u32 warps;              // cells per CTA
    u64* ring;              // completion rings, cell c at ring_offset[c]
    const u64* ring_offset;
    hbfsim_prefetch_stats_v1* out;
};

// std::mt19937_64 (parameters of the C++ standard's [rand.predef]).
__device__ void mt_seed(u64* mt, u64 seed)
{
    if ((threadIdx.x & 31u) == 0) {
        u64 x = seed;
        mt[0] = x;
        for (u32 k = 1; k < kMtWords; ++k) {
            x = 6364136223846793005ull * (x ^ (x >> 62)) + k;
            mt[k] = x;
        }
    }
    __syncwarp();
}

__device__ __forceinline__ u64 mt_mix(u64 cur, u64 next, u64 far)
{
    const u64 y = (cur & 0xFFFFFFFF80000000ull) | (next & 0x7FFFFFFFull);
    return far ^ (y >> 1) ^ ((y & 1u) ? 0xB5026F5AA96619E9ull : 0ull);
}

// Both halves of the twist read the words they replace and their right
// neighbours, so each half computes into registers first, then writes.
__device__ void mt_twist(u64* mt)
{
    const u32 lane = threadIdx.x & 31u;
    u64 v[5];
#pragma unroll
    for (u32 t = 0; t < 5; ++t) {  // words 0..155: partners 156..311 still old
        const u32 k = lane + 32 * t;
        if (k < 156) v[t] = mt_mix(mt[k], mt[k + 1], mt[k + 156]);
    }
    __syncwarp();
#pragma unroll
    for (u32 t = 0; t < 5; ++t) {
        const u32 k = lane + 32 * t;
        if (k < 156) mt[k] = v[t];
    }
    __syncwarp();
#pragma unroll
    for (u32 t = 0; t < 5; ++t) {  // words 156..311: partners 0..155 already new
        const u32 k = 156 + lane + 32 * t;
        if (k < kMtWords) v[t] = mt_mix(mt[k], mt[(k + 1) % kMtWords], mt[k - 156]);
    }
    __syncwarp();
#pragma unroll
    for (u32 t = 0; t < 5; ++t) {
        const u32 k = 156 + lane + 32 * t;
        if (k < kMtWords) mt[k] = v[t];
    }
    __syncwarp();
}

// One uniform double in [0, 1) from one 64-bit draw, as the standard's
// generate_canonical<double, 53> computes it for a 2^64-range engine.
__device__ __forceinline__ double mt_canonical(u64* mt, u32& index)
{
    if (index >= kMtWords) {
        mt_twist(mt);
        index = 0;
    }
    u64 y = mt[index++];
    y ^= (y >> 29) & 0x5555555555555555ull;
    y ^= (y << 17) & 0x71D67FFFEDA60000ull;
    y ^= (y << 37) & 0xFFF7EEE000000000ull;
    y ^= y >> 43;
    const double r = __dmul_rn(__ull2double_rn(y), 0x1p-64);
    return r >= 1.0 ? 0x1.fffffffffffffp-1 : r;
}

// Slot of `page` among the live slots [0, hi), or -1.
__device__ __forceinline__ int buffer_find(const u64* page, const u32* seq, u32 hi, u64 p)
{
    const u32 lane = threadIdx.x & 31u;
    for (u32 base = 0; base < hi; base += 32) {
        const u32 s = base + lane;
        const u32 m = __ballot_sync(kFull, s < hi && seq[s] != 0 && page[s] == p);
        if (m) return static_cast<int>(base + __ffs(m) - 1);
    }
    return -1;
}

__global__ void __launch_bounds__(128) prefetch_sweep_kernel(const SweepArgs a)
{
    extern __shared__ __align__(16) u64 smem[];
    const u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const u32 cell = blockIdx.x * a.warps + warp;
    if (cell >= a.count) return;  // whole warps leave; the kernel has no block barrier
    const u32 S = a.slots;
    u64* mt = smem + static_cast<u64>(warp) * (kMtWords + kRingSmem + 3ull * S);
    u64* ring_smem = mt + kMtWords;
    u64* page = ring_smem + kRingSmem;
    u64* arr = page + S;
    u32* seq = reinterpret_cast<u32*>(arr + S);
    u32* free_stack = seq + S;  // free slots, lowest on top
    const hbfsim_prefetch_cell_v1 c = a.cells[cell];
    for (u32 s = lane; s < S; s += 32) {
        seq[s] = 0;
        free_stack[s] = S - 1 - s;
    }
    u32 free_top = S;
    mt_seed(mt, c.seed);
    u32 mt_index = kMtWords;
    const u32 capacity = c.buffer_pages ? c.buffer_pages : 1u;
    const u32 servers = c.max_in_flight ? c.max_in_flight : 1u;
    u64* ring = servers <= kRingSmem ? ring_smem : a.ring + a.ring_offset[cell];
    u32 ring_slot = 0;          // next server in round-robin order
    bool ring_full = false;     // every server has served a read
    u64 clock = 0, wrong = kWrongPageBase;
    u64 stall = 0, misses = 0, hits = 0, issued = 0, wasted = 0;
    u32 live = 0, hi = 0, next_seq = 1;
    const bool prefetching = c.policy != 0 && c.lead_distance > 0;
    u64 chunk_cur = 0, chunk_tgt = 0;

    auto media_issue = [&](u64 now) -> u64 {
        const u32 slot = ring_slot;
        const u64 earliest = ring_full ? ring[slot] : 0;  // one broadcast read
        const u64 done = (now > earliest ? now : earliest) + c.read_latency_ns;
        __syncwarp();
        if (lane == 0) ring[slot] = done;
        __syncwarp();
        if (++ring_slot == servers) {
            ring_slot = 0;
            ring_full = true;
        }
        return done;
    };

    // The stream in chunks of 32 accesses: lane j holds the page of access
    // base + j and of its prefetch target; the next chunk's loads are issued
    // before the current chunk's steps, so their latency is hidden.
    const u64 lead = c.lead_distance;
    auto load_chunk = [&](u64 base, u64& cur, u64& tgt) {
        const u64 i = base + lane;
        cur = i < a.n ? a.pages[i] : 0;
        tgt = i + lead < a.n ? a.pages[i + lead] : 0;
    };
    u64 next_cur = 0, next_tgt = 0;
    load_chunk(0, next_cur, next_tgt);
    for (u64 i = 0; i < a.n; ++i) {
        const u32 j = static_cast<u32>(i & 31u);
        if (j == 0) {
            const u64 cur = next_cur, tgt = next_tgt;
            if (i + 32 < a.n) load_chunk(i + 32, next_cur, next_tgt);
            chunk_cur = cur;
            chunk_tgt = tgt;
        }
        const u64 demand = __shfl_sync(kFull, chunk_cur, j);
        const u64 ahead = __shfl_sync(kFull, chunk_tgt, j);
        clock += c.compute_ns_per_access;
        int dslot = -1;
        bool scanned = false;
        if (prefetching) {
            const u64 target = i + lead;
            bool predict = false;
            u64 predicted = 0;
            if (c.policy == 1) {
                predicted = demand + 1;
                predict = true;
            } else if (target < a.n) {
                predicted = mt_canonical(mt, mt_index) < c.accuracy ? ahead : wrong++;
                predict = true;
            }
            // one pass over the live slots finds the predicted page, the
            // demanded page and the oldest entry
            int pslot = -1;
            u32 best = 0xffffffffu, best_slot = 0;
            for (u32 base = 0; base < hi; base += 32) {
                const u32 s_ = base + lane;
                const u32 q = s_ < hi ? seq[s_] : 0u;
                const u64 pg = page[s_];
                const u32 mp = __ballot_sync(kFull, q != 0 && predict && pg == predicted);
                const u32 md = __ballot_sync(kFull, q != 0 && pg == demand);
                if (mp) pslot = static_cast<int>(base + __ffs(mp) - 1);
                if (md) dslot = static_cast<int>(base + __ffs(md) - 1);
                if (q != 0 && q < best) {
                    best = q;
                    best_slot = s_;
                }
            }
            scanned = true;
            if (predict && pslot < 0) {
                const u64 landed = media_issue(clock);
                if (live == capacity) {
                    // full: drop the oldest entry first (the reference inserts,
                    // then drops the oldest; the new page is never the oldest,
                    // so the order does not matter), so that live entries fit
                    // in `capacity` slots
                    const u32 oldest = __reduce_min_sync(kFull, best);
                    const u32 owner = __ffs(__ballot_sync(kFull, best == oldest)) - 1;
                    const u32 e = __shfl_sync(kFull, best_slot, owner);
                    __syncwarp();
                    if (lane == 0) {
                        seq[e] = 0;
                        free_stack[free_top] = e;
                    }
                    __syncwarp();
                    ++free_top;
                    if (dslot == static_cast<int>(e)) dslot = -1;
                    --live;
                    ++wasted;
                }
                const u32 f = free_stack[free_top - 1];  // a free slot
                --free_top;
                __syncwarp();
                if (lane == 0) {
                    page[f] = predicted;
                    arr[f] = landed;
                    seq[f] = next_seq;
                }
                __syncwarp();
                ++next_seq;
                ++live;
                hi = f + 1 > hi ? f + 1 : hi;
                ++issued;
                if (predicted == demand) dslot = static_cast<int>(f);
            }
        }
        const int k = scanned ? dslot : buffer_find(page, seq, hi, demand);
        if (k >= 0) {
            const u64 landed = arr[k];
            __syncwarp();
            if (lane == 0) {
                seq[k] = 0;
                free_stack[free_top] = static_cast<u32>(k);
            }
            __syncwarp();
            ++free_top;
            --live;
            ++hits;
            if (landed > clock) {
                stall += landed - clock;
                clock = landed;
            }
        } else {
            const u64 landed = media_issue(clock);
            ++misses;
            stall += landed - clock;
            clock = landed;
        }
    }
    if (lane == 0) {
        hbfsim_prefetch_stats_v1 s{};
        s.total_ns = clock;
        s.stall_ns = stall;
        s.demand_accesses = a.n;
        s.demand_misses = misses;
        s.prefetch_hits = hits;
        s.prefetch_issued = issued;
        s.prefetch_wasted = wasted + live;  // left over, never used
        a.out[cell] = s;
    }
}

}  // namespace
}  // namespace hbfb

using namespace hbfb;

extern "C" int hbfsim_prefetch_sweep_v1(const uint64_t* pages, uint64_t count,
                                        const hbfsim_prefetch_cell_v1* cells,
                                        uint32_t cell_count, hbfsim_prefetch_stats_v1* out,
                                        void* stream)
{
    if ((count && !pages) || (cell_count && (!cells || !out))) return HBFSIM_INVALID_ARGUMENT;
    if (cell_count == 0) return HBFSIM_OK;
    if (count >= 0xfffffffeull) return HBFSIM_UNSUPPORTED;  // insertion numbers are 32-bit
    for (uint32_t k = 0; k < cell_count; ++k)
        if (cells[k].policy > 2) return HBFSIM_INVALID_ARGUMENT;
    if (count == 0) {
        for (uint32_t k = 0; k < cell_count; ++k) out[k] = hbfsim_prefetch_stats_v1{};
        return HBFSIM_OK;
    }
    std::uint32_t max_buffer = 1;
    std::vector<std::uint64_t> offset(cell_count);
    std::uint64_t ring_words = 0;
    for (uint32_t k = 0; k < cell_count; ++k) {
        max_buffer = std::max<std::uint32_t>(max_buffer, std::max<std::uint32_t>(1, cells[k].buffer_pages));
        offset[k] = ring_words;
        ring_words += std::max<std::uint32_t>(1, cells[k].max_in_flight);
    }
    const std::uint32_t slots = (max_buffer + 31) / 32 * 32;  // live entries never exceed the buffer
    const std::uint64_t warp_bytes = 8ull * (kMtWords + kRingSmem + 3ull * slots);
    if (warp_bytes > 200ull * 1024) return HBFSIM_UNSUPPORTED;  // buffer too large for a warp
    const std::uint32_t warps = static_cast<std::uint32_t>(
        std::max<std::uint64_t>(1, std::min<std::uint64_t>(4, (200ull * 1024) / warp_bytes)));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    hbfsim_prefetch_cell_v1* d_cells = nullptr;
    hbfsim_prefetch_stats_v1* d_out = nullptr;
    std::uint64_t *d_ring = nullptr, *d_offset = nullptr;
    int rc = HBFSIM_CUDA_ERROR;
    if (cudaMalloc(&d_cells, sizeof(hbfsim_prefetch_cell_v1) * cell_count) == cudaSuccess &&
        cudaMalloc(&d_out, sizeof(hbfsim_prefetch_stats_v1) * cell_count) == cudaSuccess &&
        cudaMalloc(&d_ring, 8 * ring_words) == cudaSuccess &&
        cudaMalloc(&d_offset, 8ull * cell_count) == cudaSuccess &&
        cudaMemcpyAsync(d_cells, cells, sizeof(hbfsim_prefetch_cell_v1) * cell_count,
                        cudaMemcpyHostToDevice, s) == cudaSuccess &&
        cudaMemcpyAsync(d_offset, offset.data(), 8ull * cell_count, cudaMemcpyHostToDevice,
                        s) == cudaSuccess) {
        SweepArgs a{};
        a.pages = pages;
        a.n = count;
        a.cells = d_cells;
        a.count = cell_count;
        a.slots = slots;
        a.warps = warps;
        a.ring = d_ring;
        a.ring_offset = d_offset;
        a.out = d_out;
        const std::uint32_t smem = static_cast<std::uint32_t>(warp_bytes * warps);
        if (cudaFuncSetAttribute(prefetch_sweep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)) == cudaSuccess) {
            prefetch_sweep_kernel<<<(cell_count + warps - 1) / warps, 32 * warps, smem, s>>>(a);
            if (cudaGetLastError() == cudaSuccess &&
                cudaMemcpyAsync(out, d_out, sizeof(hbfsim_prefetch_stats_v1) * cell_count,
                                cudaMemcpyDeviceToHost, s) == cudaSuccess &&
                cudaStreamSynchronize(s) == cudaSuccess)
                rc = HBFSIM_OK;
        }
    }
    cudaFree(d_cells);
    cudaFree(d_out);
    cudaFree(d_ring);
    cudaFree(d_offset);
    return rc;
}
