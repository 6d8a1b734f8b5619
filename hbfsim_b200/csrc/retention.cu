// retention.cu -- per-block retention-age ledger on the device.
//
// Reference: experiments/eq3_system_thermal/reliability.py (ReliabilityLedger)
// as run_maintenance_point.py:189, 225-234 drives it: every epoch, each block
// of a die ages by (end - start) * exp(Ea/kB * (1/Tref - 1/T)) at the midpoint
// of the die's temperature at the start and at the end of the epoch (the
// first epoch starts from the configured initial temperature)
// (arrhenius_acceleration, reliability.py:17-23; advance_temperature_many,
// 109-135).  Refresh is due on the 24 h wall cadence or, with the
// "equivalent_age_or_wall" trigger, once the equivalent age reaches 24 h
// (due_reasons, 76-88); a committed refresh resets the age and restarts the
// cadence at its completion (record_refresh_terminal, 172-187).  Program and
// erase counts follow _media_terminal (138-159).
//
// B200 layout: structure of arrays over the context's local blocks, block id
// ((local channel * D + die) * planes + plane) * blocks_per_plane + block.  The
// epoch is one map over blocks after one Arrhenius rate per die (the
// reference's same-temperature cohort); the due query is a stable compaction
// (per-CTA counts, one-CTA scan, ordered write); program counts decode a
// batch of accesses and add per block.  All blocks share one accounted
// frontier (the reference keeps one per block; its drivers advance every
// block over the same epochs).
#include "context.h"
#include "decode.cuh"

#include <cmath>
#include <vector>

namespace hbfb {

struct RetentionState {
    hbfsim_retention_config_v1 cfg{};
    std::uint64_t blocks = 0;
    std::uint32_t blocks_per_plane = 0;
    std::uint32_t pages_per_block = 0;
    std::uint32_t local_dies = 0;
    std::uint64_t frontier_ns = 0;       // accounted through (every block)
    double* d_age = nullptr;             // equivalent age, ns
    std::uint64_t* d_next_due = nullptr; // next wall-cadence due tick
    std::uint64_t* d_last_commit = nullptr;  // last committed refresh (kNever: none)
    std::uint32_t* d_counts = nullptr;   // [4][blocks]: program started / completed,
                                         // erase started / completed
    double* d_prev_temp = nullptr;       // per local die: the last epoch's temperature
    double* d_prev_next = nullptr;       // per local die: this epoch's (swapped after it)
    std::uint32_t* d_error = nullptr;
    std::uint32_t* d_cta_counts = nullptr;
    std::uint32_t cta_capacity = 0;
    std::uint64_t* d_count = nullptr;
};

namespace {

constexpr double kKbEvPerK = 8.62e-5;           // reliability.py:12
constexpr std::uint64_t kNever = ~std::uint64_t{0};
constexpr std::uint32_t kThreads = 256;
constexpr std::uint32_t kItems = 8;
constexpr std::uint32_t kTile = kThreads * kItems;

enum RetentionError : std::uint32_t {
    kErrTemperature = 1u,  // a temperature that is not finite and positive
    kErrBlock = 2u,        // a block id outside the ledger
};

struct RGuard {
    explicit RGuard(hbfsim_context* c) : lock(c->mu) { cudaSetDevice(c->device); }
    std::lock_guard<std::mutex> lock;
};

template <class T>
bool ralloc(T** p, std::uint64_t n)
{
    return cudaMalloc(reinterpret_cast<void**>(p), sizeof(T) * (n ? n : 1)) == cudaSuccess;
}

template <class T>
void rfree(T*& p)
{
    if (p) cudaFree(p);
    p = nullptr;
}

__global__ void init_kernel(double* age, std::uint64_t* next_due, std::uint64_t* last_commit,
                            std::uint32_t* counts, std::uint64_t n, double initial_age,
                            std::uint64_t due, double* prev_temp, std::uint32_t dies,
                            double initial_temp)
{
    const std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < dies) prev_temp[i] = initial_temp;
    if (i >= n) return;
    age[i] = initial_age;
    next_due[i] = due;
    last_commit[i] = kNever;
    for (int k = 0; k < 4; ++k) counts[k * n + i] = 0;
}

// One epoch of the ledger in one launch.  Each CTA ages kTile consecutive
// blocks; first it computes the Arrhenius rate of every local die (the
// cohort of its blocks) that its blocks belong to -- at the midpoint of the
// previous and current temperature, or at the current one -- into shared
// memory.  The CTA holding a die's first block also records that die's
// temperature for the next epoch, in a second buffer that the host swaps
// in after the launch, so no CTA reads a temperature another has replaced.
struct AgeArgs {
    const double* temp;         // per local die, or per global die (global_index)
    const double* prev;         // per local die, the last epoch's
    double* prev_next;          // per local die, written for the next epoch
    double* age;
    std::uint64_t n;            // blocks
    std::uint64_t blocks_per_die;
    double interval;            // end - start of the epoch, ns
    std::uint32_t D;
    std::uint32_t shard_rank, shard_count;
    std::uint32_t global_index;  // temp is indexed by global die (thermal model)
    std::uint32_t midpoint;      // use (prev + current) / 2
    double ea_over_kb;
    double inv_tref;
    std::uint32_t* error;
};

__device__ __forceinline__ double die_rate(const AgeArgs& a, std::uint32_t i, bool owner)
{
    std::uint32_t src = i;
    if (a.global_index) {
        const std::uint32_t c = i / a.D, d = i - c * a.D;
        src = (c * a.shard_count + a.shard_rank) * a.D + d;
    }
    const double cur = a.temp[src];
    const double t = a.midpoint ? __dadd_rn(a.prev[i], cur) / 2 : cur;
    if (owner) a.prev_next[i] = cur;
    if (!(t > 0.0) || !isfinite(t)) {
        atomicOr(a.error, kErrTemperature);
        return 0.0;
    }
    // reliability.py:17-23, same operation order
    return exp(__dmul_rn(a.ea_over_kb, __dsub_rn(a.inv_tref, __ddiv_rn(1.0, t))));
}

__global__ void __launch_bounds__(kThreads) age_kernel(const AgeArgs a)
{
    __shared__ double s_rate[kTile];
    const std::uint64_t b0 = static_cast<std::uint64_t>(blockIdx.x) * kTile;
    const std::uint64_t last = (b0 + kTile < a.n ? b0 + kTile : a.n) - 1;
    const std::uint64_t d_lo = b0 / a.blocks_per_die, d_hi = last / a.blocks_per_die;
    // a CTA's kTile blocks span at most kTile dies
    for (std::uint64_t k = threadIdx.x; k <= d_hi - d_lo; k += kThreads) {
        const std::uint64_t d = d_lo + k;
        s_rate[k] = die_rate(a, static_cast<std::uint32_t>(d), d * a.blocks_per_die >= b0);
    }
    __syncthreads();
#pragma unroll
    for (std::uint32_t j = 0; j < kItems; ++j) {
        const std::uint64_t i = b0 + j * kThreads + threadIdx.x;
        if (i >= a.n) break;
        // reliability.py:125-131: delta = (end - start) * rate; age +=
        // delta, rounded as two operations (no fused multiply-add)
        a.age[i] = __dadd_rn(a.age[i],
                             __dmul_rn(a.interval, s_rate[i / a.blocks_per_die - d_lo]));
    }
}

__device__ __forceinline__ std::uint32_t due_bits(const double* age,
                                                  const std::uint64_t* next_due,
                                                  std::uint64_t i, std::uint64_t at,
                                                  std::uint32_t age_trigger, double period)
{
    std::uint32_t r = at >= next_due[i] ? 1u : 0u;                // WALL_24H_SCENARIO_CADENCE
    if (age_trigger && age[i] >= period) r |= 2u;                // EQUIVALENT_AGE_24H_...
    return r;
}

struct DueArgs {
    const double* age;
    const std::uint64_t* next_due;
    std::uint64_t n;
    std::uint64_t at;
    std::uint32_t age_trigger;
    double period;
    std::uint32_t* cta_counts;
    std::uint32_t ctas;
    std::uint32_t* blocks;
    std::uint8_t* reasons;
    std::uint64_t capacity;
    std::uint64_t* count;
};

__device__ __forceinline__ std::uint32_t block_sum_exclusive(std::uint32_t v, std::uint32_t* s,
                                                             std::uint32_t& total)
{
    const std::uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    std::uint32_t inc = v;
#pragma unroll
    for (std::uint32_t d = 1; d < 32; d <<= 1) {
        const std::uint32_t o = __shfl_up_sync(0xffffffffu, inc, d);
        if (lane >= d) inc += o;
    }
    if (lane == 31) s[warp] = inc;
    __syncthreads();
    if (threadIdx.x == 0) {
        std::uint32_t run = 0;
        for (std::uint32_t w = 0; w < blockDim.x / 32; ++w) {
            const std::uint32_t t = s[w];
            s[w] = run;
            run += t;
        }
        s[blockDim.x / 32] = run;
    }
    __syncthreads();
    const std::uint32_t res = s[warp] + inc - v;
    total = s[blockDim.x / 32];
    __syncthreads();
    return res;
}

// tile of kTile blocks per CTA, thread t owns blocks t*kItems .. +kItems-1
__global__ void __launch_bounds__(kThreads) due_count_kernel(const DueArgs a)
{
    __shared__ std::uint32_t s[kThreads / 32 + 1];
    const std::uint64_t base = static_cast<std::uint64_t>(blockIdx.x) * kTile +
                               static_cast<std::uint64_t>(threadIdx.x) * kItems;
    std::uint32_t mine = 0;
    for (std::uint32_t j = 0; j < kItems; ++j) {
        const std::uint64_t i = base + j;
        if (i < a.n && due_bits(a.age, a.next_due, i, a.at, a.age_trigger, a.period)) ++mine;
    }
    std::uint32_t total;
    block_sum_exclusive(mine, s, total);
    if (threadIdx.x == 0) a.cta_counts[blockIdx.x] = total;
}

__global__ void __launch_bounds__(1024) due_scan_kernel(const DueArgs a)
{
    __shared__ std::uint32_t s[1024 / 32 + 1];
    std::uint32_t carry = 0;
    for (std::uint32_t b0 = 0; b0 < a.ctas; b0 += blockDim.x) {
        const std::uint32_t b = b0 + threadIdx.x;
        const std::uint32_t v = b < a.ctas ? a.cta_counts[b] : 0u;
        std::uint32_t total;
        const std::uint32_t ex = block_sum_exclusive(v, s, total);
        if (b < a.ctas) a.cta_counts[b] = carry + ex;
        carry += total;
    }
    if (threadIdx.x == 0) *a.count = carry;
}

__global__ void __launch_bounds__(kThreads) due_write_kernel(const DueArgs a)
{
    __shared__ std::uint32_t s[kThreads / 32 + 1];
    const std::uint64_t base = static_cast<std::uint64_t>(blockIdx.x) * kTile +
                               static_cast<std::uint64_t>(threadIdx.x) * kItems;
    std::uint32_t bits[kItems];
    std::uint32_t mine = 0;
    for (std::uint32_t j = 0; j < kItems; ++j) {
        const std::uint64_t i = base + j;
        bits[j] = i < a.n ? due_bits(a.age, a.next_due, i, a.at, a.age_trigger, a.period) : 0u;
        mine += bits[j] ? 1u : 0u;
    }
    std::uint32_t total;
    std::uint64_t at = a.cta_counts[blockIdx.x] + block_sum_exclusive(mine, s, total);
    for (std::uint32_t j = 0; j < kItems; ++j) {
        if (!bits[j]) continue;
        if (at < a.capacity) {
            a.blocks[at] = static_cast<std::uint32_t>(base + j);
            a.reasons[at] = static_cast<std::uint8_t>(bits[j]);
        }
        ++at;
    }
}

// reliability.py:172-187 with committed = true at the accounted frontier
__global__ void refresh_kernel(const std::uint32_t* blocks, std::uint64_t count, double* age,
                               std::uint64_t* next_due, std::uint64_t* last_commit,
                               std::uint64_t n, std::uint64_t completion, std::uint64_t period,
                               std::uint32_t* error)
{
    const std::uint64_t k = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (k >= count) return;
    const std::uint64_t b = blocks[k];
    if (b >= n) {
        atomicOr(error, kErrBlock);
        return;
    }
    age[b] = 0.0;
    last_commit[b] = completion;
    next_due[b] = completion + period;
}

// reliability.py:138-159 for a list of completed erases (succeeded, started)
__global__ void erase_kernel(const std::uint32_t* blocks, std::uint64_t count,
                             std::uint32_t* counts, std::uint64_t n, std::uint32_t* error)
{
    const std::uint64_t k = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (k >= count) return;
    const std::uint64_t b = blocks[k];
    if (b >= n) {
        atomicOr(error, kErrBlock);
        return;
    }
    atomicAdd(&counts[2 * n + b], 1u);
    atomicAdd(&counts[3 * n + b], 1u);
}

// Every modeled write of a batch programs one page of its block
// (record_program with succeeded = phase_started = true).
struct ProgramArgs {
    DecodeParams dp;
    const std::uint64_t* address;
    const std::uint32_t* bytes;
    const std::uint8_t* op;
    std::uint64_t count;
    std::uint32_t* counts;
    std::uint64_t n;
    std::uint32_t planes, blocks_per_plane, pages_per_block;
    std::uint32_t* error;
};

__global__ void program_kernel(const ProgramArgs a)
{
    const std::uint64_t i = static_cast<std::uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= a.count || a.op[i] != 1) return;
    const Decoded d = classify_decode(a.dp, a.address[i], a.bytes[i], 1u, true);
    if (d.status != kModeled) return;
    const std::uint64_t blk = d.page / a.pages_per_block;
    if (blk >= a.blocks_per_plane) {
        atomicOr(a.error, kErrBlock);
        return;
    }
    const std::uint64_t b =
        ((static_cast<std::uint64_t>(d.local) * a.dp.dies + d.die) * a.planes + d.plane) *
            a.blocks_per_plane + blk;
    if (b >= a.n) {
        atomicOr(a.error, kErrBlock);
        return;
    }
    atomicAdd(&a.counts[b], 1u);
    atomicAdd(&a.counts[a.n + b], 1u);
}

int take_error(RetentionState* r)
{
    std::uint32_t e = 0;
    if (cudaMemcpy(&e, r->d_error, 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemset(r->d_error, 0, 4) != cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    return e ? HBFSIM_INVALID_ARGUMENT : HBFSIM_OK;
}

}  // namespace

void retention_destroy(RetentionState* r)
{
    if (!r) return;
    rfree(r->d_age);
    rfree(r->d_next_due);
    rfree(r->d_last_commit);
    rfree(r->d_counts);
    rfree(r->d_prev_temp);
    rfree(r->d_prev_next);
    rfree(r->d_error);
    rfree(r->d_cta_counts);
    rfree(r->d_count);
    delete r;
}

}  // namespace hbfb

using namespace hbfb;

extern "C" {

int hbfsim_retention_configure_v1(hbfsim_context* c, const hbfsim_retention_config_v1* cfg)
{
    if (!c || !cfg || cfg->struct_size != sizeof(hbfsim_retention_config_v1) ||
        cfg->version != HBFSIM_RETENTION_CONFIG_V1_VERSION)
        return HBFSIM_INVALID_ARGUMENT;
    // reliability.py:36-55: the scenario contract's allowed values
    if ((cfg->ea_ev != 1.01 && cfg->ea_ev != 1.04 && cfg->ea_ev != 1.08) ||
        !(cfg->initial_temperature_k > 0.0) || !std::isfinite(cfg->initial_temperature_k) ||
        cfg->tref_k != 358.15 || cfg->period_ns != 86'400'000'000'000ull ||
        cfg->refresh_trigger > 1 || cfg->initial_wall_age_ns > cfg->period_ns ||
        cfg->epoch_ns > ~std::uint64_t{0} - cfg->period_ns)
        return HBFSIM_INVALID_ARGUMENT;
    RGuard g(c);
    if (c->mode != HBFSIM_MODEL_DIE_V1) return HBFSIM_UNSUPPORTED;  // blocks need the die geometry
    const Profile& p = c->profile;
    const std::uint64_t per_plane_unit = static_cast<std::uint64_t>(c->channels_total) *
                                         p.dies_per_channel * p.planes_per_die * p.page_bytes;
    const std::uint64_t pages = (p.capacity_bytes + per_plane_unit - 1) / per_plane_unit;
    const std::uint64_t bpp = std::max<std::uint64_t>(1, (pages + p.pages_per_block - 1) /
                                                             p.pages_per_block);
    const std::uint64_t blocks = static_cast<std::uint64_t>(c->C) * c->D * p.planes_per_die * bpp;
    if (bpp > 0xffffffffull || blocks > 0xffffffffull) return HBFSIM_UNSUPPORTED;
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    retention_destroy(c->retention);
    c->retention = nullptr;
    auto* r = new (std::nothrow) RetentionState();
    if (!r) return HBFSIM_CUDA_ERROR;
    r->cfg = *cfg;
    r->blocks = blocks;
    r->blocks_per_plane = static_cast<std::uint32_t>(bpp);
    r->pages_per_block = p.pages_per_block;
    r->local_dies = c->C * c->D;
    r->frontier_ns = cfg->epoch_ns;
    const std::uint32_t ctas = static_cast<std::uint32_t>((blocks + kTile - 1) / kTile);
    if (!ralloc(&r->d_age, blocks) || !ralloc(&r->d_next_due, blocks) ||
        !ralloc(&r->d_last_commit, blocks) || !ralloc(&r->d_counts, 4 * blocks) ||
        !ralloc(&r->d_prev_temp, r->local_dies) || !ralloc(&r->d_prev_next, r->local_dies) ||
        !ralloc(&r->d_error, 1) || !ralloc(&r->d_cta_counts, ctas) || !ralloc(&r->d_count, 1)) {
        retention_destroy(r);
        return HBFSIM_CUDA_ERROR;
    }
    r->cta_capacity = ctas;
    cudaMemset(r->d_error, 0, 4);
    // reliability.py:63-70: age = initial equivalent age, wall due at
    // epoch + period - initial wall age
    const std::uint64_t due = cfg->epoch_ns + cfg->period_ns - cfg->initial_wall_age_ns;
    const std::uint64_t span = std::max<std::uint64_t>(blocks, r->local_dies);
    init_kernel<<<static_cast<unsigned>((span + 255) / 256), 256>>>(
        r->d_age, r->d_next_due, r->d_last_commit, r->d_counts, blocks,
        static_cast<double>(cfg->initial_age_ns), due, r->d_prev_temp, r->local_dies,
        cfg->initial_temperature_k);
    if (cudaDeviceSynchronize() != cudaSuccess) {
        retention_destroy(r);
        return HBFSIM_CUDA_ERROR;
    }
    c->retention = r;
    return HBFSIM_OK;
}

uint64_t hbfsim_retention_blocks_v1(hbfsim_context* c)
{
    return c && c->retention ? c->retention->blocks : 0;
}

int hbfsim_retention_advance_v1(hbfsim_context* c, uint64_t end_ns, const double* die_temp_k,
                                void* stream)
{
    if (!c) return HBFSIM_INVALID_ARGUMENT;
    RGuard g(c);
    RetentionState* r = c->retention;
    if (!r || end_ns < r->frontier_ns) return HBFSIM_INVALID_ARGUMENT;
    const double* temps = die_temp_k;
    bool thermal = false;
    if (!temps) {  // the thermal model's die means, midpoint of the epoch
        if (!c->thermal) return HBFSIM_INVALID_ARGUMENT;
        temps = thermal_die_temperatures(c->thermal);
        thermal = true;
    }
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    AgeArgs a{};
    a.temp = temps;
    a.prev = r->d_prev_temp;
    a.prev_next = r->d_prev_next;
    a.age = r->d_age;
    a.n = r->blocks;
    a.blocks_per_die = static_cast<std::uint64_t>(c->profile.planes_per_die) *
                       r->blocks_per_plane;
    a.interval = static_cast<double>(end_ns - r->frontier_ns);
    a.D = c->D;
    a.shard_rank = c->shard_rank;
    a.shard_count = c->shard_count;
    a.global_index = thermal ? 1u : 0u;
    a.midpoint = thermal ? 1u : 0u;
    a.ea_over_kb = r->cfg.ea_ev / kKbEvPerK;
    a.inv_tref = 1.0 / r->cfg.tref_k;
    a.error = r->d_error;
    age_kernel<<<static_cast<unsigned>((r->blocks + kTile - 1) / kTile), kThreads, 0, s>>>(a);
    if (cudaGetLastError() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    std::swap(r->d_prev_temp, r->d_prev_next);
    r->frontier_ns = end_ns;
    return HBFSIM_OK;
}

int hbfsim_retention_due_v1(hbfsim_context* c, uint64_t at_ns, uint32_t* blocks,
                            uint8_t* reasons, uint64_t capacity, uint64_t* count, void* stream)
{
    if (!c || !count || (capacity && (!blocks || !reasons))) return HBFSIM_INVALID_ARGUMENT;
    RGuard g(c);
    RetentionState* r = c->retention;
    if (!r || at_ns < r->frontier_ns) return HBFSIM_INVALID_ARGUMENT;  // reliability.py:79-80
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    DueArgs a{};
    a.age = r->d_age;
    a.next_due = r->d_next_due;
    a.n = r->blocks;
    a.at = at_ns;
    a.age_trigger = r->cfg.refresh_trigger;
    a.period = static_cast<double>(r->cfg.period_ns);
    a.ctas = r->cta_capacity;
    a.cta_counts = r->d_cta_counts;
    a.blocks = blocks;
    a.reasons = reasons;
    a.capacity = capacity;
    a.count = r->d_count;
    due_count_kernel<<<a.ctas, kThreads, 0, s>>>(a);
    due_scan_kernel<<<1, 1024, 0, s>>>(a);
    due_write_kernel<<<a.ctas, kThreads, 0, s>>>(a);
    if (cudaMemcpyAsync(count, r->d_count, 8, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    return take_error(r);
}

int hbfsim_retention_refresh_v1(hbfsim_context* c, const uint32_t* blocks, uint64_t count,
                                void* stream)
{
    if (!c || (count && !blocks)) return HBFSIM_INVALID_ARGUMENT;
    RGuard g(c);
    RetentionState* r = c->retention;
    if (!r) return HBFSIM_INVALID_ARGUMENT;
    if (count == 0) return HBFSIM_OK;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    refresh_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, s>>>(
        blocks, count, r->d_age, r->d_next_due, r->d_last_commit, r->blocks, r->frontier_ns,
        r->cfg.period_ns, r->d_error);
    return cudaGetLastError() == cudaSuccess ? HBFSIM_OK : HBFSIM_CUDA_ERROR;
}

int hbfsim_retention_record_erase_v1(hbfsim_context* c, const uint32_t* blocks, uint64_t count,
                                     void* stream)
{
    if (!c || (count && !blocks)) return HBFSIM_INVALID_ARGUMENT;
    RGuard g(c);
    RetentionState* r = c->retention;
    if (!r) return HBFSIM_INVALID_ARGUMENT;
    if (count == 0) return HBFSIM_OK;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    erase_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, s>>>(
        blocks, count, r->d_counts, r->blocks, r->d_error);
    return cudaGetLastError() == cudaSuccess ? HBFSIM_OK : HBFSIM_CUDA_ERROR;
}

int hbfsim_retention_record_programs_v1(hbfsim_context* c, const uint64_t* address,
                                        const uint32_t* bytes, const uint8_t* operation,
                                        uint64_t count, void* stream)
{
    if (!c || (count && (!address || !bytes || !operation))) return HBFSIM_INVALID_ARGUMENT;
    RGuard g(c);
    RetentionState* r = c->retention;
    if (!r) return HBFSIM_INVALID_ARGUMENT;
    if (count == 0) return HBFSIM_OK;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    ProgramArgs a{};
    a.dp = media_decode_params(c, c->d_ranges, static_cast<std::uint32_t>(c->ranges.size()));
    a.address = address;
    a.bytes = bytes;
    a.op = operation;
    a.count = count;
    a.counts = r->d_counts;
    a.n = r->blocks;
    a.planes = c->profile.planes_per_die;
    a.blocks_per_plane = r->blocks_per_plane;
    a.pages_per_block = r->pages_per_block;
    a.error = r->d_error;
    program_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, s>>>(a);
    return cudaGetLastError() == cudaSuccess ? HBFSIM_OK : HBFSIM_CUDA_ERROR;
}

int hbfsim_get_retention_v1(hbfsim_context* c, double* age_ns, uint64_t* next_wall_due_ns,
                            uint64_t* last_refresh_commit_ns, uint32_t* counts, uint64_t blocks,
                            uint64_t* frontier_ns)
{
    if (!c) return HBFSIM_INVALID_ARGUMENT;
    RGuard g(c);
    RetentionState* r = c->retention;
    if (!r || blocks != r->blocks) return HBFSIM_INVALID_ARGUMENT;
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    if ((age_ns && cudaMemcpy(age_ns, r->d_age, 8 * blocks, cudaMemcpyDeviceToHost)) ||
        (next_wall_due_ns &&
         cudaMemcpy(next_wall_due_ns, r->d_next_due, 8 * blocks, cudaMemcpyDeviceToHost)) ||
        (last_refresh_commit_ns && cudaMemcpy(last_refresh_commit_ns, r->d_last_commit,
                                              8 * blocks, cudaMemcpyDeviceToHost)) ||
        (counts && cudaMemcpy(counts, r->d_counts, 16 * blocks, cudaMemcpyDeviceToHost)))
        return HBFSIM_CUDA_ERROR;
    if (frontier_ns) *frontier_ns = r->frontier_ns;
    return take_error(r);
}

}  // extern "C"
