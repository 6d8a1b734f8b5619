// context.cu -- the C ABI of the B200 access-timing library.
//
// Existing HBFSim exports (include/hbfsim/api.h) keep their signatures and
// error codes; the batch, time, factor and checkpoint exports are additive
// (include/hbfsim/batch_v1.h).  Every entry point converts failures into an
// hbfsim_error code; nothing throws across the ABI.
#include "context.h"

#include <algorithm>
#include <numeric>
#include <cerrno>
#include <cstring>
#include <limits>
#include <new>
#include <sys/stat.h>

using namespace hbfb;

namespace {

constexpr std::uint32_t kRangeCapacity = 32768;  // hbf_device.cuh:21
constexpr std::uint64_t kU64Max = std::numeric_limits<std::uint64_t>::max();

std::uint64_t sat_add(std::uint64_t a, std::uint64_t b)
{
    return b > kU64Max - a ? kU64Max : a + b;
}

std::uint64_t sat_mul(std::uint64_t a, std::uint64_t b)
{
    if (a == 0 || b == 0) return 0;
    return a > kU64Max / b ? kU64Max : a * b;
}

// hbf_device.cuh:746-757
std::uint64_t fast_transfer_ns(std::uint32_t bytes, std::uint64_t bw)
{
    if (bytes == 0 || bw == 0) return 0;
    const std::uint64_t num = static_cast<std::uint64_t>(bytes) * 1000000000ull;
    return (num + bw - 1) / bw;
}

std::uint64_t ceil_div128(unsigned __int128 n, std::uint64_t d)
{
    const unsigned __int128 q = (n + d - 1) / d;
    return q > kU64Max ? kU64Max : static_cast<std::uint64_t>(q);
}

bool valid_ring_capacity(std::uint32_t c)
{
    return c >= 2 && c <= 4096 && (c & (c - 1)) == 0;
}

bool make_dirs(const std::string& path)
{
    std::string cur;
    for (std::size_t i = 0; i <= path.size(); ++i) {
        if (i == path.size() || path[i] == '/') {
            if (!cur.empty() && ::mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST)
                return false;
        }
        if (i < path.size()) cur.push_back(path[i]);
    }
    struct stat st {};
    return ::stat(path.c_str(), &st) == 0 && S_ISDIR(st.st_mode);
}

template <typename T>
cudaError_t dalloc(T** p, std::uint64_t count)
{
    *p = nullptr;
    if (count == 0) count = 1;
    return cudaMalloc(reinterpret_cast<void**>(p), sizeof(T) * count);
}

template <typename T>
void dfree(T*& p)
{
    if (p) cudaFree(p);
    p = nullptr;
}

bool is_fast(const hbfsim_context* c) { return c->mode == HBFSIM_MODEL_FAST; }

std::uint32_t log2u(std::uint64_t v)
{
    std::uint32_t s = 0;
    while ((std::uint64_t{1} << s) < v) ++s;
    return s;
}

struct Guard {
    explicit Guard(hbfsim_context* c) : lock(c->mu) { cudaSetDevice(c->device); }
    std::lock_guard<std::mutex> lock;
};

int upload_ranges(hbfsim_context* c)
{
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    const std::uint32_t need = static_cast<std::uint32_t>(c->ranges.size());
    if (need > c->d_range_capacity || c->d_ranges == nullptr) {
        dfree(c->d_ranges);
        std::uint32_t cap = std::max<std::uint32_t>(16, c->d_range_capacity);
        while (cap < need) cap *= 2;
        if (dalloc(&c->d_ranges, cap) != cudaSuccess) {
            c->d_range_capacity = 0;
            return HBFSIM_CUDA_ERROR;
        }
        c->d_range_capacity = cap;
    }
    if (need &&
        cudaMemcpy(c->d_ranges, c->ranges.data(), sizeof(DevRange) * need,
                   cudaMemcpyHostToDevice) != cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

// With a thermal grid configured, the epoch controller writes the factors
// on the device; bring them back into the host copies.
int pull_thermal_factors(hbfsim_context* c)
{
    std::uint32_t *r, *t;
    std::uint64_t* a;
    thermal_factor_arrays(c->thermal, &r, &t, &a);
    if (cudaMemcpy(c->refresh_permille.data(), r, 4ull * c->C, cudaMemcpyDeviceToHost) ||
        cudaMemcpy(c->throttle_permille.data(), t, 4ull * c->stacks, cudaMemcpyDeviceToHost) ||
        cudaMemcpy(c->admit_after.data(), a, 8ull * c->stacks, cudaMemcpyDeviceToHost))
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

// Recompute the per-channel device tables from the factor inputs.
int update_tables(hbfsim_context* c)
{
    const Profile& p = c->profile;
    const std::uint64_t bw = channel_bandwidth(p);
    std::vector<std::uint64_t> h_bw(c->C);
    std::vector<i64> h_tr(c->C), h_tp(c->C), h_ad(c->C);
    c->x_max = 0;
    c->t_max = 0;
    c->admit_max = 0;
    for (std::uint32_t k = 0; k < c->C; ++k) {
        const std::uint32_t g = k * c->shard_count + c->shard_rank;
        const std::uint32_t stack = g < c->channels_total ? g % c->stacks : 0;
        const std::uint32_t r = c->refresh_permille[k];
        std::uint64_t eff = static_cast<std::uint64_t>(
            static_cast<unsigned __int128>(bw) * (1000u - r) / 1000u);
        if (eff == 0) eff = 1;
        const std::uint32_t thr = c->throttle_permille[stack];
        const std::uint64_t tr = sat_mul(
            ceil_div128(static_cast<unsigned __int128>(p.read_latency_ns) * thr, 1000),
            p.time_scale);
        const std::uint64_t tp = sat_mul(
            ceil_div128(static_cast<unsigned __int128>(p.program_latency_ns) * thr, 1000),
            p.time_scale);
        h_bw[k] = eff;
        h_tr[k] = static_cast<i64>(tr);
        h_tp[k] = static_cast<i64>(tp);
        h_ad[k] = static_cast<i64>(c->admit_after[stack]);
        const std::uint64_t x = sat_mul(
            ceil_div128(static_cast<unsigned __int128>(p.page_bytes) * 1000000000ull, eff),
            p.time_scale);
        c->x_max = std::max(c->x_max, x);
        c->t_max = std::max({c->t_max, tr, tp});
        c->admit_max = std::max(c->admit_max, c->admit_after[stack]);
    }
    if (is_fast(c)) {
        c->x_max = sat_mul(fast_transfer_ns(p.page_bytes, p.aggregate_bandwidth_bytes_per_s),
                           p.time_scale);
        c->t_max = sat_mul(std::max(p.read_latency_ns, p.program_latency_ns), p.time_scale);
        c->admit_max = 0;
    }
    if (c->thermal) {  // the epoch controller may raise the factors later
        std::uint64_t xb, ob, ab;
        thermal_tick_bounds(c->thermal, &xb, &ob, &ab);
        c->x_max = std::max(c->x_max, xb);
        c->t_max = std::max(c->t_max, ob);
        c->admit_max = std::max(c->admit_max, ab);
    }
    // one shared bandwidth whose 1e9 / bw reduces to 1 / 2^s: the kernels
    // take the shift from their arguments instead of the channel table
    c->x_uniform_shift = 0xffu;
    if (c->C > 0 && std::all_of(h_bw.begin(), h_bw.end(),
                                [&](std::uint64_t v) { return v == h_bw[0]; })) {
        const std::uint64_t g = std::gcd<std::uint64_t, std::uint64_t>(1000000000ull, h_bw[0]);
        const std::uint64_t num = 1000000000ull / g, den = h_bw[0] / g;
        if (num == 1 && (den & (den - 1)) == 0) {
            std::uint32_t sh = 0;
            while ((1ull << sh) < den) ++sh;
            if (sh < 32) c->x_uniform_shift = sh;
        }
    }
    const std::size_t bytes = sizeof(std::uint64_t) * c->C;
    if (cudaMemcpyAsync(c->d_chan_bw, h_bw.data(), bytes, cudaMemcpyHostToDevice, c->stream) ||
        cudaMemcpyAsync(c->d_t_read, h_tr.data(), bytes, cudaMemcpyHostToDevice, c->stream) ||
        cudaMemcpyAsync(c->d_t_prog, h_tp.data(), bytes, cudaMemcpyHostToDevice, c->stream) ||
        cudaMemcpyAsync(c->d_admit, h_ad.data(), bytes, cudaMemcpyHostToDevice, c->stream) ||
        cudaStreamSynchronize(c->stream))
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

void free_geometry(hbfsim_context* c)
{
    dfree(c->d_state[0]);
    dfree(c->d_state[1]);
    dfree(c->d_chan_bw);
    dfree(c->d_t_read);
    dfree(c->d_t_prog);
    dfree(c->d_admit);
    dfree(c->d_die_read_bytes);
    dfree(c->d_die_writes);
    dfree(c->d_act_stage);
    dfree(c->d_agg);
    dfree(c->d_incoming);
    dfree(c->d_scan_groups);
    c->scratch_ctas = 0;
}

// (Re)build everything that depends on stacks / striping / sharding; resets
// the timing state to zero.
int configure_geometry(hbfsim_context* c, std::uint32_t stacks,
                       std::uint32_t stripe, std::uint32_t rank,
                       std::uint32_t shards)
{
    const Profile& p = c->profile;
    if (stacks == 0 || shards == 0 || rank >= shards) return HBFSIM_INVALID_ARGUMENT;
    if (stripe == 0) stripe = p.page_bytes;
    if (stripe < 512 || (stripe & (stripe - 1)) != 0) return HBFSIM_INVALID_ARGUMENT;
    const unsigned __int128 total = static_cast<unsigned __int128>(stacks) * p.channels;
    if (total > 65535) return HBFSIM_UNSUPPORTED;
    if (is_fast(c) && shards != 1) return HBFSIM_UNSUPPORTED;  // one global tail
    if (!is_fast(c) && p.dies_per_channel > 15) return HBFSIM_UNSUPPORTED;
    // stripe units of the whole media space must fit 32 bits
    if (p.capacity_bytes / stripe >= 0xffffffffull) return HBFSIM_UNSUPPORTED;
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    free_geometry(c);
    retention_destroy(c->retention);  // its blocks follow the geometry
    c->retention = nullptr;
    c->stacks = stacks;
    c->stripe_bytes = stripe;
    c->shard_rank = rank;
    c->shard_count = shards;
    c->channels_total = static_cast<std::uint32_t>(total);
    c->D = is_fast(c) ? 0 : p.dies_per_channel;
    c->K = is_fast(c) ? 1 : c->D + 1;
    c->C = is_fast(c) ? 1 : (c->channels_total + shards - 1) / shards;
    const std::string& s = p.plane_allocation_scheme;
    for (int k = 0; k < 4; ++k)
        c->order[k] = s[k] == 'C' ? 0 : s[k] == 'W' ? 1 : s[k] == 'D' ? 2 : 3;
    // FAST with an empirical profile: one more word, the packed burst state
    const std::uint64_t words = static_cast<std::uint64_t>(c->C) * c->K + (c->empirical ? 1 : 0);
    if (dalloc(&c->d_state[0], words) || dalloc(&c->d_state[1], words) ||
        dalloc(&c->d_chan_bw, c->C) || dalloc(&c->d_t_read, c->C) ||
        dalloc(&c->d_t_prog, c->C) || dalloc(&c->d_admit, c->C) ||
        dalloc(&c->d_die_read_bytes, std::uint64_t{c->C} * std::max(1u, c->D)) ||
        dalloc(&c->d_die_writes, std::uint64_t{c->C} * std::max(1u, c->D)) ||
        dalloc(&c->d_act_stage, 2ull * c->C * std::max(1u, c->D)))
        return HBFSIM_CUDA_ERROR;
    cudaMemset(c->d_state[0], 0, sizeof(std::uint64_t) * words);
    cudaMemset(c->d_state[1], 0, sizeof(std::uint64_t) * words);
    cudaMemset(c->d_die_read_bytes, 0, 8ull * c->C * std::max(1u, c->D));
    cudaMemset(c->d_die_writes, 0, 8ull * c->C * std::max(1u, c->D));
    c->state_words_allocated = words;
    c->cur = 0;
    c->refresh_permille.assign(c->C, 0);
    c->throttle_permille.assign(c->stacks, 1000);
    c->admit_after.assign(c->stacks, 0);
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    return update_tables(c);
}

DecodeParams decode_params(const hbfsim_context* c)
{
    const Profile& p = c->profile;
    DecodeParams d{};
    d.ranges = c->d_ranges;
    d.range_count = static_cast<std::uint32_t>(c->ranges.size());
    if (c->ranges.size() == 1) {
        const DevRange& r = c->ranges[0];
        d.one = SingleRange{r.base, r.length, r.file_offset, (u64{1} << r.reserved) - 1,
                            r.timing, 1u};
    }
    d.stripe_shift = log2u(c->stripe_bytes);
    d.stacks = c->stacks;
    d.dies = p.dies_per_channel;
    d.planes = p.planes_per_die;
    d.page_bytes = p.page_bytes;
    d.shard_rank = c->shard_rank;
    d.shard_count = c->shard_count;
    d.channels_total = c->channels_total;
    d.local_channels = c->C;
    for (int k = 0; k < 4; ++k) d.order[k] = c->order[k];
    d.radix[0] = make_fastdiv(c->channels_total);
    d.radix[1] = make_fastdiv(1);
    d.radix[2] = make_fastdiv(p.dies_per_channel);
    d.radix[3] = make_fastdiv(p.planes_per_die);
    d.shard_div = make_fastdiv(c->shard_count);
    d.stack_div = make_fastdiv(c->stacks);
    const std::uint32_t radix[4] = {c->channels_total, 1, p.dies_per_channel,
                                    p.planes_per_die};
    std::uint64_t stride = 1, chan_stride = 1, die_stride = 1;
    for (int k = 0; k < 4; ++k) {
        if (c->order[k] == 0) chan_stride = stride;
        if (c->order[k] == 2) die_stride = stride;
        stride *= radix[c->order[k]];
    }
    // strides beyond 32 bits mean the digit is always 0 for 32-bit units
    d.chan_stride = make_fastdiv(chan_stride > 0xffffffffull ? 0xffffffffu
                                                             : static_cast<std::uint32_t>(chan_stride));
    d.die_stride = make_fastdiv(die_stride > 0xffffffffull ? 0xffffffffu
                                                           : static_cast<std::uint32_t>(die_stride));
    auto is_pow2 = [](std::uint64_t v) { return v != 0 && (v & (v - 1)) == 0; };
    d.pow2 = is_pow2(chan_stride) && chan_stride <= 0x80000000ull && is_pow2(die_stride) &&
             die_stride <= 0x80000000ull && is_pow2(c->channels_total) &&
             is_pow2(p.dies_per_channel) && is_pow2(c->shard_count);
    if (d.pow2) {
        d.chan_shift = log2u(chan_stride);
        d.chan_mask = c->channels_total - 1;
        d.die_shift = log2u(die_stride);
        d.die_mask = p.dies_per_channel - 1;
        d.shard_shift = log2u(c->shard_count);
        d.shard_mask = c->shard_count - 1;
    }
    return d;
}

TimingParams timing_params(const hbfsim_context* c)
{
    const Profile& p = c->profile;
    TimingParams t{};
    t.model = is_fast(c) ? kModelFast : kModelDie;
    t.dies = c->D;
    t.state_k = c->K;
    t.time_scale = p.time_scale;
    const std::uint64_t x = fast_transfer_ns(p.page_bytes, p.aggregate_bandwidth_bytes_per_s);
    t.fast_x = static_cast<i64>(sat_mul(x, p.time_scale));
    t.fast_l_read = static_cast<i64>(sat_mul(p.read_latency_ns, p.time_scale));
    t.fast_l_prog = static_cast<i64>(sat_mul(p.program_latency_ns, p.time_scale));
    t.fast_service_read = std::max(x, p.read_latency_ns);   // hbf_device.cuh:797-817
    t.fast_service_prog = std::max(x, p.program_latency_ns);
    t.chan_bw = c->d_chan_bw;
    // the thermal controller rewrites the bandwidth table on the device
    t.x_shift = c->thermal ? 0xffu : c->x_uniform_shift;
    // x_max and t_max already cover the thermal controller's factors
    t.step_max = c->x_max + c->t_max < (1ull << 40)
                     ? static_cast<i64>(c->x_max + c->t_max) : 0;
    t.admit_zero = c->admit_max == 0 ? 1u : 0u;
    t.chan_t_read = c->d_t_read;
    t.chan_t_prog = c->d_t_prog;
    t.chan_admit = c->d_admit;
    // per-die activity feeds the thermal epoch controller only
    const bool track = c->mode == HBFSIM_MODEL_DIE_V1 && (c->thermal || c->track_activity);
    t.die_read_bytes = track ? c->d_die_read_bytes : nullptr;
    t.die_writes = track ? c->d_die_writes : nullptr;
    t.act_stage = track ? c->d_act_stage : nullptr;
    return t;
}

cudaEvent_t take_event(hbfsim_context* c)
{
    if (!c->event_pool.empty()) {
        cudaEvent_t e = c->event_pool.back();
        c->event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void mark_launch(void* owner, int slot, int phase, cudaStream_t stream)
{
    auto* c = static_cast<hbfsim_context*>(owner);
    if (phase == 0) {
        c->marks.push_back({slot, take_event(c), take_event(c)});
        cudaEventRecord(c->marks.back().begin, stream);
    } else if (!c->marks.empty()) {
        cudaEventRecord(c->marks.back().end, stream);
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

// Empirical burst-curve profile: the control-header check and the service
// of every run length (hbf_device.cuh:978-1128), on the profile's curve.
// An invalid header makes every timed access Unsupported, as the reference's
// resolve_fast_or_hybrid does (hbf_device.cu:773-777, 797-801).
int setup_empirical(hbfsim_context* c)
{
    const Profile& p = c->profile;
    std::uint32_t pages[6];
    std::uint64_t cum[6];
    for (int i = 0; i < 6; ++i) {
        pages[i] = p.empirical[i].pages;
        cum[i] = p.empirical[i].cumulative_ns;
    }
    std::vector<std::uint64_t> table(kRunCap + 1, 0);
    empirical_service_table(pages, cum, 6, table.data());
    const bool valid = empirical_control_valid(1, 6, p.program_latency_ns, pages, cum);
    c->emp.ok = valid && p.time_scale != 0 && c->request_timeout_ns != 0 ? 1u : 0u;
    c->emp.program_ns = p.program_latency_ns;
    c->emp.time_scale = p.time_scale;
    std::uint64_t largest = p.program_latency_ns;
    for (std::uint32_t r = 1; r <= kRunCap; ++r) largest = std::max(largest, table[r]);
    c->emp_scaled_max = c->emp.ok ? sat_mul(largest, p.time_scale) : 0;
    if (dalloc(&c->d_emp_service, kRunCap + 1) || dalloc(&c->d_emp_words, kEmpScratchWords) ||
        cudaMemcpy(c->d_emp_service, table.data(), 8 * table.size(), cudaMemcpyHostToDevice) !=
            cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    c->emp.service = c->d_emp_service;
    return HBFSIM_OK;
}

// One batch of the empirical FAST model (device arrays).  Bound proof: the
// batch adds at most n times the largest scaled service; below 2^59 (with
// arrivals and the carried tail checked below 2^59 on the device) no tick
// reaches 2^60 and the parallel kernels are exact.
int run_empirical_batch(hbfsim_context* c, const BatchIO& io, cudaStream_t stream,
                        std::uint32_t* error, const LaunchHooks& hooks)
{
    const bool sequential =
        sat_mul(c->emp_scaled_max, io.n) >= static_cast<std::uint64_t>(kArrivalLimit);
    EmpiricalScratch s{};
    s.words = c->d_emp_words;
    s.error = error;
    s.last_arrival = c->d_last_arrival;
    s.counters = c->d_counters;
    s.state_in = c->d_state[c->cur];
    s.state_out = c->d_state[1 - c->cur];
    const cudaError_t err = launch_empirical(decode_params(c), c->emp, io, s, sequential,
                                             c->sm_count, stream, hooks);
    if (err != cudaSuccess) return HBFSIM_CUDA_ERROR;
    c->cur = 1 - c->cur;
    return HBFSIM_OK;
}

int model_supported(const hbfsim_context* c)
{
    if (c->mode != HBFSIM_MODEL_FAST && c->mode != HBFSIM_MODEL_DIE_V1)
        return HBFSIM_UNSUPPORTED;  // REFERENCE/HYBRID need MQSim
    return HBFSIM_OK;
}

// Times n accesses already on the device.  Caller holds the lock.  With
// `ranges` set, the accesses are decoded against that table instead of the
// registered ranges (media addresses of Capacity-mode actions), and their
// arrivals need not be ordered.
int run_device_batch(hbfsim_context* c, const BatchIO& io, cudaStream_t stream,
                     const DevRange* ranges = nullptr, std::uint32_t range_count = 0)
{
    if (io.n == 0) return HBFSIM_OK;
    if (c->empirical) {
        if (ranges) return HBFSIM_UNSUPPORTED;  // media actions: die model only
        return run_empirical_batch(c, io, stream, c->d_error, c->hooks());
    }
    // Bound proof for the parallel path.  Pass 1 checks on the device that
    // every arrival and every carried state word is below 2^59; here the host
    // checks that the admission ticks are too and that the batch can add less
    // than 2^59 (n times the largest transfer plus die time).  Then no tick
    // reaches 2^60 and signed max-plus arithmetic equals the saturating one.
    const std::uint64_t per = sat_add(c->x_max, c->t_max);
    const std::uint64_t growth = sat_mul(per, io.n);
    const bool sequential = growth >= static_cast<std::uint64_t>(kArrivalLimit) ||
                            c->admit_max >= static_cast<std::uint64_t>(kArrivalLimit) ||
                            c->x_max > 0xffffffull || c->t_max >= (1ull << 40);
    BatchPlan plan{};
    if (plan_batch(io.n, c->C, c->K, c->D, c->sm_count, &plan) != 0) return HBFSIM_UNSUPPORTED;
    if (plan.ctas > c->scratch_ctas) {
        dfree(c->d_agg);
        dfree(c->d_incoming);
        dfree(c->d_scan_groups);
        const std::uint64_t ctas = std::max<std::uint64_t>(plan.ctas, 2ull * c->sm_count);
        const std::uint64_t ranges = 2 * ctas;  // a CTA may time its tile's halves
        if (dalloc(&c->d_agg, ranges * c->C * c->K * (c->K + 1)) ||
            dalloc(&c->d_incoming, ranges * c->C * c->K) ||
            dalloc(&c->d_scan_groups, lb_group_words(ranges, c->C, c->K))) {
            c->scratch_ctas = 0;
            return HBFSIM_CUDA_ERROR;
        }
        c->scratch_ctas = ctas;
    }
    BatchScratch s{};
    s.agg = c->d_agg;
    s.incoming = c->d_incoming;
    s.scan_groups = c->d_scan_groups;
    s.scan_lb = c->d_scan_lb;
    s.ranges_capacity = 2 * c->scratch_ctas;
    s.error = c->d_error;
    s.last_arrival = c->d_last_arrival;
    s.counters = c->d_counters;
    s.state_in = c->d_state[c->cur];
    s.state_out = c->d_state[1 - c->cur];
    DecodeParams dp = decode_params(c);
    TimingParams tp = timing_params(c);
    if (ranges) {
        dp.ranges = ranges;
        dp.range_count = range_count;
        dp.one.valid = 0;
        tp.any_order = 1;
    }
    const cudaError_t err = launch_batch(dp, tp, io, plan, s, sequential, stream, c->hooks());
    if (err != cudaSuccess) return HBFSIM_CUDA_ERROR;
    c->cur = 1 - c->cur;
    return HBFSIM_OK;
}

}  // namespace

namespace hbfb {
int run_media_batch(hbfsim_context* c, const BatchIO& io, const DevRange* ranges,
                    std::uint32_t range_count, cudaStream_t stream)
{
    return run_device_batch(c, io, stream, ranges, range_count);
}

DecodeParams media_decode_params(const hbfsim_context* c, const DevRange* ranges,
                                 std::uint32_t range_count)
{
    DecodeParams dp = decode_params(c);
    dp.ranges = ranges;
    dp.range_count = range_count;
    dp.one.valid = 0;
    return dp;
}

TimingParams context_timing_params(const hbfsim_context* c) { return timing_params(c); }
}  // namespace hbfb

hbfb::LaunchHooks hbfsim_context::hooks()
{
    hbfb::LaunchHooks h;
    if (profiling) {
        h.owner = this;
        h.mark = mark_launch;
    }
    return h;
}

extern "C" {

uint32_t hbfsim_abi_version(void) { return 1u; }

int hbfsim_context_create(const hbfsim_options* options, hbfsim_context** out)
{
    if (out) *out = nullptr;
    // context.cpp:424-433 valid_options, plus this build's die model
    if (!out || !options || !options->profile_path || !options->profile_path[0] ||
        !options->report_dir || !options->report_dir[0] ||
        (options->mode > HBFSIM_MODEL_HYBRID && options->mode != HBFSIM_MODEL_DIE_V1) ||
        !valid_ring_capacity(options->ring_capacity) || options->request_timeout_ns == 0)
        return HBFSIM_INVALID_ARGUMENT;
    Profile profile;
    if (!load_profile(options->profile_path, &profile).empty()) return HBFSIM_INVALID_ARGUMENT;
    if (!make_dirs(options->report_dir)) return HBFSIM_IO_ERROR;
    auto* c = new (std::nothrow) hbfsim_context();
    if (!c) return HBFSIM_IO_ERROR;
    c->profile = profile;
    c->report_dir = options->report_dir;
    c->mode = options->mode;
    c->request_timeout_ns = options->request_timeout_ns;
    if (cudaGetDevice(&c->device) != cudaSuccess ||
        cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, c->device) !=
            cudaSuccess ||
        cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        dalloc(&c->d_error, 1) || dalloc(&c->d_last_arrival, 1) || dalloc(&c->d_counters, 1) ||
        dalloc(&c->d_sample_seq, 1) ||
        dalloc(&c->d_sample_counts, hbfsim_context::kSampleCtas) ||
        dalloc(&c->d_scan_lb, 2 + kLbFlagWords)) {
        hbfsim_context_destroy(c);
        return HBFSIM_CUDA_ERROR;
    }
    cudaMemset(c->d_scan_lb, 0, 4 * (2 + kLbFlagWords));
    cudaMemset(c->d_error, 0, sizeof(std::uint32_t));
    cudaMemset(c->d_last_arrival, 0, sizeof(std::uint64_t));
    cudaMemset(c->d_counters, 0, sizeof(DevCounters));
    cudaMemset(c->d_sample_seq, 0, sizeof(std::uint64_t));
    c->empirical = is_fast(c) && profile.has_empirical;
    int rc = configure_geometry(c, 1, 0, 0, 1);
    if (rc == HBFSIM_OK && c->empirical) rc = setup_empirical(c);
    if (rc != HBFSIM_OK) {
        hbfsim_context_destroy(c);
        return rc;
    }
    *out = c;
    return HBFSIM_OK;
}

int hbfsim_register_device(hbfsim_context* c, void* device_ptr, size_t length,
                           const hbfsim_range_options* o)
{
    if (!c || !device_ptr || length == 0 || !o) return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    // range_table.cpp:17-120
    const std::uint64_t base = reinterpret_cast<std::uintptr_t>(device_ptr);
    if (length > kU64Max - base || o->permissions == 0 ||
        (o->permissions & ~static_cast<std::uint32_t>(HBFSIM_RANGE_READ_WRITE)) != 0 ||
        o->cache_policy != HBFSIM_CACHE_POLICY_NONE)
        return HBFSIM_INVALID_ARGUMENT;
    if (o->mode != HBFSIM_RANGE_MODE_TIMING && o->mode != HBFSIM_RANGE_MODE_CAPACITY)
        return HBFSIM_INVALID_ARGUMENT;
    if (c->ranges.size() >= kRangeCapacity) return HBFSIM_UNSUPPORTED;
    const std::uint64_t page = c->profile.page_bytes;
    if (length > kU64Max - (page - 1)) return HBFSIM_UNSUPPORTED;
    const std::uint64_t extent = (length + page - 1) / page * page;
    if (c->next_file_offset > c->profile.capacity_bytes ||
        extent > c->profile.capacity_bytes - c->next_file_offset)
        return HBFSIM_UNSUPPORTED;
    const auto at = std::lower_bound(
        c->ranges.begin(), c->ranges.end(), base,
        [](const DevRange& r, std::uint64_t b) { return r.base < b; });
    const std::size_t index = static_cast<std::size_t>(at - c->ranges.begin());
    if ((index != 0 && c->ranges[index - 1].base + c->ranges[index - 1].length > base) ||
        (index != c->ranges.size() && base + length > c->ranges[index].base))
        return HBFSIM_INVALID_ARGUMENT;
    DevRange r{};
    r.base = base;
    r.length = length;
    r.file_offset = c->next_file_offset;
    r.page_bytes = page;
    r.range_id = c->next_range_id;
    r.mode = o->mode;
    r.permissions = o->permissions;
    r.reserved = log2u(page);
    r.end = base + length;
    r.ok = (r.mode == 1 || r.mode == 2) && page != 0 && page <= 0xffffffffull ? 1u : 0u;
    r.timing = r.ok && r.mode == HBFSIM_RANGE_MODE_TIMING ? (r.permissions & 3u) : 0u;
    c->ranges.insert(at, r);
    const int rc = upload_ranges(c);
    if (rc != HBFSIM_OK) {
        c->ranges.erase(c->ranges.begin() + static_cast<long>(index));
        return rc;
    }
    ++c->next_range_id;
    c->next_file_offset += extent;
    return HBFSIM_OK;
}

int hbfsim_map_file(hbfsim_context* c, const char* path, uint64_t, size_t length,
                    const hbfsim_range_options* o, void** out)
{
    if (out) *out = nullptr;
    if (!c || !path || !path[0] || length == 0 || !o || !out) return HBFSIM_INVALID_ARGUMENT;
    return HBFSIM_UNSUPPORTED;  // file-backed capacity bytes: out of scope
}

int hbfsim_flush(hbfsim_context* c)
{
    if (!c) return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    DevCounters k{};
    if (cudaMemcpy(&k, c->d_counters, sizeof k, cudaMemcpyDeviceToHost) != cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    if (k.errors > c->errors_reported) {
        c->errors_reported = k.errors;
        if (k.error_code & kErrWait) {  // a bounded wait of the fused thermal step ran out
            thermal_reset_barrier(c->thermal);
            k.error_code &= ~static_cast<unsigned long long>(kErrWait);
            cudaMemcpy(&c->d_counters->error_code, &k.error_code, 8, cudaMemcpyHostToDevice);
            return HBFSIM_TIMEOUT;
        }
        return HBFSIM_INVALID_ARGUMENT;  // a batch was refused (unsorted arrivals)
    }
    return HBFSIM_OK;
}

int hbfsim_get_stats(hbfsim_context* c, hbfsim_stats* out)
{
    if (!c || !out) return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    DevCounters k{};
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(&k, c->d_counters, sizeof k, cudaMemcpyDeviceToHost) != cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    *out = {};
    if (is_fast(c)) {
        out->fast_requests = k.modeled;
        out->fast_modeled_ns = k.fast_modeled_ns;
    } else {
        out->requests_submitted = k.modeled;
        out->requests_completed = k.modeled;
        out->reference_requests = k.modeled;
        out->fast_modeled_ns = 0;
    }
    return HBFSIM_OK;
}

int hbfsim_get_capacity_stats_v1(hbfsim_context* c, hbfsim_capacity_stats_v1* out)
{
    if (!c || !out || out->struct_size != sizeof(hbfsim_capacity_stats_v1) ||
        out->version != HBFSIM_CAPACITY_STATS_V1_VERSION)
        return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    if (!c->capacity) return HBFSIM_INVALID_ARGUMENT;  // context.cpp:2019-2022: no service
    const std::uint32_t size = out->struct_size, version = out->version;
    std::memset(out, 0, sizeof *out);
    out->struct_size = size;
    out->version = version;
    capacity_stats(c->capacity, out);
    return HBFSIM_OK;
}

int hbfsim_unregister(hbfsim_context* c, void* range_base)
{
    if (!c || !range_base) return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    const std::uint64_t base = reinterpret_cast<std::uintptr_t>(range_base);
    const auto at = std::lower_bound(
        c->ranges.begin(), c->ranges.end(), base,
        [](const DevRange& r, std::uint64_t b) { return r.base < b; });
    if (at == c->ranges.end() || at->base != base) return HBFSIM_INVALID_ARGUMENT;
    const DevRange saved = *at;
    const auto index = at - c->ranges.begin();
    c->ranges.erase(at);
    const int rc = upload_ranges(c);
    if (rc != HBFSIM_OK) c->ranges.insert(c->ranges.begin() + index, saved);
    return rc;
}

void hbfsim_context_destroy(hbfsim_context* c)
{
    if (!c) return;
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    if (c->thermal) thermal_destroy(c->thermal);
    if (c->capacity) capacity_destroy(c->capacity);
    retention_destroy(c->retention);
    free_geometry(c);
    dfree(c->d_ranges);
    dfree(c->d_error);
    dfree(c->d_last_arrival);
    dfree(c->d_counters);
    dfree(c->d_sample_seq);
    dfree(c->d_sample_counts);
    dfree(c->d_scan_lb);
    dfree(c->d_emp_service);
    dfree(c->d_emp_words);
    for (auto& p : c->d_stage) {
        if (p) cudaFree(p);
        p = nullptr;
    }
    for (auto& m : c->marks) {
        cudaEventDestroy(m.begin);
        cudaEventDestroy(m.end);
    }
    for (auto e : c->event_pool) cudaEventDestroy(e);
    if (c->stream) cudaStreamDestroy(c->stream);
    if (c->copy_in) cudaStreamDestroy(c->copy_in);
    if (c->copy_out) cudaStreamDestroy(c->copy_out);
    delete c;
}

int hbfsim_set_geometry_v1(hbfsim_context* c, const hbfsim_geometry_v1* g)
{
    if (!c || !g || g->struct_size != sizeof(hbfsim_geometry_v1) ||
        g->version != HBFSIM_GEOMETRY_V1_VERSION)
        return HBFSIM_INVALID_ARGUMENT;
    Guard lock(c);
    if (c->thermal) return HBFSIM_UNSUPPORTED;  // set geometry before thermal
    return configure_geometry(c, g->stacks, g->stripe_bytes, g->shard_rank, g->shard_count);
}

int hbfsim_submit_access_batch_v1(hbfsim_context* c, const hbfsim_access_batch_v1* b,
                                  void* stream)
{
    if (!c || !b || b->struct_size != sizeof(hbfsim_access_batch_v1) ||
        b->version != HBFSIM_ACCESS_BATCH_V1_VERSION)
        return HBFSIM_INVALID_ARGUMENT;
    if (b->count && (!b->address || !b->bytes || !b->operation || !b->arrival_ns ||
                     !b->done_ns || !b->latency_ns || !b->status))
        return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    const int ok = model_supported(c);
    if (ok != HBFSIM_OK) return ok;
    BatchIO io{b->address, b->bytes, b->operation, b->arrival_ns, b->done_ns,
               b->latency_ns, b->status, b->count, false};
    io.aligned = aligned16(io.address) && aligned16(io.bytes) && aligned16(io.op) &&
                 aligned16(io.arrival) && aligned16(io.done) && aligned16(io.latency) &&
                 aligned16(io.status);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    return run_device_batch(c, io, s);
}

int hbfsim_submit_access_batch_host_v1(hbfsim_context* c, const hbfsim_access_batch_v1* b)
{
    if (!c || !b || b->struct_size != sizeof(hbfsim_access_batch_v1) ||
        b->version != HBFSIM_ACCESS_BATCH_V1_VERSION)
        return HBFSIM_INVALID_ARGUMENT;
    if (b->count && (!b->address || !b->bytes || !b->operation || !b->arrival_ns ||
                     !b->done_ns || !b->latency_ns || !b->status))
        return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    const int ok = model_supported(c);
    if (ok != HBFSIM_OK) return ok;
    if (b->count == 0) return HBFSIM_OK;
    constexpr std::uint64_t kStage = 1ull << 22;  // accesses per pipeline stage
    constexpr std::uint64_t kStageBytes = kStage * 48;
    if (!c->d_stage[0]) {
        if (cudaMalloc(&c->d_stage[0], kStageBytes) || cudaMalloc(&c->d_stage[1], kStageBytes) ||
            cudaStreamCreateWithFlags(&c->copy_in, cudaStreamNonBlocking) ||
            cudaStreamCreateWithFlags(&c->copy_out, cudaStreamNonBlocking))
            return HBFSIM_CUDA_ERROR;
        c->stage_capacity = kStage;
    }
    cudaEvent_t in_done[2], run_done[2], out_done[2];
    for (int k = 0; k < 2; ++k) {
        cudaEventCreateWithFlags(&in_done[k], cudaEventDisableTiming);
        cudaEventCreateWithFlags(&run_done[k], cudaEventDisableTiming);
        cudaEventCreateWithFlags(&out_done[k], cudaEventDisableTiming);
        cudaEventRecord(out_done[k], c->copy_out);
    }
    int rc = HBFSIM_OK;
    const std::uint64_t n = b->count;
    std::uint64_t chunk_index = 0;
    for (std::uint64_t at = 0; at < n && rc == HBFSIM_OK; at += kStage, ++chunk_index) {
        const int s = static_cast<int>(chunk_index & 1);
        const std::uint64_t m = std::min(kStage, n - at);
        auto* base = static_cast<unsigned char*>(c->d_stage[s]);
        auto* d_addr = reinterpret_cast<std::uint64_t*>(base);
        auto* d_arr = reinterpret_cast<std::uint64_t*>(base + 8 * kStage);
        auto* d_done = reinterpret_cast<std::uint64_t*>(base + 16 * kStage);
        auto* d_lat = reinterpret_cast<std::uint64_t*>(base + 24 * kStage);
        auto* d_bytes = reinterpret_cast<std::uint32_t*>(base + 32 * kStage);
        auto* d_op = base + 36 * kStage;
        auto* d_st = base + 37 * kStage;
        cudaStreamWaitEvent(c->copy_in, out_done[s], 0);
        if (cudaMemcpyAsync(d_addr, b->address + at, 8 * m, cudaMemcpyHostToDevice, c->copy_in) ||
            cudaMemcpyAsync(d_arr, b->arrival_ns + at, 8 * m, cudaMemcpyHostToDevice, c->copy_in) ||
            cudaMemcpyAsync(d_bytes, b->bytes + at, 4 * m, cudaMemcpyHostToDevice, c->copy_in) ||
            cudaMemcpyAsync(d_op, b->operation + at, m, cudaMemcpyHostToDevice, c->copy_in)) {
            rc = HBFSIM_CUDA_ERROR;
            break;
        }
        cudaEventRecord(in_done[s], c->copy_in);
        cudaStreamWaitEvent(c->stream, in_done[s], 0);
        BatchIO io{d_addr, d_bytes, d_op, d_arr, d_done, d_lat, d_st, m, true};
        rc = run_device_batch(c, io, c->stream);
        cudaEventRecord(run_done[s], c->stream);
        cudaStreamWaitEvent(c->copy_out, run_done[s], 0);
        if (cudaMemcpyAsync(b->done_ns + at, d_done, 8 * m, cudaMemcpyDeviceToHost, c->copy_out) ||
            cudaMemcpyAsync(b->latency_ns + at, d_lat, 8 * m, cudaMemcpyDeviceToHost, c->copy_out) ||
            cudaMemcpyAsync(b->status + at, d_st, m, cudaMemcpyDeviceToHost, c->copy_out))
            rc = HBFSIM_CUDA_ERROR;
        cudaEventRecord(out_done[s], c->copy_out);
    }
    if (cudaStreamSynchronize(c->copy_out) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess)
        rc = HBFSIM_CUDA_ERROR;
    for (int k = 0; k < 2; ++k) {
        cudaEventDestroy(in_done[k]);
        cudaEventDestroy(run_done[k]);
        cudaEventDestroy(out_done[k]);
    }
    return rc;
}

int hbfsim_reset_state_v1(hbfsim_context* c, void* stream)
{
    if (!c) return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    if (cudaMemsetAsync(c->d_state[c->cur], 0, 8 * c->state_words_allocated, s) ||
        cudaMemsetAsync(c->d_last_arrival, 0, sizeof(std::uint64_t), s))
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

int hbfsim_set_profiling_v1(hbfsim_context* c, int enable)
{
    if (!c) return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    c->profiling = enable != 0;
    return HBFSIM_OK;
}

int hbfsim_get_kernel_times_v1(hbfsim_context* c, hbfsim_kernel_times_v1* out)
{
    if (!c || !out || out->struct_size != sizeof(hbfsim_kernel_times_v1) ||
        out->version != HBFSIM_KERNEL_TIMES_V1_VERSION)
        return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    for (int k = 0; k < HBFSIM_KERNEL_SLOTS_V1; ++k) {
        out->launches[k] = 0;
        out->total_ms[k] = 0.0;
    }
    for (auto& m : c->marks) {
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, m.begin, m.end) == cudaSuccess) {
            out->launches[m.slot] += 1;
            out->total_ms[m.slot] += ms;
        }
        c->event_pool.push_back(m.begin);
        c->event_pool.push_back(m.end);
    }
    c->marks.clear();
    return HBFSIM_OK;
}

int hbfsim_get_simulated_time_v1(hbfsim_context* c, uint64_t* ns)
{
    if (!c || !ns) return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    DevCounters k{};
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(&k, c->d_counters, sizeof k, cudaMemcpyDeviceToHost) != cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    *ns = k.max_done;
    return HBFSIM_OK;
}

int hbfsim_get_batch_stats_v1(hbfsim_context* c, hbfsim_batch_stats_v1* out)
{
    if (!c || !out || out->struct_size != sizeof(hbfsim_batch_stats_v1) ||
        out->version != HBFSIM_BATCH_STATS_V1_VERSION)
        return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    DevCounters k{};
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(&k, c->d_counters, sizeof k, cudaMemcpyDeviceToHost) != cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    out->modeled = k.modeled;
    out->bypass = k.bypass;
    out->unsupported = k.unsupported;
    out->foreign = k.foreign;
    out->latency_sum_ns = k.latency_sum;
    out->max_done_ns = k.max_done;
    out->fast_modeled_ns = k.fast_modeled_ns;
    out->batches = k.batches;
    out->device_errors = k.errors;
    return HBFSIM_OK;
}

int hbfsim_decode_batch_v1(hbfsim_context* c, const uint64_t* address, const uint32_t* bytes,
                           const uint8_t* operation, uint64_t count, hbfsim_decoded_v1* out,
                           void* stream)
{
    if (!c || (count && (!address || !bytes || !operation || !out)))
        return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    return launch_decode(decode_params(c), address, bytes, operation, count, out, s,
                         c->hooks()) ==
                   cudaSuccess
               ? HBFSIM_OK
               : HBFSIM_CUDA_ERROR;
}

int hbfsim_sample_batch_v1(hbfsim_context* c, const uint64_t* address, const uint32_t* bytes,
                           const uint8_t* operation, uint64_t count, uint8_t* sample,
                           void* stream)
{
    if (!c || (count && (!address || !bytes || !operation || !sample)))
        return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    const Profile& p = c->profile;
    // reference context.cpp:975-981: rate * (long double) UINT64_MAX
    const std::uint64_t threshold =
        p.reference_sample_rate >= 1.0
            ? ~std::uint64_t{0}
            : static_cast<std::uint64_t>(p.reference_sample_rate *
                                         static_cast<long double>(~std::uint64_t{0}));
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    return launch_sample(decode_params(c), address, bytes, operation, count, sample,
                         p.reference_warmup_requests, threshold, c->d_sample_seq,
                         c->d_sample_counts, hbfsim_context::kSampleCtas, s, c->hooks()) ==
                   cudaSuccess
               ? HBFSIM_OK
               : HBFSIM_CUDA_ERROR;
}

int hbfsim_set_channel_factors_v1(hbfsim_context* c, const uint32_t* refresh,
                                  const uint32_t* throttle, const uint64_t* admit)
{
    if (!c) return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    if (refresh)
        for (std::uint32_t k = 0; k < c->C; ++k)
            if (refresh[k] > 999) return HBFSIM_INVALID_ARGUMENT;
    if (throttle)
        for (std::uint32_t k = 0; k < c->stacks; ++k)
            if (throttle[k] == 0) return HBFSIM_INVALID_ARGUMENT;
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    if (c->thermal) {  // the controller's values are the ones in force
        const int rc = pull_thermal_factors(c);
        if (rc != HBFSIM_OK) return rc;
    }
    if (refresh) c->refresh_permille.assign(refresh, refresh + c->C);
    if (throttle) c->throttle_permille.assign(throttle, throttle + c->stacks);
    if (admit) c->admit_after.assign(admit, admit + c->stacks);
    const int rc = update_tables(c);
    if (rc != HBFSIM_OK || !c->thermal) return rc;
    // keep the controller's copy in step: the next epoch starts from these
    std::uint32_t *r, *t;
    std::uint64_t* a;
    thermal_factor_arrays(c->thermal, &r, &t, &a);
    if (cudaMemcpy(r, c->refresh_permille.data(), 4ull * c->C, cudaMemcpyHostToDevice) ||
        cudaMemcpy(t, c->throttle_permille.data(), 4ull * c->stacks, cudaMemcpyHostToDevice) ||
        cudaMemcpy(a, c->admit_after.data(), 8ull * c->stacks, cudaMemcpyHostToDevice))
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

int hbfsim_get_channel_factors_v1(hbfsim_context* c, uint32_t* refresh, uint32_t* throttle,
                                  uint64_t* admit)
{
    if (!c) return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    if (c->thermal) {
        if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
        const int rc = pull_thermal_factors(c);
        if (rc != HBFSIM_OK) return rc;
    }
    if (refresh) std::copy(c->refresh_permille.begin(), c->refresh_permille.end(), refresh);
    if (throttle) std::copy(c->throttle_permille.begin(), c->throttle_permille.end(), throttle);
    if (admit) std::copy(c->admit_after.begin(), c->admit_after.end(), admit);
    return HBFSIM_OK;
}

uint64_t hbfsim_state_words_v1(hbfsim_context* c)
{
    return c ? c->state_words_allocated : 0;
}

int hbfsim_get_state_v1(hbfsim_context* c, uint64_t* host_words, uint64_t words)
{
    if (!c || !host_words || words != c->state_words_allocated) return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(host_words, c->d_state[c->cur], 8 * words, cudaMemcpyDeviceToHost) !=
            cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

int hbfsim_set_state_v1(hbfsim_context* c, const uint64_t* host_words, uint64_t words)
{
    if (!c || !host_words || words != c->state_words_allocated) return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(c->d_state[c->cur], host_words, 8 * words, cudaMemcpyHostToDevice) !=
            cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

int hbfsim_get_die_activity_v1(hbfsim_context* c, uint64_t* read_bytes, uint64_t* writes,
                               uint64_t count)
{
    if (!c || count != static_cast<std::uint64_t>(c->C) * std::max(1u, c->D))
        return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    if (read_bytes &&
        cudaMemcpy(read_bytes, c->d_die_read_bytes, 8 * count, cudaMemcpyDeviceToHost))
        return HBFSIM_CUDA_ERROR;
    if (writes && cudaMemcpy(writes, c->d_die_writes, 8 * count, cudaMemcpyDeviceToHost))
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Batch entry point that allocates nothing.
//
// Some callers cannot call cudaMalloc while they run: an inference server that
// has reserved almost all device memory for its own pool up front (vLLM sizes
// its KV cache that way) would see the allocation fail, and in any process a
// first-time cudaMalloc can synchronize the device and stall every other
// stream.  hbfsim_submit_access_batch_static_v1 therefore takes its scratch --
// the per-CTA range aggregates, the carried states and the batch error word --
// from the fixed array below instead of from memory the context allocates.
//
// The array is 8 MiB.  Every GPU that loads this library holds it until the
// process exits.  All calls, from every context, share it, and it keeps the
// previous call's contents: the error word is cleared by each call and every
// other byte a call reads is written by that call first.  Calls whose work
// overlaps on the GPU (different streams, or different contexts on one
// device, without ordering between them) race on the array; serialize them.
// In host code the array's name is only a stand-in for the device variable:
// its device address is looked up with cudaGetSymbolAddress once per device,
// on that device's first call, so that first call should come before any
// stream capture begins.  Under CUDA's lazy module loading the array's
// device memory is committed only when this library's module loads on the
// device (its first kernel launch or symbol lookup there), so a caller that
// reserves almost all memory should make its first call before reserving.
// ---------------------------------------------------------------------------
namespace {

constexpr std::size_t kStaticScratchBytes = std::size_t{8} << 20;
constexpr std::size_t kStaticErrorBytes = 256;  // error word, padded
// then the look-back scan's counters and flags at a fixed address (zero as
// the array is, and left zero by every scan)
constexpr std::size_t kStaticLbBytes = (4 * (2 + kLbFlagWords) + 255) / 256 * 256;
constexpr std::size_t kStaticHeadBytes = kStaticErrorBytes + kStaticLbBytes;
constexpr int kMaxDevices = 64;

}  // namespace

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

namespace {

std::mutex g_static_mu;
void* g_static_address[kMaxDevices] = {};

// Device address of g_static_scratch on `device` (which must be current).
int static_scratch_address(int device, void** out)
{
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (device < 0 || device >= kMaxDevices) return HBFSIM_UNSUPPORTED;
    if (!g_static_address[device]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p)
            return HBFSIM_CUDA_ERROR;
        g_static_address[device] = p;
    }
    *out = g_static_address[device];
    return HBFSIM_OK;
}

}  // namespace

extern "C" int hbfsim_submit_access_batch_static_v1(hbfsim_context* c,
                                                    const hbfsim_access_batch_v1* b,
                                                    void* stream)
{
    if (!c || !b || b->struct_size != sizeof(hbfsim_access_batch_v1) ||
        b->version != HBFSIM_ACCESS_BATCH_V1_VERSION)
        return HBFSIM_INVALID_ARGUMENT;
    if (b->count && (!b->address || !b->bytes || !b->operation || !b->arrival_ns ||
                     !b->done_ns || !b->latency_ns || !b->status))
        return HBFSIM_INVALID_ARGUMENT;
    Guard g(c);
    const int ok = model_supported(c);
    if (ok != HBFSIM_OK) return ok;
    if (b->count == 0) return HBFSIM_OK;
    void* base = nullptr;
    const int rc = static_scratch_address(c->device, &base);
    if (rc != HBFSIM_OK) return rc;
    BatchIO io{b->address, b->bytes, b->operation, b->arrival_ns, b->done_ns,
               b->latency_ns, b->status, b->count, false};
    io.aligned = aligned16(io.address) && aligned16(io.bytes) && aligned16(io.op) &&
                 aligned16(io.arrival) && aligned16(io.done) && aligned16(io.latency) &&
                 aligned16(io.status);
    if (c->empirical) {  // scratch allocated with the context
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
        return run_empirical_batch(c, io, st, reinterpret_cast<std::uint32_t*>(base),
                                   LaunchHooks{});
    }
    // the same bound proof as the allocating entry point
    const std::uint64_t growth = sat_mul(sat_add(c->x_max, c->t_max), io.n);
    const bool sequential = growth >= static_cast<std::uint64_t>(kArrivalLimit) ||
                            c->admit_max >= static_cast<std::uint64_t>(kArrivalLimit) ||
                            c->x_max > 0xffffffull || c->t_max >= (1ull << 40);
    BatchPlan plan{};
    if (plan_batch(io.n, c->C, c->K, c->D, c->sm_count, &plan) != 0) return HBFSIM_UNSUPPORTED;
    // Fit the CTA grid to the array: each CTA needs its range aggregate and
    // its incoming state.  Fewer CTAs cover longer ranges; results do not
    // depend on how the batch is split.  A shape whose single CTA does not
    // fit is refused.
    // (plus, per group of 32 CTAs, the look-back scan's group words)
    const std::uint64_t words_per_cta =
        static_cast<std::uint64_t>(c->C) * c->K * (c->K + 1) + static_cast<std::uint64_t>(c->C) * c->K;
    const std::uint64_t group_words = lb_group_words(1, c->C, c->K);
    const std::uint64_t avail = (kStaticScratchBytes - kStaticHeadBytes) / 8;
    const std::uint64_t max_ctas =
        avail > group_words ? (avail - group_words) / (words_per_cta + group_words / 32 + 1) : 0;
    if (max_ctas == 0) return HBFSIM_UNSUPPORTED;
    if (plan.ctas > max_ctas) {
        const std::uint64_t tiles = (io.n + plan.T - 1) / plan.T;
        const std::uint64_t per = (tiles + max_ctas - 1) / max_ctas;
        plan.tiles_per_cta = static_cast<std::uint32_t>(per);
        plan.ctas = static_cast<std::uint32_t>((tiles + per - 1) / per);
    }
    auto* bytes = static_cast<unsigned char*>(base);
    BatchScratch s{};
    s.error = reinterpret_cast<std::uint32_t*>(bytes);
    s.agg = reinterpret_cast<i64*>(bytes + kStaticHeadBytes);
    s.incoming = s.agg + static_cast<std::uint64_t>(plan.ctas) * c->C * c->K * (c->K + 1);
    s.scan_groups = s.incoming + static_cast<std::uint64_t>(plan.ctas) * c->C * c->K;
    s.scan_lb = reinterpret_cast<std::uint32_t*>(bytes + kStaticErrorBytes);
    s.ranges_capacity = plan.ctas;  // one range per CTA here
    s.last_arrival = c->d_last_arrival;
    s.counters = c->d_counters;
    s.state_in = c->d_state[c->cur];
    s.state_out = c->d_state[1 - c->cur];
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    if (launch_batch(decode_params(c), timing_params(c), io, plan, s, sequential, st,
                     LaunchHooks{}) != cudaSuccess)
        return HBFSIM_CUDA_ERROR;
    c->cur = 1 - c->cur;
    return HBFSIM_OK;
}
