// context.h -- the hbfsim_context object behind the C ABI (internal).
#pragma once

#include "../../include/hbfsim/batch_v1.h"
#include "empirical.h"
#include "profile.h"
#include "timing.h"

#include <mutex>
#include <string>
#include <vector>

namespace hbfb {
struct ThermalState;    // thermal.cu
struct CapacityState;   // capacity.cu
struct RetentionState;  // retention.cu
}

struct hbfsim_context {
    hbfb::Profile profile;
    std::string report_dir;
    std::uint32_t mode = 0;            // hbfsim_options.mode
    std::uint64_t request_timeout_ns = 0;
    int device = 0;
    int sm_count = 148;
    cudaStream_t stream = nullptr;
    std::mutex mu;

    // ranges (host copy sorted by base; device copy mirrors it)
    std::vector<hbfb::DevRange> ranges;
    std::uint64_t next_file_offset = 0;
    std::uint32_t next_range_id = 1;
    hbfb::DevRange* d_ranges = nullptr;
    std::uint32_t d_range_capacity = 0;

    // geometry
    std::uint32_t stacks = 1;
    std::uint32_t stripe_bytes = 0;
    std::uint32_t shard_rank = 0;
    std::uint32_t shard_count = 1;
    std::uint32_t channels_total = 0;  // stacks * profile.channels
    std::uint32_t C = 0;               // local channels (state rows)
    std::uint32_t D = 0;               // dies per channel (die model)
    std::uint32_t K = 0;               // state words per channel
    std::uint8_t order[4] = {0, 1, 2, 3};

    // timing state, double-buffered: batches read cur, write 1-cur
    std::uint64_t* d_state[2] = {nullptr, nullptr};
    int cur = 0;
    std::uint64_t state_words_allocated = 0;

    // per-batch scratch
    hbfb::i64* d_agg = nullptr;
    hbfb::i64* d_incoming = nullptr;
    hbfb::i64* d_scan_groups = nullptr;     // look-back range scan: group maps and states
    std::uint32_t* d_scan_lb = nullptr;     // its counters and flags (zero between scans)
    std::uint64_t scratch_ctas = 0;
    std::uint32_t* d_error = nullptr;
    std::uint64_t* d_last_arrival = nullptr;
    hbfb::DevCounters* d_counters = nullptr;
    // hybrid sampler: running count of timed accesses, per-CTA scratch
    std::uint64_t* d_sample_seq = nullptr;
    std::uint64_t* d_sample_counts = nullptr;
    static constexpr std::uint32_t kSampleCtas = 1024;
    std::uint64_t errors_reported = 0;

    // channel factor tables (device, per local channel) + host inputs
    std::uint64_t* d_chan_bw = nullptr;
    hbfb::i64* d_t_read = nullptr;
    hbfb::i64* d_t_prog = nullptr;
    hbfb::i64* d_admit = nullptr;
    std::vector<std::uint32_t> refresh_permille;   // per local channel
    std::vector<std::uint32_t> throttle_permille;  // per stack
    std::vector<std::uint64_t> admit_after;        // per stack
    std::uint64_t x_max = 0;   // largest transfer tick of any access (scaled)
    // every channel's transfer is (bytes + 2^x_shift - 1) >> x_shift (one
    // bandwidth of 1e9 / 2^x_shift bytes per second); 0xff when not
    std::uint32_t x_uniform_shift = 0xffu;
    std::uint64_t t_max = 0;   // largest die op tick (scaled, throttled)
    std::uint64_t admit_max = 0;

    // per-die activity since the last epoch (die model), index c*D+d
    unsigned long long* d_die_read_bytes = nullptr;
    unsigned long long* d_die_writes = nullptr;
    unsigned long long* d_act_stage = nullptr;  // [C*D][2], one batch's pass-1 count

    // host-buffer pipeline
    cudaStream_t copy_in = nullptr;
    cudaStream_t copy_out = nullptr;
    void* d_stage[2] = {nullptr, nullptr};
    std::uint64_t stage_capacity = 0;  // accesses per stage

    // FAST model with an empirical burst-curve profile: read service per run
    // length (device table), per-batch scratch, bound of one scaled service.
    // The state then holds one more word: the packed burst state.
    bool empirical = false;
    hbfb::EmpiricalParams emp{};
    std::uint64_t* d_emp_service = nullptr;
    std::uint64_t* d_emp_words = nullptr;
    std::uint64_t emp_scaled_max = 0;

    hbfb::ThermalState* thermal = nullptr;
    hbfb::CapacityState* capacity = nullptr;  // Capacity-mode LRU (capacity.cu)
    hbfb::RetentionState* retention = nullptr;  // per-block retention ledger (retention.cu)
    bool track_activity = false;  // accumulate per-die activity without thermal

    // launch profiling (event pairs per kernel slot)
    bool profiling = false;
    struct Mark {
        int slot;
        cudaEvent_t begin;
        cudaEvent_t end;
    };
    std::vector<Mark> marks;
    std::vector<cudaEvent_t> event_pool;
    hbfb::LaunchHooks hooks();
};

namespace hbfb {
// thermal.cu
void thermal_destroy(ThermalState* t);
void capacity_destroy(CapacityState* c);
void retention_destroy(RetentionState* r);
// Device array of the grid's per-die mean temperatures (global die g*D+d).
const double* thermal_die_temperatures(const ThermalState* t);
void thermal_reset_barrier(ThermalState* t);
// Times media actions (device arrays) decoded against `ranges`, in batch
// order whatever their arrivals; carries the context's timing state.
int run_media_batch(hbfsim_context* c, const BatchIO& io, const DevRange* ranges,
                    std::uint32_t range_count, cudaStream_t stream);
DecodeParams media_decode_params(const hbfsim_context* c, const DevRange* ranges,
                                 std::uint32_t range_count);
TimingParams context_timing_params(const hbfsim_context* c);
void capacity_stats(const CapacityState* c, hbfsim_capacity_stats_v1* out);
// Device arrays of the factors the epoch controller derived (refresh per
// local channel, throttle permille and admit-after tick per stack).
void thermal_factor_arrays(ThermalState* t, std::uint32_t** refresh, std::uint32_t** throttle,
                           std::uint64_t** admit);
// Largest transfer tick, die-op tick and admit tick the controller can put
// into the channel tables (bounds for the parallel path's tick proof).
void thermal_tick_bounds(const ThermalState* t, std::uint64_t* x, std::uint64_t* op,
                         std::uint64_t* admit);
}
