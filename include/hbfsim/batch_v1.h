/*
 * hbfsim/batch_v1.h -- additive, versioned exports for batched access timing
 * on B200.  None of these exist in the reference C API; each struct carries
 * struct_size and version the way hbfsim_capacity_stats_v1 does
 * (reference include/hbfsim/api.h:66-90), so later versions can grow them.
 *
 * Every entry point returns an hbfsim_error code and never throws.  Device
 * pointers are plain CUDA device addresses; `stream` is a cudaStream_t passed
 * as void* (NULL = the context's own stream).  Calls on one context are
 * serialized by the context; contexts are independent.
 *
 * Reference interfaces replaced, per entry point:
 *   hbfsim_submit_access_batch_v1   the per-access device helper
 *       __hbfsim_resolve (src/cuda_runtime/device/hbf_device.cu:963-1344)
 *       and its fast-model step resolve_fast_or_hybrid (hbf_device.cu:765-960),
 *       run over a whole batch instead of one instrumented load at a time
 *   hbfsim_decode_batch_v1          find_range_index / media_descriptor
 *       (hbf_device.cuh:826-944) plus the stripe decode of
 *       src/ucie/bank_layout.cpp:59-72 and src/ucie/stack_router.cpp:52-59
 *   hbfsim_get_simulated_time_v1    the modeled clock the reference reads
 *       from fast_channel_tail_ns (hbf_device.cuh:70) / MQSim's engine.now
 *   hbfsim_advance_epoch_v1         ThermalModel::advance_to
 *       (src/eq3_thermal/thermal.cpp:242-311) on the eq3 layered grid
 *       (tools/eq3_layered_export.py:48-114) plus the control sample of
 *       CpuService (src/eq3_thermal/cpu_service.cpp:221-283)
 *   hbfsim_submit_capacity_batch_v1 CapacityPageService::resolve
 *       (src/host_service/capacity_page_service.cpp:97-210) with exact LRU
 *       (adapters/vllm_capacity/placement_policy.py:68-93) and the
 *       program-then-read media actions (request_dispatcher.cpp:107-126,
 *       294-298)
 */
#ifndef HBFSIM_BATCH_V1_H
#define HBFSIM_BATCH_V1_H

#include "api.h"

#ifdef __cplusplus
extern "C" {
#endif

/* hbfsim_options.mode value selecting the per-die max-plus model. */
#define HBFSIM_MODEL_DIE_V1 3u

/* Per-access status written by the batch path. */
enum hbfsim_access_status_v1 {
    HBFSIM_ACCESS_MODELED = 1,      /* timed (reference RequestStatus::Ready) */
    HBFSIM_ACCESS_UNSUPPORTED = 6,  /* rejected (RequestStatus::Unsupported)  */
    HBFSIM_ACCESS_BYPASS = 8,       /* outside every range: native, untimed   */
    HBFSIM_ACCESS_FOREIGN = 9       /* another shard's channel                */
};

/* ---- geometry: stacks, striping and channel sharding ---- */
#define HBFSIM_GEOMETRY_V1_VERSION 1u
typedef struct hbfsim_geometry_v1 {
    uint32_t struct_size;
    uint32_t version;
    uint32_t stacks;         /* UCIe stack_count; profile channels are per stack */
    uint32_t stripe_bytes;   /* power of two, >= 512; 0 = page_bytes           */
    uint32_t shard_rank;     /* this context owns channels g % shard_count == rank */
    uint32_t shard_count;    /* 1 = no sharding                                 */
    uint32_t reserved[2];
} hbfsim_geometry_v1;

/* Must be called before the first batch (defaults: 1 stack, page striping,
 * 1 shard). */
int hbfsim_set_geometry_v1(hbfsim_context* context,
                           const hbfsim_geometry_v1* geometry);

/* ---- access batches ---- */
#define HBFSIM_ACCESS_BATCH_V1_VERSION 1u
typedef struct hbfsim_access_batch_v1 {
    uint32_t struct_size;
    uint32_t version;
    uint64_t count;
    const uint64_t* address;     /* device address of the access            */
    const uint32_t* bytes;       /* access size                             */
    const uint8_t* operation;    /* 0 read, 1 write                         */
    const uint64_t* arrival_ns;  /* simulated arrival tick, non-decreasing  */
    uint64_t* done_ns;           /* out: completion tick                    */
    uint64_t* latency_ns;        /* out: done - arrival                     */
    uint8_t* status;             /* out: hbfsim_access_status_v1            */
} hbfsim_access_batch_v1;

/* Times one batch with the context's model, continuing from the die/channel
 * state the previous batch left.  All pointers are device pointers.  Runs
 * asynchronously on `stream`; results are valid once the stream reaches the
 * end of the call.  Arrivals must be non-decreasing within a batch and must
 * not go below the previous batch's; a violation is recorded on the device,
 * leaves the context state unchanged, and is returned by the next
 * hbfsim_flush.  The outputs of such a refused batch are unspecified (the
 * latency buffer doubles as working space between the two timing passes). */
int hbfsim_submit_access_batch_v1(hbfsim_context* context,
                                  const hbfsim_access_batch_v1* batch,
                                  void* stream);

/* The same batch call without any device allocation.  No counterpart in
 * the reference.  For callers that must not call cudaMalloc while running
 * -- a server that pre-reserved nearly all device memory for its own pool,
 * or code that cannot afford the device-wide synchronization a first
 * cudaMalloc may cause.  Its scratch (per-CTA range aggregates, carried
 * states, the batch error word) lives in one 8 MiB device array that the
 * library defines statically; every GPU that loads the library holds those
 * 8 MiB until the process exits.  All calls share the array: calls whose
 * work overlaps on the GPU race and must be serialized by the caller.  The
 * first call on a device looks up the array's device address; make that
 * first call before any stream capture begins.  With CUDA's lazy module
 * loading (the default) the 8 MiB are committed when the library's device
 * code first loads on a device -- at that first call, or at any earlier
 * library call that launches a kernel there -- so a caller that is about to
 * reserve nearly all device memory should make one call first.  Returns
 * HBFSIM_UNSUPPORTED
 * when one CTA's scratch (local channels * (D+1) * (D+3) * 8 bytes, plus the
 * range scan's 64 KiB of flags and its per-group words) exceeds the array;
 * otherwise it times the batch exactly as hbfsim_submit_access_batch_v1
 * does. */
int hbfsim_submit_access_batch_static_v1(hbfsim_context* context,
                                         const hbfsim_access_batch_v1* batch,
                                         void* stream);

/* The same call with HOST pointers: copies in, times, copies out, pipelined
 * over chunks on the context's streams.  Synchronous. */
int hbfsim_submit_access_batch_host_v1(hbfsim_context* context,
                                       const hbfsim_access_batch_v1* batch);

/* Returns the timing state to idle -- every die and channel free at tick 0,
 * no arrival seen yet -- without touching ranges, factors or counters.
 * Asynchronous on `stream`; replaces the carried state the way
 * hbfsim_set_state_v1 does, without a host round trip. */
int hbfsim_reset_state_v1(hbfsim_context* context, void* stream);

/* Simulated time: the latest completion tick modeled so far. Synchronizes. */
int hbfsim_get_simulated_time_v1(hbfsim_context* context, uint64_t* ns);

#define HBFSIM_BATCH_STATS_V1_VERSION 1u
typedef struct hbfsim_batch_stats_v1 {
    uint32_t struct_size;
    uint32_t version;
    uint64_t modeled;
    uint64_t bypass;
    uint64_t unsupported;
    uint64_t foreign;
    uint64_t latency_sum_ns;   /* wrapping sum over modeled accesses */
    uint64_t max_done_ns;
    uint64_t fast_modeled_ns;  /* sum of fast_service_ns (FAST model) */
    uint64_t batches;
    uint64_t device_errors;    /* batches refused on the device */
} hbfsim_batch_stats_v1;

int hbfsim_get_batch_stats_v1(hbfsim_context* context,
                              hbfsim_batch_stats_v1* out);

/* ---- launch profiling ----
 * When enabled, every kernel launch of the context is bracketed by CUDA
 * events on its launching stream; hbfsim_get_kernel_times_v1 synchronizes,
 * adds up the device time of each kernel kind and clears the record.
 * Slots: 0 pass 1, 1 range scan, 2 pass 2, 3 sequential, 4 decode,
 *        5 thermal step, 6 epoch controller, 7 other. */
#define HBFSIM_KERNEL_SLOTS_V1 8
#define HBFSIM_KERNEL_TIMES_V1_VERSION 1u
typedef struct hbfsim_kernel_times_v1 {
    uint32_t struct_size;
    uint32_t version;
    uint64_t launches[HBFSIM_KERNEL_SLOTS_V1];
    double total_ms[HBFSIM_KERNEL_SLOTS_V1];
} hbfsim_kernel_times_v1;

int hbfsim_set_profiling_v1(hbfsim_context* context, int enable);
int hbfsim_get_kernel_times_v1(hbfsim_context* context,
                               hbfsim_kernel_times_v1* out);

/* ---- decode only (range lookup + stripe decode) ---- */
typedef struct hbfsim_decoded_v1 {
    uint64_t media_address;  /* page-aligned media address */
    uint64_t page;           /* page index inside the plane */
    uint32_t status;
    uint32_t range_index;
    uint32_t stack;
    uint32_t channel;        /* global channel */
    uint32_t die;
    uint32_t plane;
} hbfsim_decoded_v1;

/* Hybrid sampler bits (reference hybrid_reference_sample,
 * src/cuda_runtime/device/hbf_device.cuh:738-744, as resolve_fast_or_hybrid
 * applies it, hbf_device.cu:779-788): for each access the timing model would
 * serve (status 1), sample[i] = 1 when the hybrid model would send it to the
 * reference media model -- its sequence number is below the profile's
 * reference_warmup_requests, or the splitmix64 mix of
 * (sequence ^ media_address ^ range_id << 32 ^ operation) is at most
 * reference_sample_rate * UINT64_MAX; 0 for every other access.  Sequence
 * numbers are the context's running count of such accesses in batch order,
 * from 0 at context creation.  Device pointers; asynchronous on `stream`. */
int hbfsim_sample_batch_v1(hbfsim_context* context, const uint64_t* address,
                           const uint32_t* bytes, const uint8_t* operation,
                           uint64_t count, uint8_t* sample, void* stream);

int hbfsim_decode_batch_v1(hbfsim_context* context, const uint64_t* address,
                           const uint32_t* bytes, const uint8_t* operation,
                           uint64_t count, hbfsim_decoded_v1* out,
                           void* stream);

/* ---- refresh / throttle factors (per epoch) ----
 * refresh_permille[c]: share of local channel c's bandwidth taken by refresh
 *   (0..999); effective bandwidth = floor(bw * (1000 - r) / 1000).
 * throttle_permille[s]: die op-time multiplier of stack s (>= 1000).
 * admit_after_ns[s]: no access of stack s starts before this tick.
 * Any pointer may be NULL to leave that table unchanged.  Host pointers. */
int hbfsim_set_channel_factors_v1(hbfsim_context* context,
                                  const uint32_t* refresh_permille,
                                  const uint32_t* throttle_permille,
                                  const uint64_t* admit_after_ns);

/* ---- state checkpoint: raw little-endian die/channel state ----
 * Layout: local channel c, state[c*(D+1)] = channel free, then die d free.
 * FAST model: one word, the channel tail.  words = size of the buffer. */
int hbfsim_get_state_v1(hbfsim_context* context, uint64_t* host_words,
                        uint64_t words);
int hbfsim_set_state_v1(hbfsim_context* context, const uint64_t* host_words,
                        uint64_t words);
uint64_t hbfsim_state_words_v1(hbfsim_context* context);

/* ---- Capacity mode: exact LRU over HBM frames ----
 * Replaces CapacityPageService::resolve
 * (src/host_service/capacity_page_service.cpp:97-210) with the exact-LRU
 * policy of adapters/vllm_capacity/placement_policy.py:68-93, decided for a
 * whole batch at once.  Pages are LRU pages of page_bytes (default 4096,
 * a power of two no larger than the profile page) in media order:
 * page = (range file offset + offset in range) / page_bytes. */
int hbfsim_capacity_configure_v1(hbfsim_context* context, uint64_t frames,
                                 uint32_t page_bytes);

/* Replacement policy of the capacity path.  LRU (the default after
 * hbfsim_capacity_configure_v1) is the offline LruCache above, decided for
 * a whole batch at once.  CLOCK is the reference runtime's second-chance
 * policy: HbmCache::begin_eviction_locked
 * (src/cuda_runtime/hbm_cache.cpp:131-175) with the frame walk of
 * CapacityPageService::resolve (capacity_page_service.cpp:97-210) -- a hit
 * sets the frame's reference bit, a miss takes the lowest free frame or,
 * with every frame full, the first frame at or after the hand whose bit is
 * clear, clearing the set bits it passes.  Switching empties the cache.
 * With CLOCK, hbfsim_get_capacity_state_v1 lists the resident pages in
 * frame order.  Returns HBFSIM_INVALID_ARGUMENT before configure, for an
 * unknown policy, or for CLOCK over zero frames. */
#define HBFSIM_CAPACITY_POLICY_LRU 0u
#define HBFSIM_CAPACITY_POLICY_CLOCK 1u
int hbfsim_capacity_policy_v1(hbfsim_context* context, uint32_t policy);

#define HBFSIM_CAPACITY_BATCH_V1_VERSION 1u
typedef struct hbfsim_capacity_batch_v1 {
    uint32_t struct_size;
    uint32_t version;
    uint64_t count;
    const uint64_t* address;     /* in CAPACITY ranges; one LRU page each   */
    const uint32_t* bytes;
    const uint8_t* operation;    /* 0 read, 1 write (dirties the page)      */
    const uint64_t* arrival_ns;  /* needed when done_ns / latency_ns are set */
    uint8_t* hit;                /* out: 1 = resident in HBM                 */
    uint64_t* victim_page;       /* out: page evicted by this access,
                                  *      UINT64_MAX if none                  */
    uint8_t* victim_dirty;       /* out: 1 = the victim must be programmed   */
    uint8_t* status;             /* out: 1 capacity access, 6 unsupported,
                                  *      8 outside every range               */
    uint64_t* done_ns;           /* out (optional): completion tick          */
    uint64_t* latency_ns;        /* out (optional): done - arrival           */
} hbfsim_capacity_batch_v1;

/* Decides hit / victim / dirty for every access, in batch order, continuing
 * from the resident list the previous batch left.  Device pointers (NULL
 * outputs are skipped).  Synchronous: returns when the results are written.
 *
 * With done_ns or latency_ns set, the misses' media actions are timed with
 * the context's per-die model (mode 3, one shard), continuing its die and
 * channel state: for each miss in batch order, the program of a dirty
 * victim's page at the access's arrival, then the read of the missed page
 * at max(arrival, program completion) (request_dispatcher.cpp:107-126,
 * 294-298); one LRU page each, at its media address.  The actions are timed
 * in parallel, in rounds or pieces (hbfsim_get_capacity_rounds_v1).  A miss completes with
 * its read; hits (served from HBM) and non-capacity accesses complete at
 * their arrival. */
int hbfsim_submit_capacity_batch_v1(hbfsim_context* context,
                                    const hbfsim_capacity_batch_v1* batch,
                                    void* stream);

/* How the last timed batch resolved its chained reads (a miss's read that
 * waits for its dirty victim's program).  First up to 3 *rounds: timing
 * passes over all its media actions, each raising the chained reads to
 * their programs' completions, until none moves (a fixed point, equal to
 * timing the actions one at a time in batch order).  If that does not
 * settle, *pieces > 0: the actions were timed in that many pieces, each
 * starting at a chained read whose arrival its program's completion had
 * raised.  *walked = 1: more than 2^20 chained reads, one thread walked the
 * actions in order.  No counterpart in the reference, which times one
 * request at a time. */
int hbfsim_get_capacity_rounds_v1(hbfsim_context* context, uint32_t* rounds,
                                  uint64_t* pieces, uint32_t* walked);

/* The resident list, oldest first (host copies; NULL arrays return only
 * *resident). */
int hbfsim_get_capacity_state_v1(hbfsim_context* context, uint64_t* resident_pages,
                                 uint8_t* resident_dirty, uint64_t count,
                                 uint64_t* resident);

/* ---- eq3 thermal grid and epoch controller ---- */
#define HBFSIM_THERMAL_MAX_LAYERS 32
#define HBFSIM_THERMAL_CONFIG_V1_VERSION 1u
typedef struct hbfsim_thermal_layer_v1 {
    double thickness_m;
    double cv_j_m3_k;
    double k_xyz_w_m_k[3];
} hbfsim_thermal_layer_v1;

typedef struct hbfsim_thermal_config_v1 {
    uint32_t struct_size;
    uint32_t version;
    uint32_t nx, ny;            /* cells per layer (uniform square mesh) */
    uint32_t layer_count;       /* bottom (index 0) to top              */
    uint32_t reserved0;
    double cell_m;
    hbfsim_thermal_layer_v1 layers[HBFSIM_THERMAL_MAX_LAYERS];
    double bottom_h_w_m2_k, bottom_ambient_k;
    double top_h_w_m2_k, top_ambient_k;
    double initial_k;
    /* per-die power law: idle W + J per byte read + J per write access */
    double die_idle_w;
    double read_j_per_byte;
    double write_j_per_access;
    /* refresh law: base permille, doubling every refresh_step_k above
     * refresh_onset_k; capped at refresh_cap_permille */
    double refresh_onset_k;
    double refresh_step_k;
    uint32_t refresh_base_permille;
    uint32_t refresh_cap_permille;
    /* throttle (hysteresis levels Normal/Light/Severe/Shutdown on the hottest
     * die of a stack, cpu_service.cpp:221-247) */
    double light_k, severe_k, shutdown_k, hysteresis_k;
    uint32_t light_permille, severe_permille;
    uint32_t reserved1[2];
    /* floorplan: die (global channel g, die d) heats layers
     * [z0, z0+z_count) over the rectangle [x0,x1) x [y0,y1) in cells.
     * Arrays of length channels_total * dies, indexed g * dies + d.
     * Host pointers; copied at configure time. */
    const uint32_t* die_z0;
    const uint32_t* die_z_count;
    const uint32_t* die_x0;
    const uint32_t* die_x1;
    const uint32_t* die_y0;
    const uint32_t* die_y1;
} hbfsim_thermal_config_v1;

int hbfsim_thermal_configure_v1(hbfsim_context* context,
                                const hbfsim_thermal_config_v1* config);

/* Closes one epoch of `epoch_s` seconds: die activity recorded by the batches
 * since the previous epoch becomes power, the grid takes one backward-Euler
 * step, and the refresh / throttle factors of the next epoch are derived from
 * the new die temperatures.  Activity counters are then cleared.
 * On grids whose sides are multiples of 4 and up to about 150 cells the whole
 * close is one cooperative kernel (capturable in a CUDA graph); its waits
 * are bounded, and one that gives up makes the next hbfsim_flush return
 * HBFSIM_TIMEOUT (the epoch's temperatures and factors are then unspecified). */
int hbfsim_advance_epoch_v1(hbfsim_context* context, double epoch_s,
                            void* stream);

/* Sharded contexts (shard_count > 1): the same epoch step driven by the
 * all-gathered activity of every global die (device pointers, index
 * g*D+d, e.g. an NCCL all-gather of each rank's
 * hbfsim_copy_die_activity_v1 output).  The grid step is replicated on every
 * rank (deterministic fp64, same launches); each rank then derives the
 * factors of its own channels. */
int hbfsim_advance_epoch_global_v1(hbfsim_context* context, double epoch_s,
                                   const uint64_t* read_bytes,
                                   const uint64_t* writes, void* stream);

/* Copies this context's per-die activity since the last epoch (local die
 * index c*D+d) into caller device buffers, asynchronously on `stream`. */
int hbfsim_copy_die_activity_v1(hbfsim_context* context, uint64_t* read_bytes,
                                uint64_t* writes, void* stream);

/* Factors the epoch controller derived (host copies; NULL to skip):
 * refresh per local channel, throttle permille / admit-after tick / level
 * (0 Normal, 1 Light, 2 Severe, 3 Shutdown) per stack. */
int hbfsim_get_thermal_factors_v1(hbfsim_context* context,
                                  uint32_t* refresh_permille,
                                  uint32_t* throttle_permille,
                                  uint64_t* admit_after_ns, uint32_t* levels);

/* Host copies of the grid temperatures (nx*ny*layers, K, cell index
 * z*nx*ny + y*nx + x) and of per-die mean temperatures. */
int hbfsim_get_temperatures_v1(hbfsim_context* context, double* out,
                               uint64_t count);
int hbfsim_get_die_temperatures_v1(hbfsim_context* context, double* out,
                                   uint64_t count);
/* Per-die activity since the last epoch: read bytes and write count, local
 * die index c*D+d.  Host copies. */
int hbfsim_get_die_activity_v1(hbfsim_context* context, uint64_t* read_bytes,
                               uint64_t* writes, uint64_t count);
/* Factors currently in force (host copies; NULL to skip). */
int hbfsim_get_channel_factors_v1(hbfsim_context* context,
                                  uint32_t* refresh_permille,
                                  uint32_t* throttle_permille,
                                  uint64_t* admit_after_ns);

/* ---- per-block retention-age ledger ----
 * Replaces the reference's ReliabilityLedger
 * (experiments/eq3_system_thermal/reliability.py:26-232) as
 * run_maintenance_point.py:189, 225-234 drives it, for every physical block
 * of the context's local channels (die model only).  Block id:
 * ((local channel * D + die) * planes + plane) * blocks_per_plane + block,
 * blocks_per_plane = ceil(capacity / (channels_total * D * planes * page)
 * / pages_per_block).  All blocks share one accounted frontier.
 * hbfsim_set_geometry_v1 drops the ledger (its blocks follow the geometry);
 * configure it again afterwards. */
#define HBFSIM_RETENTION_CONFIG_V1_VERSION 1u
typedef struct hbfsim_retention_config_v1 {
    uint32_t struct_size;
    uint32_t version;
    double ea_ev;                  /* 1.01, 1.04 or 1.08 (reliability.py:9)    */
    double tref_k;                 /* fixed at 358.15 (reliability.py:41-43)  */
    uint64_t period_ns;            /* fixed at 24 h (reliability.py:44-46)    */
    uint64_t initial_age_ns;       /* initial_equivalent_age_ns               */
    uint64_t initial_wall_age_ns;  /* at most period_ns                       */
    uint64_t epoch_ns;             /* maintenance_epoch_ns: the start tick    */
    double initial_temperature_k;  /* every die's temperature at the start    */
    uint32_t refresh_trigger;      /* 0 wall_only, 1 equivalent_age_or_wall   */
    uint32_t reserved;
} hbfsim_retention_config_v1;

int hbfsim_retention_configure_v1(hbfsim_context* context,
                                  const hbfsim_retention_config_v1* config);
/* Number of blocks in the ledger (0 when not configured). */
uint64_t hbfsim_retention_blocks_v1(hbfsim_context* context);
/* Ages every block from the frontier to end_ns (advance_temperature_many,
 * reliability.py:109-135).  die_temp_k: device array of one temperature per
 * local die (c*D+d), used as is; NULL: the thermal model's die means, at the
 * midpoint of the previous and current value (run_maintenance_point.py:
 * 229-234).  Asynchronous on `stream`. */
int hbfsim_retention_advance_v1(hbfsim_context* context, uint64_t end_ns,
                                const double* die_temp_k, void* stream);
/* Blocks due at at_ns (due_reasons, reliability.py:76-88), ascending, with
 * reason bits (1 WALL_24H_SCENARIO_CADENCE, 2 EQUIVALENT_AGE_24H_
 * CONSERVATIVE_POLICY) into device arrays of `capacity` entries; *count
 * (host) gets the number due, which may exceed capacity.  Synchronous. */
int hbfsim_retention_due_v1(hbfsim_context* context, uint64_t at_ns,
                            uint32_t* blocks, uint8_t* reasons,
                            uint64_t capacity, uint64_t* count, void* stream);
/* Committed refresh of the listed blocks (device array) at the frontier
 * (record_refresh_terminal, reliability.py:172-187). */
int hbfsim_retention_refresh_v1(hbfsim_context* context, const uint32_t* blocks,
                                uint64_t count, void* stream);
/* Completed erases of the listed blocks (_media_terminal, 138-159). */
int hbfsim_retention_record_erase_v1(hbfsim_context* context,
                                     const uint32_t* blocks, uint64_t count,
                                     void* stream);
/* Every modeled write of an access batch (device arrays) as one completed
 * program of its block (record_program, reliability.py:161-165). */
int hbfsim_retention_record_programs_v1(hbfsim_context* context,
                                        const uint64_t* address,
                                        const uint32_t* bytes,
                                        const uint8_t* operation,
                                        uint64_t count, void* stream);
/* Host copies (NULL to skip): equivalent age (ns, fp64), next wall due,
 * last committed refresh (UINT64_MAX: none), counts [4][blocks] (program
 * started, program completed, erase started, erase completed), frontier.
 * Returns HBFSIM_INVALID_ARGUMENT once after a device-side rejection (a
 * temperature not finite and positive, a block id out of range). */
int hbfsim_get_retention_v1(hbfsim_context* context, double* age_ns,
                            uint64_t* next_wall_due_ns,
                            uint64_t* last_refresh_commit_ns, uint32_t* counts,
                            uint64_t blocks, uint64_t* frontier_ns);

/* ---- prefetch model sweeps ----
 * Replaces hbfsim::simulate_prefetch (src/prefetch/prefetch_model.cpp:117-195,
 * include/hbfsim/prefetch_model.hpp:24-99) over many configurations at once:
 * every cell walks the same page stream with its own policy, accuracy, lead
 * distance, staging buffer, media concurrency, read latency, compute time
 * per access and predictor seed.  Results equal the reference's, cell for
 * cell. */
typedef struct hbfsim_prefetch_cell_v1 {
    uint32_t policy;                  /* 0 None, 1 NextPage, 2 Accuracy */
    uint32_t lead_distance;
    double accuracy;
    uint32_t buffer_pages;
    uint32_t max_in_flight;
    uint64_t read_latency_ns;
    uint64_t compute_ns_per_access;
    uint64_t seed;
} hbfsim_prefetch_cell_v1;

typedef struct hbfsim_prefetch_stats_v1 {
    uint64_t total_ns;
    uint64_t stall_ns;
    uint64_t demand_accesses;
    uint64_t demand_misses;
    uint64_t prefetch_hits;
    uint64_t prefetch_issued;
    uint64_t prefetch_wasted;
} hbfsim_prefetch_stats_v1;

/* pages: device array of `count` media pages in demand order; cells and
 * out: host arrays of cell_count entries.  Synchronous on `stream`.
 * HBFSIM_UNSUPPORTED for a staging buffer beyond about 8,000 pages or a
 * stream of 2^32 - 2 accesses or more. */
int hbfsim_prefetch_sweep_v1(const uint64_t* pages, uint64_t count,
                             const hbfsim_prefetch_cell_v1* cells,
                             uint32_t cell_count, hbfsim_prefetch_stats_v1* out,
                             void* stream);

/* ---- UCIe streaming-link timing ----
 * Replaces hbfsim::ucie::StreamingLink (src/ucie/link.cpp,
 * include/hbfsim/ucie/link.hpp:54-113) for batches of independent links
 * (one per stack, module or sweep cell), each driven as follows: its
 * messages are offered in input order; the next one is enqueued at
 * max(ready, the link's tick) once its direction has fewer than
 * max_accepted messages in flight and its ready tick is not past the link's
 * next event; after each step every delivered message is consumed
 * consume_ns[direction] later.  Delivery ticks and counters equal the
 * reference link's under that driver. */
typedef struct hbfsim_link_profile_v1 {
    uint32_t gt_per_second;        /* 8, 16 or 32 (x64 lanes)               */
    uint32_t initial_ar_granules;  /* 3 .. 65535                            */
    uint32_t initial_r_granules;   /* 14 .. 65535                           */
    uint32_t max_accepted;         /* messages in flight per direction     */
    uint64_t propagation_ns;       /* at most 1e9                           */
    uint64_t consume_ns[2];        /* consumer delay: 0 AR, 1 R             */
} hbfsim_link_profile_v1;

typedef struct hbfsim_link_result_v1 {
    /* per direction (0 AR, 1 R): flits, wire bytes, UCIe header bytes, CRC
     * bytes, AoU header bytes, AoU message bytes, unused message bytes,
     * credit-only flits (link.hpp:38-48 DirectionCounters) */
    uint64_t counters[2][8];
    uint64_t now;                  /* the link's last event tick           */
    uint32_t ar_credits;
    uint32_t r_credits;
    int32_t status;                /* 0, or an hbfsim_error for this link  */
    uint32_t reserved;
} hbfsim_link_result_v1;

/* links: count; profiles, offsets (links + 1, messages of link k are
 * [offsets[k], offsets[k+1])) and results: host arrays; direction (0 AR,
 * 1 R), ready (non-decreasing per link) and delivered: device arrays.
 * Synchronous on `stream`. */
int hbfsim_link_batch_v1(const hbfsim_link_profile_v1* profiles, uint32_t links,
                         const uint64_t* offsets, const uint8_t* direction,
                         const uint64_t* ready, uint64_t* delivered,
                         hbfsim_link_result_v1* results, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HBFSIM_BATCH_V1_H */
