/*
 * hbf_oracle.h -- CPU restatement of the HBFSim batched access-timing path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code.  It is the checker that the CUDA path is compared against
 * (tests/, __graft_entry__.smoke(), and bench.py's cpu_baseline leg only).
 *
 * Every function cites the reference file:line it restates.  Paths are
 * relative to the HBFSim source tree.
 *
 * Parity status:
 *   - range lookup / media descriptor / fast model arithmetic: pinned to the
 *     reference (src/cuda_runtime/device/hbf_device.cuh) by golden vectors
 *     produced from the reference headers compiled here (oracle/Makefile).
 *   - per-die max-plus model, stripe decode, refresh/throttle scaling: the
 *     reference has no implementation (MQSim is an absent submodule), so the
 *     semantics are fixed by this build and written out below.  PARITY
 *     UNPINNED for those parts.
 */
#ifndef HBF_ORACLE_H
#define HBF_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Per-access status codes written by the batch path. */
enum {
    OR_STATUS_MODELED = 1,      /* timed by the model (reference: Ready)      */
    OR_STATUS_UNSUPPORTED = 6,  /* rejected (reference: Unsupported)          */
    OR_STATUS_BYPASS = 8,       /* outside every range: native HBM, untimed  */
    OR_STATUS_FOREIGN = 9       /* belongs to another shard's channels       */
};

enum { OR_MODEL_FAST = 1, OR_MODEL_DIE = 3 };

/* One registered range (the fields of SharedRangeRecord that the path reads,
 * hbf_device.cuh:105-118). */
typedef struct or_range {
    uint64_t base;
    uint64_t length;
    uint64_t file_offset;
    uint32_t range_id;
    uint32_t mode;         /* 1 timing, 2 capacity */
    uint32_t permissions;  /* bit0 read, bit1 write */
    uint32_t reserved;
    uint64_t page_bytes;
} or_range;

typedef struct or_geometry {
    uint32_t stacks;
    uint32_t channels_per_stack;
    uint32_t dies_per_channel;
    uint32_t planes_per_die;
    uint32_t stripe_bytes;     /* power of two */
    uint32_t page_bytes;
    uint8_t order[4];          /* fastest-varying first: 0=C 1=W 2=D 3=P */
    uint32_t shard_rank;       /* channel g belongs to shard g % shard_count */
    uint32_t shard_count;
} or_geometry;

typedef struct or_timing {
    uint32_t model;                 /* OR_MODEL_FAST or OR_MODEL_DIE */
    uint32_t time_scale;
    uint64_t read_latency_ns;
    uint64_t program_latency_ns;
    uint64_t aggregate_bandwidth;   /* bytes/s, FAST model */
    uint64_t page_bytes;            /* FAST model transfer size */
} or_timing;

typedef struct or_decoded {
    uint64_t media_address;  /* page-aligned media address (media_descriptor) */
    uint64_t page;           /* page index inside the plane */
    uint32_t status;
    uint32_t range_index;
    uint32_t stack;
    uint32_t channel;        /* global channel, 0 .. stacks*channels-1 */
    uint32_t die;
    uint32_t plane;
} or_decoded;

typedef struct or_stats {
    uint64_t modeled;
    uint64_t bypass;
    uint64_t unsupported;
    uint64_t foreign;
    uint64_t fast_modeled_ns;   /* sum of fast_service_ns (FAST model) */
    uint64_t latency_sum;       /* saturating sum of latency, modeled only */
    uint64_t max_done;          /* simulated time after the batch */
} or_stats;

/* ---- reference arithmetic (hbf_device.cuh) ---- */
uint64_t or_saturating_add(uint64_t a, uint64_t b);
uint64_t or_saturating_multiply(uint64_t a, uint32_t b);
uint64_t or_fast_transfer_ns(uint32_t bytes, uint64_t bandwidth);
uint64_t or_fast_service_ns(uint64_t base_latency, uint32_t bytes,
                            uint64_t bandwidth);
uint32_t or_find_range_index(const or_range* ranges, uint32_t count,
                             uint64_t address);
int or_access_supported(const or_range* r, uint64_t address, uint32_t bytes,
                        uint32_t op);
int or_range_overlaps(const or_range* r, uint64_t address, uint32_t bytes);
int or_media_descriptor(const or_range* r, uint64_t address, uint32_t bytes,
                        uint32_t op, uint64_t* logical_address,
                        uint32_t* media_bytes);
/* Sampling threshold from a profile's reference_sample_rate
 * (src/cuda_runtime/context.cpp:975-981): UINT64_MAX for rate >= 1, else
 * rate * (long double) UINT64_MAX truncated. */
uint64_t or_sample_threshold(double rate);

int or_hybrid_reference_sample(uint64_t sequence, uint32_t warmup,
                               uint64_t threshold, uint64_t key);

/* ---- classification + decode of a whole batch ---- */
void or_decode_batch(const or_range* ranges, uint32_t count,
                     const or_geometry* g, const uint64_t* address,
                     const uint32_t* bytes, const uint8_t* op, uint64_t n,
                     or_decoded* out);

/* ---- timing ----
 * state layout (uint64 each):
 *   FAST: state[0] = fast channel tail
 *   DIE : per local channel c: state[c*(D+1)] = channel free,
 *         state[c*(D+1)+1+d] = die d free.
 * chan_bw[c]: effective channel bandwidth of local channel c (DIE only).
 * t_read[s], t_prog[s]: die op times of stack s, already throttled (DIE).
 * admit[s]: no access of stack s starts before this tick (DIE; NULL = 0).
 */
int or_run_batch(const or_range* ranges, uint32_t count, const or_geometry* g,
                 const or_timing* t, const uint64_t* chan_bw,
                 const uint64_t* t_read, const uint64_t* t_prog,
                 const uint64_t* admit, const uint64_t* address, const uint32_t* bytes,
                 const uint8_t* op, const uint64_t* arrival, uint64_t n,
                 uint64_t* state, uint64_t* done, uint64_t* latency,
                 uint8_t* status, or_stats* stats);

/* Multithreaded variant of the DIE model, sharded by channel over host
 * threads (channels are independent).  Same results as or_run_batch. */
int or_run_batch_threads(const or_range* ranges, uint32_t count,
                         const or_geometry* g, const or_timing* t,
                         const uint64_t* chan_bw, const uint64_t* t_read,
                         const uint64_t* t_prog, const uint64_t* admit,
                         const uint64_t* address,
                         const uint32_t* bytes, const uint8_t* op,
                         const uint64_t* arrival, uint64_t n, uint64_t* state,
                         uint64_t* done, uint64_t* latency, uint8_t* status,
                         or_stats* stats, int threads);

/* ---- capacity mode: exact LRU over frames (placement_policy.py:68-93) ----
 * pages[i]: logical page of access i, writes[i]: 1 for a write.
 * Outputs per access: hit (1/0), victim page (UINT64_MAX if none),
 * victim_dirty (1 if the evicted page had been written while resident). */
void or_lru_run(const uint64_t* pages, const uint8_t* writes, uint64_t n,
                uint64_t frames, uint8_t* hit, uint64_t* victim,
                uint8_t* victim_dirty);

/* ---- capacity mode: second-chance CLOCK (the reference runtime's policy,
 * src/cuda_runtime/hbm_cache.cpp:131-175 driven by
 * capacity_page_service.cpp:97-210).  State carries across runs. */
void* or_clock_new(uint64_t frames);
void or_clock_free(void* state);
void or_clock_run(void* state, const uint64_t* pages, const uint8_t* writes, uint64_t n,
                  uint8_t* hit, uint64_t* victim, uint8_t* victim_dirty);

/* ---- capacity mode: media actions of the misses, timed with the die model
 * in batch order (request_dispatcher.cpp:107-126, 294-298): for a miss, the
 * program of a dirty victim's page at the access's arrival, then the read of
 * the missed page at max(arrival, program completion); one LRU page
 * (2^page_shift bytes) each, at its media address (page << page_shift).
 * Hits and non-capacity accesses (status != 1) complete at their arrival. */
void or_capacity_timing(const or_geometry* g, const or_timing* t,
                        const uint64_t* chan_bw, const uint64_t* t_read,
                        const uint64_t* t_prog, const uint64_t* admit,
                        const uint8_t* status, const uint8_t* hit, const uint64_t* page,
                        const uint64_t* victim, const uint8_t* victim_dirty,
                        const uint64_t* arrival, uint64_t n, uint32_t page_shift,
                        uint64_t* state, uint64_t* done, uint64_t* latency);

/* ---- empirical burst-curve profile (FAST model with empirical_vmem) ----
 * hbf_device.cuh:959-1140 and the empirical branch of resolve_fast_or_hybrid
 * (hbf_device.cu:797-838). */
typedef struct or_empirical {
    uint32_t flags;               /* header empirical_flags (1 = on) */
    uint32_t count;               /* header empirical_point_count */
    uint64_t program_latency_ns;  /* header program_latency_ns */
    uint32_t pages[6];
    uint64_t cumulative_ns[6];
} or_empirical;

uint64_t or_empirical_cumulative_ns(const uint32_t* pages, const uint64_t* cumulative,
                                    uint32_t count, uint32_t run_pages);
uint64_t or_empirical_service_ns(const uint32_t* pages, const uint64_t* cumulative,
                                 uint32_t count, uint32_t run_pages);
/* Returns 1 when valid; *packed and *run_pages get the new state (on an
 * invalid update *packed keeps `previous` and *run_pages is 0). */
int or_update_empirical_burst(uint64_t previous, uint64_t page, uint32_t operation,
                              uint64_t* packed, uint32_t* run_pages);
int or_empirical_control_valid(const or_empirical* e);
/* Returns 1 when valid; all outputs 0 otherwise. */
int or_empirical_request_service(const or_empirical* e, uint64_t previous, uint64_t page,
                                 uint32_t operation, uint64_t* service_ns,
                                 uint64_t* packed, uint32_t* run_pages);
/* A batch of the empirical FAST model: classification as or_run_batch, then
 * per timed access in (arrival, index) order the empirical branch's checks
 * (a 4 KiB media page on a 4 KiB boundary, time_scale and request timeout
 * nonzero, the header valid: else Unsupported), the burst update and the
 * tail step target = max(tail, arrival) + service * time_scale.
 * state[0] = channel tail, state[1] = packed burst state. */
int or_run_empirical_batch(const or_range* ranges, uint32_t count, const or_empirical* e,
                           uint32_t time_scale, uint64_t request_timeout_ns,
                           const uint64_t* address, const uint32_t* bytes,
                           const uint8_t* op, const uint64_t* arrival, uint64_t n,
                           uint64_t* state, uint64_t* done, uint64_t* latency,
                           uint8_t* status, or_stats* stats);

/* ---- prefetch model (src/prefetch/prefetch_model.cpp, include/hbfsim/
 * prefetch_model.hpp): a discrete-event walk of a page stream with a
 * prefetcher, a FIFO staging buffer and max_in_flight media servers. ---- */
typedef struct or_prefetch_cell {
    uint32_t policy;          /* 0 none, 1 next page, 2 accuracy */
    uint32_t lead_distance;
    double accuracy;
    uint32_t buffer_pages;
    uint32_t max_in_flight;
    uint64_t read_latency_ns;
    uint64_t compute_ns_per_access;
    uint64_t seed;
} or_prefetch_cell;

typedef struct or_prefetch_stats {
    uint64_t total_ns;
    uint64_t stall_ns;
    uint64_t demand_accesses;
    uint64_t demand_misses;
    uint64_t prefetch_hits;
    uint64_t prefetch_issued;
    uint64_t prefetch_wasted;
} or_prefetch_stats;

/* Returns 0, or -1 when memory runs out. */
int or_prefetch_run(const uint64_t* pages, uint64_t n, const or_prefetch_cell* cell,
                    or_prefetch_stats* stats);

/* ---- UCIe streaming link (src/ucie/link.cpp, include/hbfsim/ucie/link.hpp:
 * Format 6 flits of 48 AoU granules, AR 3 / R 14 granules per message,
 * credits returned as legal grants on the reverse direction's flits) under
 * the batch driver: messages offered in input order, enqueued at
 * max(ready, link time) once their direction has room and their ready time
 * is not past the next event; each delivery consumed consume_ns[direction]
 * later. ---- */
typedef struct or_link_profile {
    uint32_t gt_per_second;       /* 8, 16 or 32 */
    uint32_t initial_ar_granules;
    uint32_t initial_r_granules;
    uint32_t max_accepted;
    uint64_t propagation_ns;
    uint64_t consume_ns[2];       /* 0 request (AR), 1 return (R) */
} or_link_profile;

typedef struct or_link_result {
    /* per direction: flits, wire bytes, UCIe header bytes, CRC bytes, AoU
     * header bytes, AoU message bytes, unused message bytes, credit-only flits */
    uint64_t counters[2][8];
    uint64_t now;
    uint32_t ar_credits;
    uint32_t r_credits;
    uint64_t heap_peak;   /* most events pending at once (bounds the device heap) */
} or_link_result;

/* direction[k] (0 AR, 1 R) and ready[k] (non-decreasing) of m messages;
 * delivered[k] gets each message's delivery tick.  0, or -1 on a time or
 * credit overflow (the reference throws) or when memory runs out. */
int or_link_run(const or_link_profile* p, const uint8_t* direction, const uint64_t* ready,
                uint64_t m, uint64_t* delivered, or_link_result* out);

#ifdef __cplusplus
}
#endif
#endif
