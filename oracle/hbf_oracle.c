/*
 * hbf_oracle.c -- CPU restatement of the HBFSim batched access-timing path.
 *
 * TEST INFRASTRUCTURE ONLY (see hbf_oracle.h).  Plain C, single file, built by
 * oracle/Makefile into oracle/libhbf_oracle.so.  The shipped library never
 * links or loads it.
 */
#include "hbf_oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define U64MAX UINT64_MAX

/* hbf_device.cuh:946-950 */
uint64_t or_saturating_add(uint64_t left, uint64_t right)
{
    return right > U64MAX - left ? U64MAX : left + right;
}

/* hbf_device.cuh:952-957 */
uint64_t or_saturating_multiply(uint64_t left, uint32_t right)
{
    return right != 0 && left > U64MAX / right ? U64MAX : left * right;
}

/* hbf_device.cuh:746-757 (64-bit wrapping arithmetic, as the reference) */
uint64_t or_fast_transfer_ns(uint32_t bytes, uint64_t bandwidth)
{
    if (bytes == 0 || bandwidth == 0) return 0;
    const uint64_t numerator = (uint64_t)bytes * 1000000000ULL;
    return (numerator + bandwidth - 1) / bandwidth;
}

/* hbf_device.cuh:797-817: the later of latency and transfer, not the sum */
uint64_t or_fast_service_ns(uint64_t base_latency, uint32_t bytes,
                            uint64_t bandwidth)
{
    const uint64_t transfer = or_fast_transfer_ns(bytes, bandwidth);
    return transfer > base_latency ? transfer : base_latency;
}

/* hbf_device.cuh:826-841: upper-bound binary search on sorted bases */
uint32_t or_find_range_index(const or_range* ranges, uint32_t count,
                             uint64_t address)
{
    uint32_t first = 0, last = count;
    while (first < last) {
        const uint32_t middle = first + (last - first) / 2;
        if (ranges[middle].base <= address) first = middle + 1;
        else last = middle;
    }
    return first == 0 ? count : first - 1;
}

/* hbf_device.cuh:843-862 */
int or_access_supported(const or_range* r, uint64_t address, uint32_t bytes,
                        uint32_t op)
{
    if (bytes == 0 || op > 1 || (r->mode != 1 && r->mode != 2) ||
        r->page_bytes == 0 || r->page_bytes > UINT32_MAX ||
        r->length > U64MAX - r->base || address < r->base ||
        address - r->base >= r->length || bytes > U64MAX - address ||
        address + bytes > r->base + r->length ||
        (r->permissions & (1u << op)) == 0)
        return 0;
    const uint64_t offset = address - r->base;
    const uint64_t last_offset = offset + bytes - 1;
    return offset / r->page_bytes == last_offset / r->page_bytes;
}

/* hbf_device.cuh:873-884 */
int or_range_overlaps(const or_range* r, uint64_t address, uint32_t bytes)
{
    if (bytes == 0 || r->length == 0 || r->base > U64MAX - r->length ||
        address > U64MAX - bytes)
        return 0;
    return address < r->base + r->length && r->base < address + bytes;
}

/* hbf_device.cuh:929-944 */
int or_media_descriptor(const or_range* r, uint64_t address, uint32_t bytes,
                        uint32_t op, uint64_t* logical_address,
                        uint32_t* media_bytes)
{
    if (!or_access_supported(r, address, bytes, op)) return 0;
    const uint64_t page_offset =
        ((address - r->base) / r->page_bytes) * r->page_bytes;
    if (page_offset > U64MAX - r->file_offset) return 0;
    *logical_address = r->file_offset + page_offset;
    *media_bytes = (uint32_t)r->page_bytes;
    return 1;
}

/* hbf_device.cuh:729-744 */
static uint64_t or_fast_hash(uint64_t value)
{
    value += 0x9e3779b97f4a7c15ULL;
    value = (value ^ (value >> 30)) * 0xbf58476d1ce4e5b9ULL;
    value = (value ^ (value >> 27)) * 0x94d049bb133111ebULL;
    return value ^ (value >> 31);
}

uint64_t or_sample_threshold(double rate)
{
    if (rate >= 1.0) return UINT64_MAX;
    return (uint64_t)(rate * (long double)UINT64_MAX);
}

int or_hybrid_reference_sample(uint64_t sequence, uint32_t warmup,
                               uint64_t threshold, uint64_t key)
{
    return sequence < warmup ||
           (threshold != 0 && or_fast_hash(sequence ^ key) <= threshold);
}

/* Classification of one access, restating the order of checks in
 * __hbfsim_resolve (hbf_device.cu:997-1003 zero bytes, 1083-1127 lookup,
 * straddle into the successor range and bypass, 1152-1179 media descriptor).
 * Capacity-mode ranges go through the capacity path, not the timing batch. */
static uint32_t or_classify(const or_range* ranges, uint32_t count,
                            uint64_t address, uint32_t bytes, uint32_t op,
                            uint32_t* range_index, uint64_t* media)
{
    *range_index = count;
    *media = 0;
    if (bytes == 0) return OR_STATUS_UNSUPPORTED;
    const uint32_t index = or_find_range_index(ranges, count, address);
    if (index == count || address < ranges[index].base ||
        address - ranges[index].base >= ranges[index].length) {
        const uint32_t successor = index == count ? 0u : index + 1u;
        if (successor < count &&
            or_range_overlaps(&ranges[successor], address, bytes))
            return OR_STATUS_UNSUPPORTED;
        return OR_STATUS_BYPASS;
    }
    uint32_t media_bytes = 0;
    if (!or_media_descriptor(&ranges[index], address, bytes, op, media,
                             &media_bytes))
        return OR_STATUS_UNSUPPORTED;
    if (ranges[index].mode != 1) return OR_STATUS_UNSUPPORTED;
    *range_index = index;
    return OR_STATUS_MODELED;
}

/* Stripe decode (builder-fixed semantics; parity unpinned).
 *   m  = file_offset + (address - base)         media byte offset
 *   u  = m / stripe_bytes                        stripe unit
 *   u is split as a mixed-radix number in the profile's allocation order,
 *   fastest letter first (CWDP: channel, way, die, plane), radices
 *   C = stacks * channels_per_stack, W = 1, D = dies, P = planes.  The rest is
 *   the row inside the plane.  Global channel g: stack = g % stacks,
 *   channel-in-stack = g / stacks (the page-stripe placement of
 *   src/ucie/stack_router.cpp:205-218).  Page inside the plane =
 *   (row * stripe + m % stripe) / page_bytes. */
static void or_decode_one(const or_geometry* g, uint64_t m, or_decoded* d)
{
    uint64_t radix[4];
    radix[0] = (uint64_t)g->stacks * g->channels_per_stack;
    radix[1] = 1;
    radix[2] = g->dies_per_channel;
    radix[3] = g->planes_per_die;
    uint64_t digit[4] = {0, 0, 0, 0};
    uint64_t u = m / g->stripe_bytes;
    for (int k = 0; k < 4; ++k) {
        const int letter = g->order[k];
        digit[letter] = u % radix[letter];
        u /= radix[letter];
    }
    d->channel = (uint32_t)digit[0];
    d->stack = (uint32_t)(digit[0] % g->stacks);
    d->die = (uint32_t)digit[2];
    d->plane = (uint32_t)digit[3];
    d->page = (u * g->stripe_bytes + m % g->stripe_bytes) / g->page_bytes;
}

void or_decode_batch(const or_range* ranges, uint32_t count,
                     const or_geometry* g, const uint64_t* address,
                     const uint32_t* bytes, const uint8_t* op, uint64_t n,
                     or_decoded* out)
{
    for (uint64_t i = 0; i < n; ++i) {
        or_decoded d;
        memset(&d, 0, sizeof d);
        uint64_t media = 0;
        d.status = or_classify(ranges, count, address[i], bytes[i], op[i],
                               &d.range_index, &media);
        d.media_address = media;
        if (d.status == OR_STATUS_MODELED) {
            const or_range* r = &ranges[d.range_index];
            or_decode_one(g, r->file_offset + (address[i] - r->base), &d);
            if (g->shard_count > 1 &&
                d.channel % g->shard_count != g->shard_rank)
                d.status = OR_STATUS_FOREIGN;
        }
        out[i] = d;
    }
}

/* ceil(bytes * 1e9 / bandwidth), exact (128-bit). */
static uint64_t or_channel_transfer_ns(uint32_t bytes, uint64_t bandwidth)
{
    if (bytes == 0 || bandwidth == 0) return 0;
    const unsigned __int128 num = (unsigned __int128)bytes * 1000000000ULL;
    const unsigned __int128 q = (num + bandwidth - 1) / bandwidth;
    return q > U64MAX ? U64MAX : (uint64_t)q;
}

/* ---- ordering: (arrival, index), stable ---- */
static const uint64_t* g_sort_arrival;
static int or_cmp_index(const void* a, const void* b)
{
    const uint64_t ia = *(const uint64_t*)a, ib = *(const uint64_t*)b;
    const uint64_t aa = g_sort_arrival[ia], ab = g_sort_arrival[ib];
    if (aa != ab) return aa < ab ? -1 : 1;
    return ia < ib ? -1 : (ia > ib ? 1 : 0);
}

static uint64_t* or_arrival_order(const uint64_t* arrival, uint64_t n)
{
    uint64_t* order = (uint64_t*)malloc(sizeof(uint64_t) * (n ? n : 1));
    if (!order) return NULL;
    int sorted = 1;
    for (uint64_t i = 0; i < n; ++i) {
        order[i] = i;
        if (i && arrival[i] < arrival[i - 1]) sorted = 0;
    }
    if (!sorted) {
        g_sort_arrival = arrival;
        qsort(order, n, sizeof(uint64_t), or_cmp_index);
    }
    return order;
}

/* FAST model step: hbf_device.cu:883-910 (tail CAS loop and target), with the
 * access's arrival tick in place of %globaltimer. */
static uint64_t or_fast_step(uint64_t* tail, uint64_t arrival, uint64_t x,
                             uint64_t latency_scaled)
{
    const uint64_t start = *tail > arrival ? *tail : arrival;
    *tail = or_saturating_add(start, x);
    const uint64_t latency_target = or_saturating_add(arrival, latency_scaled);
    return latency_target > *tail ? latency_target : *tail;
}

/* DIE model step (builder-fixed semantics, parity unpinned):
 *   start = max(arrival, channel_free, die_free[d])
 *   channel_free = start + X          (channel carries command + data)
 *   die_free[d]  = channel_free + T   (die runs tR / tPROG)
 *   done = die_free[d]                                        */
static uint64_t or_die_step(uint64_t* chan, uint64_t* die, uint64_t arrival,
                            uint64_t admit, uint64_t x, uint64_t t)
{
    uint64_t start = arrival > admit ? arrival : admit;
    if (*chan > start) start = *chan;
    if (*die > start) start = *die;
    *chan = or_saturating_add(start, x);
    *die = or_saturating_add(*chan, t);
    return *die;
}

typedef struct or_job {
    const or_range* ranges;
    const or_geometry* g;
    const or_timing* t;
    const uint64_t* chan_bw;
    const uint64_t* t_read;
    const uint64_t* t_prog;
    const uint64_t* admit;
    const uint32_t* bytes;
    const uint8_t* op;
    const uint64_t* arrival;
    const or_decoded* dec;
    const uint64_t* order;      /* modeled accesses in (arrival, index) order */
    uint64_t order_n;
    uint64_t* state;
    uint64_t* done;
    uint64_t* latency;
    uint32_t channel_begin, channel_end;  /* local channels this job owns */
    uint64_t latency_sum;
    uint64_t max_done;
    uint64_t fast_modeled_ns;
} or_job;

static void or_run_job(or_job* j)
{
    const or_geometry* g = j->g;
    const or_timing* t = j->t;
    const uint32_t dies = g->dies_per_channel;
    const uint32_t shards = g->shard_count ? g->shard_count : 1;
    for (uint64_t k = 0; k < j->order_n; ++k) {
        const uint64_t i = j->order[k];
        const or_decoded* d = &j->dec[i];
        const uint64_t a = j->arrival[i];
        uint64_t done;
        if (t->model == OR_MODEL_FAST) {
            const or_range* r = &j->ranges[d->range_index];
            const uint64_t base = j->op[i] ? t->program_latency_ns
                                           : t->read_latency_ns;
            const uint64_t x = or_saturating_multiply(
                or_fast_transfer_ns((uint32_t)r->page_bytes,
                                    t->aggregate_bandwidth),
                t->time_scale);
            done = or_fast_step(&j->state[0], a, x,
                                or_saturating_multiply(base, t->time_scale));
            j->fast_modeled_ns += or_fast_service_ns(
                base, (uint32_t)r->page_bytes, t->aggregate_bandwidth);
        } else {
            const uint32_t c = d->channel / shards;
            if (c < j->channel_begin || c >= j->channel_end) continue;
            uint64_t* st = &j->state[(uint64_t)c * (dies + 1)];
            const uint64_t x = or_saturating_multiply(
                or_channel_transfer_ns(j->bytes[i], j->chan_bw[c]),
                t->time_scale);
            const uint64_t top = j->op[i] ? j->t_prog[d->stack]
                                          : j->t_read[d->stack];
            const uint64_t tt = or_saturating_multiply(top, t->time_scale);
            const uint64_t adm = j->admit ? j->admit[d->stack] : 0;
            done = or_die_step(&st[0], &st[1 + d->die], a, adm, x, tt);
        }
        j->done[i] = done;
        j->latency[i] = done - a;
        j->latency_sum = or_saturating_add(j->latency_sum, done - a);
        if (done > j->max_done) j->max_done = done;
    }
}

static void* or_thread_main(void* arg)
{
    or_run_job((or_job*)arg);
    return NULL;
}

typedef struct or_decode_job {
    const or_range* ranges;
    uint32_t count;
    const or_geometry* g;
    const uint64_t* address;
    const uint32_t* bytes;
    const uint8_t* op;
    uint64_t begin, end;
    or_decoded* out;
} or_decode_job;

static void* or_decode_main(void* arg)
{
    or_decode_job* j = (or_decode_job*)arg;
    or_decode_batch(j->ranges, j->count, j->g, j->address + j->begin,
                    j->bytes + j->begin, j->op + j->begin, j->end - j->begin,
                    j->out + j->begin);
    return NULL;
}

int or_run_batch_threads(const or_range* ranges, uint32_t count,
                         const or_geometry* g, const or_timing* t,
                         const uint64_t* chan_bw, const uint64_t* t_read,
                         const uint64_t* t_prog, const uint64_t* admit,
                         const uint64_t* address,
                         const uint32_t* bytes, const uint8_t* op,
                         const uint64_t* arrival, uint64_t n, uint64_t* state,
                         uint64_t* done, uint64_t* latency, uint8_t* status,
                         or_stats* stats, int threads)
{
    memset(stats, 0, sizeof *stats);
    if (threads < 1) threads = 1;
    or_decoded* dec = (or_decoded*)malloc(sizeof(or_decoded) * (n ? n : 1));
    if (!dec) return -1;
    /* decode: independent per access, split over the threads */
    {
        or_decode_job* dj = (or_decode_job*)calloc((size_t)threads, sizeof(or_decode_job));
        pthread_t* tid = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
        for (int k = 0; k < threads; ++k) {
            dj[k].ranges = ranges; dj[k].count = count; dj[k].g = g;
            dj[k].address = address; dj[k].bytes = bytes; dj[k].op = op;
            dj[k].begin = n * (uint64_t)k / (uint64_t)threads;
            dj[k].end = n * (uint64_t)(k + 1) / (uint64_t)threads;
            dj[k].out = dec;
        }
        if (threads == 1) {
            or_decode_main(&dj[0]);
        } else {
            for (int k = 0; k < threads; ++k)
                pthread_create(&tid[k], NULL, or_decode_main, &dj[k]);
            for (int k = 0; k < threads; ++k) pthread_join(tid[k], NULL);
        }
        free(dj); free(tid);
    }
    uint64_t* order = or_arrival_order(arrival, n);
    if (!order) { free(dec); return -1; }
    uint64_t m = 0;
    for (uint64_t k = 0; k < n; ++k) {
        const uint64_t i = order[k];
        status[i] = (uint8_t)dec[i].status;
        done[i] = arrival[i];
        latency[i] = 0;
        switch (dec[i].status) {
        case OR_STATUS_MODELED: order[m++] = i; break;
        case OR_STATUS_BYPASS: stats->bypass++; break;
        case OR_STATUS_FOREIGN: stats->foreign++; break;
        default: stats->unsupported++; break;
        }
    }
    stats->modeled = m;
    const uint32_t shards = g->shard_count ? g->shard_count : 1;
    const uint32_t channels_total = g->stacks * g->channels_per_stack;
    const uint32_t local = (channels_total + shards - 1) / shards;
    if (t->model == OR_MODEL_FAST) threads = 1;
    if ((uint32_t)threads > local) threads = (int)local;
    or_job* jobs = (or_job*)calloc((size_t)threads, sizeof(or_job));
    pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    for (int k = 0; k < threads; ++k) {
        or_job* j = &jobs[k];
        j->ranges = ranges; j->g = g; j->t = t; j->chan_bw = chan_bw;
        j->t_read = t_read; j->t_prog = t_prog; j->admit = admit;
        j->bytes = bytes; j->op = op;
        j->arrival = arrival; j->dec = dec; j->order = order; j->order_n = m;
        j->state = state; j->done = done; j->latency = latency;
        j->channel_begin = (uint32_t)((uint64_t)local * k / threads);
        j->channel_end = (uint32_t)((uint64_t)local * (k + 1) / threads);
        if (t->model == OR_MODEL_FAST) { j->channel_begin = 0; j->channel_end = ~0u; }
    }
    if (threads == 1) {
        or_run_job(&jobs[0]);
    } else {
        for (int k = 0; k < threads; ++k)
            pthread_create(&tids[k], NULL, or_thread_main, &jobs[k]);
        for (int k = 0; k < threads; ++k) pthread_join(tids[k], NULL);
    }
    for (int k = 0; k < threads; ++k) {
        stats->latency_sum = or_saturating_add(stats->latency_sum,
                                               jobs[k].latency_sum);
        if (jobs[k].max_done > stats->max_done)
            stats->max_done = jobs[k].max_done;
        stats->fast_modeled_ns += jobs[k].fast_modeled_ns;
    }
    free(jobs); free(tids); free(order); free(dec);
    return 0;
}

int or_run_batch(const or_range* ranges, uint32_t count, const or_geometry* g,
                 const or_timing* t, const uint64_t* chan_bw,
                 const uint64_t* t_read, const uint64_t* t_prog,
                 const uint64_t* admit, const uint64_t* address, const uint32_t* bytes,
                 const uint8_t* op, const uint64_t* arrival, uint64_t n,
                 uint64_t* state, uint64_t* done, uint64_t* latency,
                 uint8_t* status, or_stats* stats)
{
    return or_run_batch_threads(ranges, count, g, t, chan_bw, t_read, t_prog,
                                admit, address, bytes, op, arrival, n, state, done,
                                latency, status, stats, 1);
}

/* ---- exact LRU (adapters/vllm_capacity/placement_policy.py:68-93) with the
 * dirty tracking of CapacityPageService::resolve
 * (src/host_service/capacity_page_service.cpp:97-210): a write marks the page
 * dirty whether it hit or missed; an evicted dirty page must be programmed. */
typedef struct { uint64_t key; int64_t node; } or_slot;

static uint64_t or_mix(uint64_t x) { return or_fast_hash(x); }

void or_lru_run(const uint64_t* pages, const uint8_t* writes, uint64_t n,
                uint64_t frames, uint8_t* hit, uint64_t* victim,
                uint8_t* victim_dirty)
{
    if (frames == 0) {
        for (uint64_t i = 0; i < n; ++i) {
            hit[i] = 0; victim[i] = U64MAX; victim_dirty[i] = 0;
        }
        return;
    }
    uint64_t cap = 16;
    while (cap < frames * 2 + 16) cap <<= 1;
    or_slot* table = (or_slot*)malloc(sizeof(or_slot) * cap);
    for (uint64_t k = 0; k < cap; ++k) table[k].node = -1;
    /* nodes: doubly linked list, head = most recent */
    uint64_t* key = (uint64_t*)malloc(sizeof(uint64_t) * frames);
    int64_t* prev = (int64_t*)malloc(sizeof(int64_t) * frames);
    int64_t* next = (int64_t*)malloc(sizeof(int64_t) * frames);
    uint8_t* dirty = (uint8_t*)malloc(frames);
    int64_t head = -1, tail = -1;
    uint64_t used = 0;
    const uint64_t mask = cap - 1;
#define OR_UNLINK(x) do { \
        if (prev[x] >= 0) next[prev[x]] = next[x]; else head = next[x]; \
        if (next[x] >= 0) prev[next[x]] = prev[x]; else tail = prev[x]; } while (0)
#define OR_PUSH_FRONT(x) do { prev[x] = -1; next[x] = head; \
        if (head >= 0) { prev[head] = x; } \
        head = x; \
        if (tail < 0) { tail = x; } } while (0)
    for (uint64_t i = 0; i < n; ++i) {
        const uint64_t p = pages[i];
        uint64_t h = or_mix(p) & mask;
        while (table[h].node >= 0 && table[h].key != p) h = (h + 1) & mask;
        victim[i] = U64MAX;
        victim_dirty[i] = 0;
        if (table[h].node >= 0) {
            const int64_t x = table[h].node;
            hit[i] = 1;
            if (writes[i]) dirty[x] = 1;
            OR_UNLINK(x);
            OR_PUSH_FRONT(x);
            continue;
        }
        hit[i] = 0;
        int64_t x;
        if (used < frames) {
            x = (int64_t)used++;
        } else {
            x = tail;
            victim[i] = key[x];
            victim_dirty[i] = dirty[x];
            OR_UNLINK(x);
            /* delete key[x] from the table (backward-shift deletion) */
            uint64_t d = or_mix(key[x]) & mask;
            while (table[d].key != key[x] || table[d].node != x)
                d = (d + 1) & mask;
            uint64_t hole = d, probe = (d + 1) & mask;
            table[hole].node = -1;
            while (table[probe].node >= 0) {
                const uint64_t ideal = or_mix(table[probe].key) & mask;
                const int moves = ((probe - ideal) & mask) >= ((probe - hole) & mask);
                if (moves) {
                    table[hole] = table[probe];
                    table[probe].node = -1;
                    hole = probe;
                }
                probe = (probe + 1) & mask;
            }
            h = or_mix(p) & mask;
            while (table[h].node >= 0) h = (h + 1) & mask;
        }
        key[x] = p;
        dirty[x] = writes[i] ? 1 : 0;
        table[h].key = p;
        table[h].node = x;
        OR_PUSH_FRONT(x);
    }
#undef OR_UNLINK
#undef OR_PUSH_FRONT
    free(table); free(key); free(prev); free(next); free(dirty);
}

/* Capacity mode with the reference runtime's policy: second-chance CLOCK
 * over `frames` frames, one page reference at a time, as
 * CapacityPageService::resolve (capacity_page_service.cpp:97-210) drives
 * HbmCache (hbm_cache.cpp): a resident page is a hit and gets its reference
 * bit (resolve, 41-52), a write also its dirty bit (mark_dirty, 80-94); a
 * miss takes the lowest free frame (free_frame, 101-110) or, once every
 * frame holds a page, the CLOCK victim (begin_eviction_locked, 131-175: the
 * hand walks the frames, clearing set reference bits, and takes the first
 * frame whose bit is clear; the hand stops one past it); the new page is
 * published referenced and clean (publish, 21-39), dirty if written.
 * The state (frame pages, bits, hand, frames in use) carries across calls
 * through `st`; or_clock_new / or_clock_free manage it. */
typedef struct or_clock {
    uint64_t frames, used, hand;
    uint64_t* page;    /* per frame */
    uint8_t* ref;
    uint8_t* dirty;
    uint64_t cap;      /* hash table: page -> frame */
    or_slot* table;
} or_clock;

void* or_clock_new(uint64_t frames)
{
    or_clock* c = (or_clock*)calloc(1, sizeof(or_clock));
    if (!c) return NULL;
    c->frames = frames;
    c->page = (uint64_t*)calloc(frames ? frames : 1, sizeof(uint64_t));
    c->ref = (uint8_t*)calloc(frames ? frames : 1, 1);
    c->dirty = (uint8_t*)calloc(frames ? frames : 1, 1);
    c->cap = 16;
    while (c->cap < frames * 2 + 16) c->cap <<= 1;
    c->table = (or_slot*)malloc(sizeof(or_slot) * c->cap);
    if (!c->page || !c->ref || !c->dirty || !c->table) return NULL;
    for (uint64_t k = 0; k < c->cap; ++k) c->table[k].node = -1;
    return c;
}

void or_clock_free(void* p)
{
    or_clock* c = (or_clock*)p;
    if (!c) return;
    free(c->page); free(c->ref); free(c->dirty); free(c->table); free(c);
}

static uint64_t or_clock_find(const or_clock* c, uint64_t page)
{
    const uint64_t mask = c->cap - 1;
    uint64_t h = or_mix(page) & mask;
    while (c->table[h].node >= 0 && c->table[h].key != page) h = (h + 1) & mask;
    return h;
}

static void or_clock_erase(or_clock* c, uint64_t page)
{
    const uint64_t mask = c->cap - 1;
    uint64_t hole = or_clock_find(c, page), probe = (hole + 1) & mask;
    c->table[hole].node = -1;
    while (c->table[probe].node >= 0) {
        const uint64_t ideal = or_mix(c->table[probe].key) & mask;
        if (((probe - ideal) & mask) >= ((probe - hole) & mask)) {
            c->table[hole] = c->table[probe];
            c->table[probe].node = -1;
            hole = probe;
        }
        probe = (probe + 1) & mask;
    }
}

void or_clock_run(void* state, const uint64_t* pages, const uint8_t* writes, uint64_t n,
                  uint8_t* hit, uint64_t* victim, uint8_t* victim_dirty)
{
    or_clock* c = (or_clock*)state;
    for (uint64_t i = 0; i < n; ++i) {
        const uint64_t p = pages[i];
        victim[i] = U64MAX;
        victim_dirty[i] = 0;
        hit[i] = 0;
        if (c->frames == 0) continue;
        uint64_t h = or_clock_find(c, p);
        if (c->table[h].node >= 0) {
            const int64_t f = c->table[h].node;
            hit[i] = 1;
            c->ref[f] = 1;
            if (writes[i]) c->dirty[f] = 1;
            continue;
        }
        uint64_t f;
        if (c->used < c->frames) {
            f = c->used++;
        } else {
            for (;;) {
                f = c->hand;
                c->hand = (c->hand + 1) % c->frames;
                if (!c->ref[f]) break;
                c->ref[f] = 0;
            }
            victim[i] = c->page[f];
            victim_dirty[i] = c->dirty[f];
            or_clock_erase(c, c->page[f]);
            h = or_clock_find(c, p);
        }
        c->page[f] = p;
        c->ref[f] = 1;
        c->dirty[f] = writes[i] ? 1 : 0;
        c->table[h].key = p;
        c->table[h].node = (int64_t)f;
    }
}

/* One media action of the capacity path through the die model. */
static uint64_t or_media_step(const or_geometry* g, const or_timing* t,
                              const uint64_t* chan_bw, const uint64_t* t_read,
                              const uint64_t* t_prog, const uint64_t* admit,
                              uint64_t media, uint32_t bytes, int op, uint64_t arrival,
                              uint64_t* state)
{
    or_decoded d;
    memset(&d, 0, sizeof d);
    or_decode_one(g, media, &d);
    const uint32_t shards = g->shard_count ? g->shard_count : 1;
    const uint32_t c = d.channel / shards;
    uint64_t* st = &state[(uint64_t)c * (g->dies_per_channel + 1)];
    const uint64_t x = or_saturating_multiply(or_channel_transfer_ns(bytes, chan_bw[c]),
                                              t->time_scale);
    const uint64_t top = op ? t_prog[d.stack] : t_read[d.stack];
    const uint64_t tt = or_saturating_multiply(top, t->time_scale);
    const uint64_t adm = admit ? admit[d.stack] : 0;
    return or_die_step(&st[0], &st[1 + d.die], arrival, adm, x, tt);
}

void or_capacity_timing(const or_geometry* g, const or_timing* t,
                        const uint64_t* chan_bw, const uint64_t* t_read,
                        const uint64_t* t_prog, const uint64_t* admit,
                        const uint8_t* status, const uint8_t* hit, const uint64_t* page,
                        const uint64_t* victim, const uint8_t* victim_dirty,
                        const uint64_t* arrival, uint64_t n, uint32_t page_shift,
                        uint64_t* state, uint64_t* done, uint64_t* latency)
{
    const uint32_t bytes = 1u << page_shift;
    for (uint64_t i = 0; i < n; ++i) {
        const uint64_t a = arrival[i];
        if (status[i] != OR_STATUS_MODELED || hit[i]) {
            done[i] = a;
            latency[i] = 0;
            continue;
        }
        uint64_t read_arrival = a;
        if (victim_dirty[i]) {
            const uint64_t p = or_media_step(g, t, chan_bw, t_read, t_prog, admit,
                                             victim[i] << page_shift, bytes, 1, a, state);
            if (p > read_arrival) read_arrival = p;
        }
        const uint64_t r = or_media_step(g, t, chan_bw, t_read, t_prog, admit,
                                         page[i] << page_shift, bytes, 0, read_arrival, state);
        done[i] = r;
        latency[i] = r - a;
    }
}

/* ---- empirical burst-curve profile ---- */

#define OR_RUN_CAP 1023u
#define OR_MAX_EMPIRICAL_PAGE ((UINT64_C(1) << 53) - 2)

/* hbf_device.cuh:959-976: ceil(delta * offset / span) as whole spans times
 * offset (saturating) plus the rounded-up share of the remainder. */
static uint64_t or_scaled_ceiling(uint64_t delta, uint32_t offset, uint32_t span)
{
    if (delta == 0 || offset == 0) return 0;
    if (span == 0) return U64MAX;
    const uint64_t whole = or_saturating_multiply(delta / span, offset);
    const uint64_t part = ((delta % span) * (uint64_t)offset + span - 1) / span;
    return or_saturating_add(whole, part);
}

/* hbf_device.cuh:978-1019: piecewise-linear cumulative time of a run; the
 * segment ending at the first breakpoint not below the run (the last one
 * past the curve), interpolated from the breakpoint before it (or 0). */
uint64_t or_empirical_cumulative_ns(const uint32_t* pages, const uint64_t* cumulative,
                                    uint32_t count, uint32_t run_pages)
{
    if (run_pages == 0) return 0;
    if (!pages || !cumulative || count == 0) return U64MAX;
    uint32_t hi = 0;
    while (hi < count && run_pages > pages[hi]) ++hi;
    if (hi == count) hi = count - 1;
    const uint32_t lo_pages = hi ? pages[hi - 1] : 0;
    const uint64_t lo_ns = hi ? cumulative[hi - 1] : 0;
    if (pages[hi] <= lo_pages || cumulative[hi] < lo_ns || run_pages < lo_pages)
        return U64MAX;
    return or_saturating_add(lo_ns, or_scaled_ceiling(cumulative[hi] - lo_ns,
                                                      run_pages - lo_pages,
                                                      pages[hi] - lo_pages));
}

/* hbf_device.cuh:1021-1032 */
uint64_t or_empirical_service_ns(const uint32_t* pages, const uint64_t* cumulative,
                                 uint32_t count, uint32_t run_pages)
{
    if (run_pages == 0) return 0;
    const uint64_t cur = or_empirical_cumulative_ns(pages, cumulative, count, run_pages);
    const uint64_t prev = or_empirical_cumulative_ns(pages, cumulative, count, run_pages - 1);
    return cur < prev ? U64MAX : cur - prev;
}

/* hbf_device.cuh:1036-1081: state = (page + 1) << 11 | op << 10 | run; the
 * run grows by one (to at most 1023) when the page follows the previous one
 * with the same operation, else restarts at 1. */
int or_update_empirical_burst(uint64_t previous, uint64_t page, uint32_t operation,
                              uint64_t* packed, uint32_t* run_pages)
{
    if (page > OR_MAX_EMPIRICAL_PAGE || operation > 1) {
        *packed = previous;
        *run_pages = 0;
        return 0;
    }
    const uint32_t prev_run = (uint32_t)(previous & OR_RUN_CAP);
    const uint32_t prev_op = (uint32_t)((previous >> 10) & 1u);
    const uint64_t prev_page_plus_one = previous >> 11;
    uint32_t run = 1;
    if (previous != 0 && prev_run != 0 && prev_op == operation &&
        prev_page_plus_one != 0 && prev_page_plus_one == page)
        run = prev_run == OR_RUN_CAP ? OR_RUN_CAP : prev_run + 1;
    *packed = ((page + 1) << 11) | ((uint64_t)operation << 10) | run;
    *run_pages = run;
    return 1;
}

/* hbf_device.cuh:1107-1128 */
int or_empirical_control_valid(const or_empirical* e)
{
    if (e->flags != 1 || e->count != 6 || e->program_latency_ns == 0) return 0;
    for (uint32_t i = 0; i < 6; ++i) {
        if (e->pages[i] == 0 || e->cumulative_ns[i] == 0) return 0;
        if (i && (e->pages[i] <= e->pages[i - 1] ||
                  e->cumulative_ns[i] <= e->cumulative_ns[i - 1]))
            return 0;
    }
    return e->pages[5] <= OR_RUN_CAP;
}

/* hbf_device.cuh:1110-1140: reads from the curve at the run length, writes
 * the header's program latency. */
int or_empirical_request_service(const or_empirical* e, uint64_t previous, uint64_t page,
                                 uint32_t operation, uint64_t* service_ns,
                                 uint64_t* packed, uint32_t* run_pages)
{
    *service_ns = 0;
    *packed = 0;
    *run_pages = 0;
    if (!or_empirical_control_valid(e)) return 0;
    uint64_t next;
    uint32_t run;
    if (!or_update_empirical_burst(previous, page, operation, &next, &run)) return 0;
    *service_ns = operation == 0
                      ? or_empirical_service_ns(e->pages, e->cumulative_ns, e->count, run)
                      : e->program_latency_ns;
    *packed = next;
    *run_pages = run;
    return 1;
}

int or_run_empirical_batch(const or_range* ranges, uint32_t count, const or_empirical* e,
                           uint32_t time_scale, uint64_t request_timeout_ns,
                           const uint64_t* address, const uint32_t* bytes,
                           const uint8_t* op, const uint64_t* arrival, uint64_t n,
                           uint64_t* state, uint64_t* done, uint64_t* latency,
                           uint8_t* status, or_stats* stats)
{
    memset(stats, 0, sizeof *stats);
    uint64_t* order = or_arrival_order(arrival, n);
    if (!order) return -1;
    const int header_ok = or_empirical_control_valid(e);
    for (uint64_t k = 0; k < n; ++k) {
        const uint64_t i = order[k];
        uint32_t index;
        uint64_t media;
        uint32_t st = or_classify(ranges, count, address[i], bytes[i], op[i], &index, &media);
        done[i] = arrival[i];
        latency[i] = 0;
        if (st == OR_STATUS_MODELED) {
            /* hbf_device.cu:773-777 and 797-801 */
            const uint64_t media_bytes = ranges[index].page_bytes;
            if (!header_ok || media_bytes != 4096 || media % media_bytes != 0 ||
                time_scale == 0 || request_timeout_ns == 0)
                st = OR_STATUS_UNSUPPORTED;
        }
        uint64_t service = 0, packed = 0;
        uint32_t run = 0;
        if (st == OR_STATUS_MODELED &&
            !or_empirical_request_service(e, state[1], media / 4096, op[i], &service,
                                          &packed, &run))
            st = OR_STATUS_UNSUPPORTED;
        status[i] = (uint8_t)st;
        if (st == OR_STATUS_BYPASS) { stats->bypass++; continue; }
        if (st != OR_STATUS_MODELED) { stats->unsupported++; continue; }
        state[1] = packed;
        const uint64_t a = arrival[i];
        const uint64_t start = state[0] > a ? state[0] : a;
        state[0] = or_saturating_add(start, or_saturating_multiply(service, time_scale));
        done[i] = state[0];
        latency[i] = state[0] - a;
        stats->modeled++;
        stats->fast_modeled_ns += service;
        stats->latency_sum = or_saturating_add(stats->latency_sum, latency[i]);
        if (state[0] > stats->max_done) stats->max_done = state[0];
    }
    free(order);
    return 0;
}

/* ---- prefetch model ---- */

/* The 64-bit Mersenne Twister of the C++ standard library (std::mt19937_64,
 * Matsumoto & Nishimura 2000; parameters from the standard's [rand.predef])
 * and the standard's generate_canonical for a double from one 64-bit draw,
 * as std::uniform_real_distribution<double>(0, 1) uses it. */
typedef struct or_mt64 {
    uint64_t x[312];
    uint32_t i;
} or_mt64;

static void or_mt64_seed(or_mt64* m, uint64_t seed)
{
    m->x[0] = seed;
    for (uint32_t k = 1; k < 312; ++k)
        m->x[k] = UINT64_C(6364136223846793005) * (m->x[k - 1] ^ (m->x[k - 1] >> 62)) + k;
    m->i = 312;
}

static uint64_t or_mt64_next(or_mt64* m)
{
    if (m->i >= 312) {
        for (uint32_t k = 0; k < 312; ++k) {
            const uint64_t y = (m->x[k] & UINT64_C(0xFFFFFFFF80000000)) |
                               (m->x[(k + 1) % 312] & UINT64_C(0x7FFFFFFF));
            m->x[k] = m->x[(k + 156) % 312] ^ (y >> 1) ^
                      ((y & 1) ? UINT64_C(0xB5026F5AA96619E9) : 0);
        }
        m->i = 0;
    }
    uint64_t y = m->x[m->i++];
    y ^= (y >> 29) & UINT64_C(0x5555555555555555);
    y ^= (y << 17) & UINT64_C(0x71D67FFFEDA60000);
    y ^= (y << 37) & UINT64_C(0xFFF7EEE000000000);
    y ^= y >> 43;
    return y;
}

static double or_canonical(or_mt64* m)
{
    const double r = (double)or_mt64_next(m) / 18446744073709551616.0;
    return r >= 1.0 ? 0x1.fffffffffffffp-1 : r;
}

/* prefetch_model.cpp:23-50: max_in_flight servers; a read issued at `now`
 * takes the server that frees first, starts at max(now, free) and ends one
 * read latency later.  A binary min-heap of free times. */
typedef struct or_heap {
    uint64_t* v;
    uint32_t n;
} or_heap;

static uint64_t or_heap_pop_push(or_heap* h, uint64_t now, uint64_t latency)
{
    const uint64_t earliest = h->v[0];
    const uint64_t done = (now > earliest ? now : earliest) + latency;
    /* replace the root with `done` and sift down */
    uint32_t k = 0;
    for (;;) {
        const uint32_t l = 2 * k + 1, r = l + 1;
        uint32_t m = k;
        uint64_t mv = done;
        if (l < h->n && h->v[l] < mv) { m = l; mv = h->v[l]; }
        if (r < h->n && h->v[r] < mv) { m = r; mv = h->v[r]; }
        if (m == k) break;
        h->v[k] = h->v[m];
        k = m;
    }
    h->v[k] = done;
    return done;
}

/* prefetch_model.cpp:52-104: pages fetched and not yet used, oldest first;
 * inserting past capacity drops the oldest. */
typedef struct or_staging {
    uint64_t* page;
    uint64_t* arrival;
    uint32_t size, capacity;
} or_staging;

static int or_staging_find(const or_staging* b, uint64_t page)
{
    for (uint32_t k = 0; k < b->size; ++k)
        if (b->page[k] == page) return (int)k;
    return -1;
}

static uint64_t or_staging_insert(or_staging* b, uint64_t page, uint64_t arrival)
{
    b->page[b->size] = page;
    b->arrival[b->size] = arrival;
    ++b->size;
    uint64_t evicted = 0;
    while (b->size > b->capacity) {
        memmove(b->page, b->page + 1, sizeof(uint64_t) * (b->size - 1));
        memmove(b->arrival, b->arrival + 1, sizeof(uint64_t) * (b->size - 1));
        --b->size;
        ++evicted;
    }
    return evicted;
}

static uint64_t or_staging_take(or_staging* b, int k)
{
    const uint64_t arrival = b->arrival[k];
    memmove(b->page + k, b->page + k + 1, sizeof(uint64_t) * (b->size - (uint32_t)k - 1));
    memmove(b->arrival + k, b->arrival + k + 1,
            sizeof(uint64_t) * (b->size - (uint32_t)k - 1));
    --b->size;
    return arrival;
}

/* prefetch_model.cpp:117-195 simulate_prefetch */
int or_prefetch_run(const uint64_t* pages, uint64_t n, const or_prefetch_cell* c,
                    or_prefetch_stats* s)
{
    memset(s, 0, sizeof *s);
    s->demand_accesses = n;
    if (n == 0) return 0;
    or_heap media;
    media.n = c->max_in_flight ? c->max_in_flight : 1;
    media.v = (uint64_t*)calloc(media.n, sizeof(uint64_t));
    or_staging buf;
    buf.capacity = c->buffer_pages ? c->buffer_pages : 1;
    buf.size = 0;
    buf.page = (uint64_t*)malloc(sizeof(uint64_t) * (buf.capacity + 1));
    buf.arrival = (uint64_t*)malloc(sizeof(uint64_t) * (buf.capacity + 1));
    or_mt64* rng = (or_mt64*)malloc(sizeof(or_mt64));
    if (!media.v || !buf.page || !buf.arrival || !rng) {
        free(media.v); free(buf.page); free(buf.arrival); free(rng);
        return -1;
    }
    or_mt64_seed(rng, c->seed);
    uint64_t clock = 0;
    uint64_t wrong = UINT64_C(1) << 60;
    for (uint64_t i = 0; i < n; ++i) {
        clock += c->compute_ns_per_access;
        if (c->policy != 0 && c->lead_distance > 0) {
            const uint64_t target = i + c->lead_distance;
            int predict = 0;
            uint64_t predicted = 0;
            if (c->policy == 1) {
                predicted = pages[i] + 1;
                predict = 1;
            } else if (target < n) {
                predicted = or_canonical(rng) < c->accuracy ? pages[target] : wrong++;
                predict = 1;
            }
            if (predict && or_staging_find(&buf, predicted) < 0) {
                const uint64_t arrival = or_heap_pop_push(&media, clock, c->read_latency_ns);
                s->prefetch_wasted += or_staging_insert(&buf, predicted, arrival);
                ++s->prefetch_issued;
            }
        }
        const int k = or_staging_find(&buf, pages[i]);
        if (k >= 0) {
            const uint64_t arrival = or_staging_take(&buf, k);
            ++s->prefetch_hits;
            if (arrival > clock) {
                s->stall_ns += arrival - clock;
                clock = arrival;
            }
        } else {
            const uint64_t arrival = or_heap_pop_push(&media, clock, c->read_latency_ns);
            ++s->demand_misses;
            s->stall_ns += arrival - clock;
            clock = arrival;
        }
    }
    s->prefetch_wasted += buf.size;
    s->total_ns = clock;
    free(media.v); free(buf.page); free(buf.arrival); free(rng);
    return 0;
}

/* ---- UCIe streaming link ---- */

enum { OR_EV_ARRIVAL, OR_EV_FLIT, OR_EV_CONSUME, OR_EV_RETRY };

typedef struct or_event {
    uint64_t t;
    uint64_t seq;      /* insertion order: equal times run in it (std::multimap) */
    uint64_t id;
    uint32_t kind, dir;
    uint32_t count;    /* flit: messages it completes */
    uint32_t grant;    /* flit: credit granules it returns */
} or_event;

typedef struct or_msg {
    uint64_t id;
    uint32_t remaining, emitted, started;
} or_msg;

typedef struct or_link {
    const or_link_profile* p;
    or_event* heap;
    uint64_t heap_n, heap_cap, seq;
    or_msg* queue[2];             /* rings of max_accepted: waiting to be sent */
    uint64_t q_head[2], q_size[2];
    uint64_t* sent[2];            /* rings: completed, waiting for delivery */
    uint64_t s_head[2], s_size[2];
    uint64_t now, cursor[2];
    uint32_t credits[2];          /* 0 AR credits, 1 R credits */
    uint32_t grant_pending[2];    /* 0 AR granules to return, 1 R granules */
    uint64_t active[2];
    int retry_pending[2];
    uint64_t counters[2][8];
    uint64_t flit_ns;
    uint64_t heap_peak;
    int error;
} or_link;

static int or_ev_less(const or_event* a, const or_event* b)
{
    return a->t < b->t || (a->t == b->t && a->seq < b->seq);
}

static void or_ev_push(or_link* L, or_event e)
{
    if (L->heap_n == L->heap_cap) {
        const uint64_t cap = L->heap_cap ? 2 * L->heap_cap : 64;
        or_event* h = (or_event*)realloc(L->heap, sizeof(or_event) * cap);
        if (!h) { L->error = 1; return; }
        L->heap = h;
        L->heap_cap = cap;
    }
    e.seq = L->seq++;
    uint64_t k = L->heap_n++;
    if (L->heap_n > L->heap_peak) L->heap_peak = L->heap_n;
    while (k > 0) {
        const uint64_t up = (k - 1) / 2;
        if (!or_ev_less(&e, &L->heap[up])) break;
        L->heap[k] = L->heap[up];
        k = up;
    }
    L->heap[k] = e;
}

static or_event or_ev_pop(or_link* L)
{
    const or_event top = L->heap[0];
    const or_event last = L->heap[--L->heap_n];
    uint64_t k = 0;
    for (;;) {
        const uint64_t l = 2 * k + 1, r = l + 1;
        uint64_t m = k;
        const or_event* mv = &last;
        if (l < L->heap_n && or_ev_less(&L->heap[l], mv)) { m = l; mv = &L->heap[l]; }
        if (r < L->heap_n && or_ev_less(&L->heap[r], mv)) { m = r; mv = &L->heap[r]; }
        if (m == k) break;
        L->heap[k] = L->heap[m];
        k = m;
    }
    if (L->heap_n) L->heap[k] = last;
    return top;
}

static uint64_t or_add_time(or_link* L, uint64_t a, uint64_t b)
{
    if (a > UINT64_MAX - b) { L->error = 1; return UINT64_MAX; }
    return a + b;
}

/* link.cpp:111-117 legal_grant: AoU grants are 1, 4, 8, ..., 128 granules */
static uint32_t or_legal_grant(uint32_t pending)
{
    if (pending == 0) return 0;
    if (pending < 4) return 1;
    uint32_t grant = 4;
    while (grant < 128 && grant * 2 <= pending) grant *= 2;
    return grant;
}

static void or_retry(or_link* L, uint32_t d)
{
    /* the pending retry of a direction is always at its cursor: a second one
     * at the same tick would run in the same step and change nothing */
    if (L->retry_pending[d]) return;
    L->retry_pending[d] = 1;
    or_event e = {L->cursor[d], 0, 0, OR_EV_RETRY, d, 0, 0};
    or_ev_push(L, e);
}

/* link.cpp:119-179 send_ready */
static void or_send_ready(or_link* L, uint32_t d)
{
    uint32_t* credit = &L->credits[d];
    uint32_t* pending = &L->grant_pending[1 - d];  /* reverse direction's granules */
    if (L->cursor[d] > L->now) {
        if (L->q_size[d] || *pending) or_retry(L, d);
        return;
    }
    const uint64_t cap = L->p->max_accepted;
    uint32_t used = 0, completed = 0;
    while (L->q_size[d] && used < 48) {
        or_msg* msg = &L->queue[d][L->q_head[d]];
        if (!msg->started) {
            const uint32_t full = d == 0 ? 3u : 14u;
            if (*credit < full) break;
            *credit -= full;   /* every granule is reserved at MsgStart */
            msg->started = 1;
        }
        const uint32_t fragment = 48 - used < msg->remaining ? 48 - used : msg->remaining;
        used += fragment;
        msg->remaining -= fragment;
        msg->emitted += fragment;
        if (msg->remaining == 0) {
            L->sent[d][(L->s_head[d] + L->s_size[d]) % cap] = msg->id;
            ++L->s_size[d];
            L->q_head[d] = (L->q_head[d] + 1) % cap;
            --L->q_size[d];
            ++completed;
        }
    }
    const uint32_t grant = or_legal_grant(*pending);
    if (used == 0 && grant == 0) return;
    *pending -= grant;
    L->cursor[d] = or_add_time(L, L->now, L->flit_ns);
    const uint64_t delivery = or_add_time(L, L->cursor[d], L->p->propagation_ns);
    or_event e = {delivery, 0, 0, OR_EV_FLIT, d, completed, grant};
    or_ev_push(L, e);
    if (L->q_size[d] || *pending) or_retry(L, d);
    uint64_t* c = L->counters[d];
    c[0] += 1;
    c[1] += 256;
    c[2] += 2;
    c[3] += 4;
    c[4] += 10;
    c[5] += (uint64_t)used * 5;
    c[6] += (uint64_t)(48 - used) * 5;
    if (used == 0) c[7] += 1;
}

int or_link_run(const or_link_profile* p, const uint8_t* direction, const uint64_t* ready,
                uint64_t m, uint64_t* delivered, or_link_result* out)
{
    or_link L;
    memset(&L, 0, sizeof L);
    memset(out, 0, sizeof *out);
    L.p = p;
    L.flit_ns = 32 / p->gt_per_second;   /* profile.cpp:63-67: 256 B at x64 */
    L.credits[0] = p->initial_ar_granules;
    L.credits[1] = p->initial_r_granules;
    const uint64_t cap = p->max_accepted ? p->max_accepted : 1;
    for (int d = 0; d < 2; ++d) {
        L.queue[d] = (or_msg*)calloc(cap, sizeof(or_msg));
        L.sent[d] = (uint64_t*)calloc(cap, sizeof(uint64_t));
    }
    /* deliveries of one step: (direction, id), consumed after the step */
    uint64_t* step_id = (uint64_t*)malloc(sizeof(uint64_t) * 2 * cap);
    uint32_t* step_dir = (uint32_t*)malloc(sizeof(uint32_t) * 2 * cap);
    if (!L.queue[0] || !L.queue[1] || !L.sent[0] || !L.sent[1] || !step_id || !step_dir)
        L.error = 1;
    uint64_t next = 0;
    while (!L.error) {
        uint64_t t_event = L.heap_n ? L.heap[0].t : UINT64_MAX;
        while (next < m) {
            const uint32_t d = direction[next];
            const uint64_t at = ready[next] > L.now ? ready[next] : L.now;
            if (L.active[d] >= p->max_accepted || at > t_event) break;
            or_event e = {at, 0, next + 1, OR_EV_ARRIVAL, d, 0, 0};   /* link.cpp:42-54 */
            or_ev_push(&L, e);
            ++L.active[d];
            ++next;
            if (at < t_event) t_event = at;
        }
        if (L.heap_n == 0) break;
        /* link.cpp:181-227 step: every event at the earliest tick, in
         * insertion order, then one send attempt per direction */
        L.now = L.heap[0].t;
        uint64_t n_step = 0;
        while (L.heap_n && L.heap[0].t == L.now && !L.error) {
            const or_event e = or_ev_pop(&L);
            if (e.kind == OR_EV_ARRIVAL) {
                or_msg* msg = &L.queue[e.dir][(L.q_head[e.dir] + L.q_size[e.dir]) % cap];
                msg->id = e.id;
                msg->remaining = e.dir == 0 ? 3u : 14u;
                msg->emitted = 0;
                msg->started = 0;
                ++L.q_size[e.dir];
            } else if (e.kind == OR_EV_FLIT) {
                const uint32_t back = 1 - e.dir;   /* the grant returns the reverse credits */
                const uint32_t maximum = back == 0 ? p->initial_ar_granules : p->initial_r_granules;
                if (e.grant > maximum - L.credits[back]) { L.error = 1; break; }
                L.credits[back] += e.grant;
                for (uint32_t k = 0; k < e.count; ++k) {
                    const uint64_t id = L.sent[e.dir][L.s_head[e.dir]];
                    L.s_head[e.dir] = (L.s_head[e.dir] + 1) % cap;
                    --L.s_size[e.dir];
                    delivered[id - 1] = L.now;
                    step_id[n_step] = id;
                    step_dir[n_step] = e.dir;
                    ++n_step;
                }
            } else if (e.kind == OR_EV_CONSUME) {
                --L.active[e.dir];
                uint32_t* pending = &L.grant_pending[e.dir];
                const uint32_t amount = e.dir == 0 ? 3u : 14u;
                if (*pending > 65535u - amount) { L.error = 1; break; }
                *pending += amount;
            } else {
                L.retry_pending[e.dir] = 0;
            }
        }
        if (L.error) break;
        or_send_ready(&L, 0);
        or_send_ready(&L, 1);
        /* the driver consumes every delivery consume_ns after it (link.cpp:56-65) */
        for (uint64_t k = 0; k < n_step; ++k) {
            or_event e = {or_add_time(&L, L.now, p->consume_ns[step_dir[k]]), 0, step_id[k],
                          OR_EV_CONSUME, step_dir[k], 0, 0};
            or_ev_push(&L, e);
        }
    }
    out->now = L.now;
    out->ar_credits = L.credits[0];
    out->r_credits = L.credits[1];
    out->heap_peak = L.heap_peak;
    memcpy(out->counters, L.counters, sizeof L.counters);
    free(L.heap);
    for (int d = 0; d < 2; ++d) { free(L.queue[d]); free(L.sent[d]); }
    free(step_id);
    free(step_dir);
    return L.error ? -1 : 0;
}
