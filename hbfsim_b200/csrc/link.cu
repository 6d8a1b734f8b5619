// link.cu -- UCIe streaming-link timing for batches of links, one thread per
// link.
//
// Reference: hbfsim::ucie::StreamingLink (src/ucie/link.cpp,
// include/hbfsim/ucie/link.hpp:54-113): Format 6 flits of 256 wire bytes carry
// 48 AoU granules of messages (a read request AR takes 3, a read return R 14);
// a message reserves all its credits when its first granule is sent; a flit
// leaves every 32/GT ns and lands after the propagation delay; a consumed
// message's granules go back to the sender as legal grants (1, 4, 8 ... 128)
// on the reverse direction's next flit, credit-only if it has no data.
//
// The link is an event walk.  Events at one tick run in the order they were
// scheduled (the reference's std::multimap), then each direction tries one
// flit.  This build walks each link on one thread with its own event heap
// keyed by (tick, scheduling number), message rings and sent rings in
// global scratch sized from the link's credit and acceptance limits; a batch
// of independent links (stacks, modules, sweep cells) runs in parallel.
//
// Batch driver (the same as the oracle's): messages of a link are offered in
// input order; the next one is scheduled at max(its ready tick, the link's
// tick) once its direction has fewer than max_accepted messages in flight
// and its ready tick is not past the link's next event; after each step,
// every delivered message is consumed consume_ns[direction] later.
#include "../../include/hbfsim/batch_v1.h"
#include "common.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

namespace hbfb {
namespace {

enum EventKind : u32 { kArrival = 0, kFlit = 1, kConsume = 2, kRetry = 3 };

struct Event {
    u64 t;
    u64 seq;     // scheduling number: equal ticks run in scheduling order
    u64 id;
    u32 meta;    // kind | dir << 2 | count << 3 | grant << 8
    u32 pad;
};

struct Msg {
    u64 id;
    u32 remaining, started;
};

struct LinkScratch {     // per link, in global memory
    Event* heap;
    Msg* queue[2];
    u64* sent[2];
    u64* step_id;
    u32* step_dir;
    u64 heap_cap;
    u64 cap;             // max_accepted
};

struct LinkArgs {
    const hbfsim_link_profile_v1* profiles;
    const u64* offsets;          // links + 1
    const u8* direction;
    const u64* ready;
    u64* delivered;
    hbfsim_link_result_v1* results;
    unsigned char* scratch;
    const u64* scratch_offset;   // per link, bytes
    u32 links;
};

__device__ __forceinline__ bool ev_less(const Event& a, const Event& b)
{
    return a.t < b.t || (a.t == b.t && a.seq < b.seq);
}

struct Walk {
    const hbfsim_link_profile_v1* p;
    LinkScratch s;
    u64 heap_n = 0, seq = 0;
    u64 q_head[2] = {0, 0}, q_size[2] = {0, 0};
    u64 s_head[2] = {0, 0}, s_size[2] = {0, 0};
    u64 now = 0, cursor[2] = {0, 0};
    u32 credits[2] = {0, 0};        // 0 AR credits, 1 R credits
    u32 grant_pending[2] = {0, 0};  // granules to give back: 0 AR, 1 R
    u64 active[2] = {0, 0};
    bool retry_pending[2] = {false, false};
    u64 counters[2][8] = {};
    u64 flit_ns = 2;
    int error = 0;

    __device__ void push(Event e)
    {
        if (heap_n >= s.heap_cap) {
            error = HBFSIM_UNSUPPORTED;  // beyond the derived bound: stop this link
            return;
        }
        e.seq = seq++;
        u64 k = heap_n++;
        while (k > 0) {
            const u64 up = (k - 1) / 2;
            if (!ev_less(e, s.heap[up])) break;
            s.heap[k] = s.heap[up];
            k = up;
        }
        s.heap[k] = e;
    }

    __device__ Event pop()
    {
        const Event top = s.heap[0];
        const Event last = s.heap[--heap_n];
        u64 k = 0;
        for (;;) {
            const u64 l = 2 * k + 1, r = l + 1;
            u64 m = k;
            Event mv = last;
            if (l < heap_n && ev_less(s.heap[l], mv)) {
                m = l;
                mv = s.heap[l];
            }
            if (r < heap_n && ev_less(s.heap[r], mv)) m = r;
            if (m == k) break;
            s.heap[k] = s.heap[m];
            k = m;
        }
        if (heap_n) s.heap[k] = last;
        return top;
    }

    __device__ u64 add_time(u64 a, u64 b)
    {
        if (a > ~u64{0} - b) {
            error = HBFSIM_INVALID_ARGUMENT;  // link.cpp:8-13 overflow_error
            return ~u64{0};
        }
        return a + b;
    }

    __device__ void retry(u32 d)
    {
        // a direction's pending retry is always at its cursor; a second one at
        // the same tick would run in the same step and change nothing
        if (retry_pending[d]) return;
        retry_pending[d] = true;
        push(Event{cursor[d], 0, 0, kRetry | (d << 2), 0});
    }

    // link.cpp:111-117
    static __device__ u32 legal_grant(u32 pending)
    {
        if (pending == 0) return 0;
        if (pending < 4) return 1;
        u32 grant = 4;
        while (grant < 128 && grant * 2 <= pending) grant *= 2;
        return grant;
    }

    // link.cpp:119-179
    __device__ void send_ready(u32 d)
    {
        u32& credit = credits[d];
        u32& pending = grant_pending[1 - d];   // the reverse direction's granules
        if (cursor[d] > now) {
            if (q_size[d] || pending) retry(d);
            return;
        }
        u32 used = 0, completed = 0;
        while (q_size[d] && used < 48) {
            Msg& msg = s.queue[d][q_head[d]];
            if (!msg.started) {
                const u32 full = d == 0 ? 3u : 14u;
                if (credit < full) break;
                credit -= full;
                msg.started = 1;
            }
            const u32 fragment = 48 - used < msg.remaining ? 48 - used : msg.remaining;
            used += fragment;
            msg.remaining -= fragment;
            if (msg.remaining == 0) {
                s.sent[d][(s_head[d] + s_size[d]) % s.cap] = msg.id;
                ++s_size[d];
                q_head[d] = (q_head[d] + 1) % s.cap;
                --q_size[d];
                ++completed;
            }
        }
        const u32 grant = legal_grant(pending);
        if (used == 0 && grant == 0) return;
        pending -= grant;
        cursor[d] = add_time(now, flit_ns);
        const u64 delivery = add_time(cursor[d], p->propagation_ns);
        push(Event{delivery, 0, 0, kFlit | (d << 2) | (completed << 3) | (grant << 8), 0});
        if (q_size[d] || pending) retry(d);
        u64* c = counters[d];
        c[0] += 1;
        c[1] += 256;
        c[2] += 2;
        c[3] += 4;
        c[4] += 10;
        c[5] += static_cast<u64>(used) * 5;
        c[6] += static_cast<u64>(48 - used) * 5;
        if (used == 0) c[7] += 1;
    }
};

__global__ void __launch_bounds__(128) link_kernel(const LinkArgs a)
{
    const u32 k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= a.links) return;
    const hbfsim_link_profile_v1& p = a.profiles[k];
    Walk w;
    w.p = &p;
    {
        unsigned char* base = a.scratch + a.scratch_offset[k];
        const u64 cap = p.max_accepted;
        const u64 heap_cap = 21 * cap + p.initial_ar_granules + p.initial_r_granules + 8;
        w.s.heap = reinterpret_cast<Event*>(base);
        base += sizeof(Event) * heap_cap;
        for (int d = 0; d < 2; ++d) {
            w.s.queue[d] = reinterpret_cast<Msg*>(base);
            base += sizeof(Msg) * cap;
        }
        for (int d = 0; d < 2; ++d) {
            w.s.sent[d] = reinterpret_cast<u64*>(base);
            base += 8 * cap;
        }
        w.s.step_id = reinterpret_cast<u64*>(base);
        base += 16 * cap;
        w.s.step_dir = reinterpret_cast<u32*>(base);
        w.s.heap_cap = heap_cap;
        w.s.cap = cap;
    }
    w.flit_ns = 32 / p.gt_per_second;   // profile.cpp:63-67
    w.credits[0] = p.initial_ar_granules;
    w.credits[1] = p.initial_r_granules;
    const u64 first = a.offsets[k], m = a.offsets[k + 1] - first;
    const u8* dir = a.direction + first;
    const u64* ready = a.ready + first;
    u64* delivered = a.delivered + first;
    u64 next = 0, last_ready = 0;
    while (!w.error) {
        u64 t_event = w.heap_n ? w.s.heap[0].t : ~u64{0};
        while (next < m) {
            const u32 d = dir[next] ? 1u : 0u;
            const u64 r = ready[next];
            if (r < last_ready) {  // the batch must be in ready order
                w.error = HBFSIM_INVALID_ARGUMENT;
                break;
            }
            const u64 at = r > w.now ? r : w.now;
            if (w.active[d] >= p.max_accepted || at > t_event) break;
            w.push(Event{at, 0, next + 1, kArrival | (d << 2), 0});   // link.cpp:42-54
            ++w.active[d];
            last_ready = r;
            ++next;
            if (at < t_event) t_event = at;
        }
        if (w.error || w.heap_n == 0) break;
        // link.cpp:181-227 step
        w.now = w.s.heap[0].t;
        u64 n_step = 0;
        while (w.heap_n && w.s.heap[0].t == w.now && !w.error) {
            const Event e = w.pop();
            const u32 kind = e.meta & 3u, d = (e.meta >> 2) & 1u;
            if (kind == kArrival) {
                Msg& msg = w.s.queue[d][(w.q_head[d] + w.q_size[d]) % w.s.cap];
                msg.id = e.id;
                msg.remaining = d == 0 ? 3u : 14u;
                msg.started = 0;
                ++w.q_size[d];
            } else if (kind == kFlit) {
                const u32 count = (e.meta >> 3) & 31u, grant = e.meta >> 8;
                const u32 back = 1 - d;   // the grant returns the reverse credits
                const u32 maximum = back == 0 ? p.initial_ar_granules : p.initial_r_granules;
                if (grant > maximum - w.credits[back]) {
                    w.error = HBFSIM_INVALID_ARGUMENT;  // link.cpp:197-200 logic_error
                    break;
                }
                w.credits[back] += grant;
                for (u32 c = 0; c < count; ++c) {
                    const u64 id = w.s.sent[d][w.s_head[d]];
                    w.s_head[d] = (w.s_head[d] + 1) % w.s.cap;
                    --w.s_size[d];
                    delivered[id - 1] = w.now;
                    w.s.step_id[n_step] = id;
                    w.s.step_dir[n_step] = d;
                    ++n_step;
                }
            } else if (kind == kConsume) {
                --w.active[d];
                const u32 amount = d == 0 ? 3u : 14u;
                if (w.grant_pending[d] > 65535u - amount) {
                    w.error = HBFSIM_INVALID_ARGUMENT;  // link.cpp:214-216
                    break;
                }
                w.grant_pending[d] += amount;
            } else {
                w.retry_pending[d] = false;
            }
        }
        if (w.error) break;
        w.send_ready(0);
        w.send_ready(1);
        for (u64 c = 0; c < n_step; ++c) {  // the driver consumes each delivery
            const u32 d = w.s.step_dir[c];
            w.push(Event{w.add_time(w.now, p.consume_ns[d]), 0, w.s.step_id[c],
                         kConsume | (d << 2), 0});
        }
    }
    hbfsim_link_result_v1 res{};
    for (int d = 0; d < 2; ++d)
        for (int c = 0; c < 8; ++c) res.counters[d][c] = w.counters[d][c];
    res.now = w.now;
    res.ar_credits = w.credits[0];
    res.r_credits = w.credits[1];
    res.status = w.error;
    a.results[k] = res;
}

std::uint64_t heap_capacity(const hbfsim_link_profile_v1& p)
{
    // arrivals and consumes in flight (2 x 2 x max_accepted), flits with data
    // (at most the granules of the messages in flight, 17 x max_accepted),
    // credit-only flits (at most one granule of credit each) and two retries
    return 21ull * p.max_accepted + p.initial_ar_granules + p.initial_r_granules + 8;
}

std::uint64_t scratch_bytes(const hbfsim_link_profile_v1& p)
{
    const std::uint64_t cap = p.max_accepted;
    const std::uint64_t bytes = sizeof(Event) * heap_capacity(p) + 2 * sizeof(Msg) * cap +
                                2 * 8 * cap + 16 * cap + 8 * cap;
    return (bytes + 255) / 256 * 256;
}

}  // namespace
}  // namespace hbfb

using namespace hbfb;

extern "C" int hbfsim_link_batch_v1(const hbfsim_link_profile_v1* profiles, uint32_t links,
                                    const uint64_t* offsets, const uint8_t* direction,
                                    const uint64_t* ready, uint64_t* delivered,
                                    hbfsim_link_result_v1* results, void* stream)
{
    if (links == 0) return HBFSIM_OK;
    if (!profiles || !offsets || !results) return HBFSIM_INVALID_ARGUMENT;
    const std::uint64_t total = offsets[links];
    if (offsets[0] != 0 || (total && (!direction || !ready || !delivered)))
        return HBFSIM_INVALID_ARGUMENT;
    std::vector<std::uint64_t> scratch_offset(links);
    std::uint64_t scratch = 0;
    for (uint32_t k = 0; k < links; ++k) {
        const auto& p = profiles[k];
        // profile.cpp:40-61 validate_link_profile (the scenario fields)
        if ((p.gt_per_second != 8 && p.gt_per_second != 16 && p.gt_per_second != 32) ||
            p.initial_ar_granules < 3 || p.initial_r_granules < 14 ||
            p.initial_ar_granules > 65535 || p.initial_r_granules > 65535 ||
            p.max_accepted == 0 || p.max_accepted > 65535 ||
            p.propagation_ns > 1'000'000'000ull || offsets[k + 1] < offsets[k])
            return HBFSIM_INVALID_ARGUMENT;
        scratch_offset[k] = scratch;
        scratch += scratch_bytes(p);
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    hbfsim_link_profile_v1* d_prof = nullptr;
    hbfsim_link_result_v1* d_res = nullptr;
    std::uint64_t *d_offsets = nullptr, *d_soff = nullptr;
    unsigned char* d_scratch = nullptr;
    int rc = HBFSIM_CUDA_ERROR;
    if (cudaMalloc(&d_prof, sizeof(hbfsim_link_profile_v1) * links) == cudaSuccess &&
        cudaMalloc(&d_res, sizeof(hbfsim_link_result_v1) * links) == cudaSuccess &&
        cudaMalloc(&d_offsets, 8ull * (links + 1)) == cudaSuccess &&
        cudaMalloc(&d_soff, 8ull * links) == cudaSuccess &&
        cudaMalloc(&d_scratch, scratch) == cudaSuccess &&
        cudaMemcpyAsync(d_prof, profiles, sizeof(hbfsim_link_profile_v1) * links,
                        cudaMemcpyHostToDevice, s) == cudaSuccess &&
        cudaMemcpyAsync(d_offsets, offsets, 8ull * (links + 1), cudaMemcpyHostToDevice, s) ==
            cudaSuccess &&
        cudaMemcpyAsync(d_soff, scratch_offset.data(), 8ull * links, cudaMemcpyHostToDevice,
                        s) == cudaSuccess &&
        (total == 0 || cudaMemsetAsync(delivered, 0, 8 * total, s) == cudaSuccess)) {
        LinkArgs a{};
        a.profiles = d_prof;
        a.offsets = d_offsets;
        a.direction = direction;
        a.ready = ready;
        a.delivered = delivered;
        a.results = d_res;
        a.scratch = d_scratch;
        a.scratch_offset = d_soff;
        a.links = links;
        link_kernel<<<(links + 127) / 128, 128, 0, s>>>(a);
        if (cudaGetLastError() == cudaSuccess &&
            cudaMemcpyAsync(results, d_res, sizeof(hbfsim_link_result_v1) * links,
                            cudaMemcpyDeviceToHost, s) == cudaSuccess &&
            cudaStreamSynchronize(s) == cudaSuccess)
            rc = HBFSIM_OK;
    }
    cudaFree(d_prof);
    cudaFree(d_res);
    cudaFree(d_offsets);
    cudaFree(d_soff);
    cudaFree(d_scratch);
    return rc;
}
