// ref_link.cpp -- drives the REFERENCE UCIe streaming link on message batches.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this driver with the
// reference's src/ucie/link.cpp and src/ucie/profile.cpp where they lie in the
// HBFSim tree; the binary lands in oracle/_ref/.  tests/golden/make_goldens.py
// runs it to produce tests/golden/link_goldens.json.
//
// The batch driver (the same rules as or_link_run in hbf_oracle.c and the
// device kernel): messages are offered in input order; the next one is
// enqueued, at max(its ready time, the link's time), once its direction has
// fewer than max_accepted messages in flight and its ready time is not past
// the link's next event; then the link steps, and every delivered message is
// consumed consume_ns[direction] after its delivery.  A direction's count of
// messages in flight drops once the step that processes the consume has run.
//
// Input (text): gt initial_ar initial_r max_accepted propagation consume_req
//               consume_ret M, then M lines "direction ready_ns".
// Output: M delivery ticks, one per line; then per direction the counters
//         flits wire ucie_header crc aou_header aou_message unused credit_only;
//         then ar_credits r_credits now.
#include <hbfsim/ucie/link.hpp>

#include <cinttypes>
#include <cstdio>
#include <limits>
#include <vector>

using hbfsim::ucie::Direction;

int main()
{
    unsigned gt = 0, ar = 0, r = 0, accepted = 0;
    unsigned long long prop = 0, consume[2] = {0, 0}, m = 0;
    if (std::scanf("%u %u %u %u %llu %llu %llu %llu", &gt, &ar, &r, &accepted, &prop, &consume[0],
                   &consume[1], &m) != 8)
        return 2;
    std::vector<unsigned> dir(m);
    std::vector<std::uint64_t> ready(m), delivered(m, 0);
    for (std::uint64_t k = 0; k < m; ++k) {
        unsigned long long t = 0;
        if (std::scanf("%u %llu", &dir[k], &t) != 2) return 2;
        ready[k] = t;
    }
    hbfsim::ucie::LinkProfile p;
    p.name = "batch";
    p.gt_per_second = gt;
    p.local_capacity_bytes = 16ULL << 30;
    p.initial_ar_granules = ar;
    p.initial_r_granules = r;
    p.max_accepted = accepted;
    p.propagation_ns = prop;
    hbfsim::ucie::StreamingLink link(p);
    std::uint64_t next = 0;
    std::uint64_t active[2] = {0, 0};
    // consumes scheduled but not yet processed: (tick, direction)
    std::vector<std::pair<std::uint64_t, unsigned>> pending;
    constexpr auto kNone = std::numeric_limits<std::uint64_t>::max();
    for (;;) {
        std::uint64_t t_event = link.next_event_ns() ? *link.next_event_ns() : kNone;
        while (next < m) {
            const unsigned d = dir[next];
            const std::uint64_t at = ready[next] > link.current_time_ns() ? ready[next]
                                                                           : link.current_time_ns();
            if (active[d] >= accepted || at > t_event) break;
            link.enqueue(d == 0 ? Direction::Request : Direction::Return, next + 1, at);
            ++active[d];
            ++next;
            if (at < t_event) t_event = at;
        }
        if (!link.next_event_ns()) break;
        const auto deliveries = link.step();
        // consumes scheduled before this step at or before its time were
        // processed by it: their messages have left the link
        std::vector<std::pair<std::uint64_t, unsigned>> keep;
        for (const auto& [at, d] : pending) {
            if (at <= link.current_time_ns()) --active[d];
            else keep.emplace_back(at, d);
        }
        pending.swap(keep);
        for (const auto& dv : deliveries) {
            const unsigned d = dv.direction == Direction::Request ? 0u : 1u;
            delivered[dv.request_id - 1] = dv.delivered_ns;
            const auto at = dv.delivered_ns + consume[d];
            link.consume(dv.direction, dv.request_id, at);
            pending.emplace_back(at, d);
        }
    }
    for (std::uint64_t k = 0; k < m; ++k) std::printf("%" PRIu64 "\n", delivered[k]);
    for (auto d : {Direction::Request, Direction::Return}) {
        const auto& c = link.counters(d);
        std::printf("%" PRIu64 " %" PRIu64 " %" PRIu64 " %" PRIu64 " %" PRIu64 " %" PRIu64 " %" PRIu64
                    " %" PRIu64 "\n",
                    c.flits, c.wire_bytes, c.ucie_header_bytes, c.crc_position_bytes,
                    c.aou_header_bytes, c.aou_message_bytes, c.unused_message_bytes,
                    c.credit_only_flits);
    }
    std::printf("%u %u %" PRIu64 "\n", link.credits(Direction::Request),
                link.credits(Direction::Return), link.current_time_ns());
    return 0;
}
