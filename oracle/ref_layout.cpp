// ref_layout.cpp -- drives the REFERENCE stripe-decode functions of the UCIe
// stack path, to pin this build's address decode (A2).
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this driver with the
// reference's src/ucie/bank_layout.cpp, src/ucie/stack_router.cpp and
// src/profile/profile.cpp where they lie in the HBFSim tree; the binary lands
// in oracle/_ref/.  tests/golden/make_goldens.py runs it to produce
// tests/golden/layout_goldens.json.
//
// Two levels, each at its own granularity:
//
//   bank   hbf_cold_read_bank (bank_layout.cpp:59-72): a module's 4 KiB media
//          LPA -> host channel, core die, bank.  Output lines
//          "bank <host_channels> <ncdu> <banks> <lpa> <channel> <die> <bank>".
//   stripe page-striped placement (stack_router.cpp:160-250): a 16 KiB page
//          p of a striped parent goes to channel c = (p + phase) % 64, whose
//          packed segment lives in stack c % 4, module c / 4.  The driver
//          registers one parent through GlobalSpanRegistry::add_page_striped
//          (which checks every segment's stack and module with
//          ContiguousStackMap::locate), places page p at
//          segment_base(c) + (p / 64) * 16 KiB + within, checks that
//          inverse_page_striped returns the logical offset, and prints
//          what locate says of that physical address.  Output lines
//          "stripe <phase> <logical offset> <stack> <module> <module-local address>".
#include <hbfsim/ucie/bank_layout.hpp>
#include <hbfsim/ucie/stack_router.hpp>

#include <cinttypes>
#include <cstdio>
#include <random>
#include <string>

using namespace hbfsim::ucie;

static int bank_cases(std::mt19937_64& rng)
{
    const unsigned ncdus[] = {1, 2, 4, 8, 16};
    const unsigned banks[] = {1, 2, 4, 8, 16};
    const unsigned channels[] = {16, 8, 4};
    for (unsigned hc : channels)
        for (unsigned nd : ncdus)
            for (unsigned nb : banks) {
                HbfBankLayout layout{};
                layout.host_channels = hc;
                layout.core_dies_per_channel = nd;
                layout.banks_per_die = nb;
                layout.scenario_assumption = hc != 16 || nb != 16;
                for (int k = 0; k < 40; ++k) {
                    // small LPAs (every digit pattern) and large ones
                    const std::uint64_t lpa = k < 24 ? static_cast<std::uint64_t>(k) * 37u + k
                                                     : rng() >> (k % 3 == 0 ? 34 : 42);
                    const HbfReadBank b = hbf_cold_read_bank(lpa, layout);
                    std::printf("bank %u %u %u %" PRIu64 " %u %u %u\n", hc, nd, nb, lpa,
                                b.host_channel, b.core_die, b.bank);
                }
                // the module-local page -> LPA step of the same layout
                for (int k = 0; k < 4; ++k) {
                    const std::uint64_t q = rng() >> 40;
                    const std::uint32_t module = static_cast<std::uint32_t>(rng() % hc);
                    const std::uint64_t lpa = hbf_media_lpa(q, module, layout);
                    const HbfReadBank b = hbf_cold_read_bank(lpa, layout);
                    std::printf("bank %u %u %u %" PRIu64 " %u %u %u\n", hc, nd, nb, lpa,
                                b.host_channel, b.core_die, b.bank);
                }
            }
    return 0;
}

static int stripe_cases(std::mt19937_64& rng, std::uint32_t phase)
{
    constexpr std::uint64_t page = 16384, modules = 16, stacks = 4;
    constexpr std::uint64_t module_bytes = 64ull << 20;
    constexpr std::uint64_t pages = 64 * 1024 + 37;  // a ragged last round
    const ContiguousStackMap map(module_bytes * modules * stacks, stacks, modules);
    GlobalSpanRegistry registry(map);
    PageStripeBacking s{};
    s.parent.region_id = 1;
    s.parent.address = 1ull << 40;
    s.parent.bytes = pages * page;
    s.parent.canonical_id = 7;
    s.parent.generation = 1;
    s.parent.endpoint_id = 3;
    s.parent.readable = true;
    s.actual_storage_bytes = pages * page;
    s.page_bytes = page;
    s.phase = phase;
    s.descriptor_sha256 = std::string(64, 'a');
    std::uint64_t base[64];
    for (std::uint32_t c = 0; c < 64; ++c) {
        const std::uint64_t p0 = (c + 64 - phase) % 64;
        const std::uint64_t count = p0 < pages ? 1 + (pages - 1 - p0) / 64 : 0;
        // each channel's packed segment at the start of its module
        base[c] = (c % stacks) * (module_bytes * modules) + (c / stacks) * module_bytes;
        s.segments.push_back(PageStripeSegment{c, base[c], count});
    }
    (void)registry.add_page_striped(s);
    for (int k = 0; k < 1200; ++k) {
        const std::uint64_t p = k < 200 ? static_cast<std::uint64_t>(k) : rng() % pages;
        const std::uint64_t within = k % 5 == 0 ? 0 : (rng() % page) & ~std::uint64_t{127};
        const std::uint32_t c = static_cast<std::uint32_t>((p + phase) % 64);
        const std::uint64_t physical = base[c] + (p / 64) * page + within;
        const PageStripeInverse inv = registry.inverse_page_striped(physical, 1, 3);
        if (inv.logical_parent_offset != p * page + within) {
            std::fprintf(stderr, "inverse mismatch at page %" PRIu64 "\n", p);
            return 1;
        }
        const StackLocation loc = map.locate(physical);
        std::printf("stripe %u %" PRIu64 " %u %u %" PRIu64 "\n", phase, p * page + within,
                    loc.stack_id, loc.module_id, loc.module_local_address);
    }
    return 0;
}

int main()
{
    std::mt19937_64 rng(20261202);
    if (bank_cases(rng)) return 1;
    for (std::uint32_t phase : {0u, 5u})
        if (stripe_cases(rng, phase)) return 1;
    return 0;
}
