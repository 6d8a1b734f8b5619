// ref_clock.cpp -- drives the REFERENCE HBM cache (second-chance CLOCK) the
// way the reference's capacity service resolves one page reference at a time.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this driver with the
// reference's src/cuda_runtime/hbm_cache.cpp where it lies in the HBFSim tree;
// the binary lands in oracle/_ref/.  tests/golden/make_goldens.py runs it to
// produce tests/golden/clock_goldens.json.
//
// Per reference (CapacityPageService::resolve,
// src/host_service/capacity_page_service.cpp:97-210, without the byte moves):
// a resident page is a hit (resolve sets its reference bit; a write marks it
// dirty); otherwise the first free frame is taken, or -- when every frame is
// full -- begin_eviction picks the CLOCK victim and complete_eviction frees
// its frame; then publish places the page (referenced, clean) and a write
// marks it dirty.
//
// Input (text): frames n, then n lines "page op".
// Output: n lines "hit victim dirty" (victim 18446744073709551615 = none).
#include "cuda_runtime/hbm_cache.hpp"

#include <cinttypes>
#include <cstdio>
#include <vector>

int main()
{
    unsigned long long frames = 0, n = 0;
    if (std::scanf("%llu %llu", &frames, &n) != 2 || frames == 0) return 2;
    std::vector<std::uint64_t> addresses(frames);
    for (unsigned long long k = 0; k < frames; ++k) addresses[k] = 4096 * (k + 1);
    hbfsim::runtime::HbmCache cache(addresses);
    for (unsigned long long i = 0; i < n; ++i) {
        unsigned long long page = 0;
        unsigned op = 0;
        if (std::scanf("%llu %u", &page, &op) != 2) return 2;
        std::uint64_t victim = ~std::uint64_t{0};
        int dirty = 0;
        if (cache.resolve(page)) {
            if (op == 1 && !cache.mark_dirty(page)) return 3;
            std::printf("1 %" PRIu64 " 0\n", victim);
            continue;
        }
        auto frame = cache.free_frame();
        if (!frame) {
            const auto eviction = cache.begin_eviction();
            if (!eviction || !cache.complete_eviction(*eviction)) return 3;
            victim = eviction->logical_page;
            dirty = eviction->dirty ? 1 : 0;
            frame = eviction->frame_address;
        }
        if (!cache.publish(page, *frame)) return 3;
        if (op == 1 && !cache.mark_dirty(page)) return 3;
        std::printf("0 %" PRIu64 " %d\n", victim, dirty);
    }
    return 0;
}
