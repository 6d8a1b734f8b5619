// ref_prefetch.cpp -- drives the REFERENCE prefetch model on given streams.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this driver with the
// reference's src/prefetch/prefetch_model.cpp where it lies in the HBFSim
// tree; the binary lands in oracle/_ref/.  tests/golden/make_goldens.py runs
// it to produce tests/golden/prefetch_goldens.json.
//
// Usage: ref_prefetch STREAM CELLS
//   STREAM  binary file of little-endian uint64 pages
//   CELLS   text, one cell per line:
//           policy accuracy lead buffer_pages max_in_flight read_ns compute_ns seed
// Prints one line per cell: total stall accesses misses hits issued wasted
#include <hbfsim/prefetch_model.hpp>

#include <cinttypes>
#include <cstdio>
#include <fstream>
#include <vector>

int main(int argc, char** argv)
{
    if (argc != 3) {
        std::fprintf(stderr, "usage: ref_prefetch STREAM CELLS\n");
        return 2;
    }
    std::ifstream in(argv[1], std::ios::binary);
    std::vector<std::uint64_t> pages;
    std::uint64_t v = 0;
    while (in.read(reinterpret_cast<char*>(&v), sizeof v)) pages.push_back(v);
    std::FILE* cells = std::fopen(argv[2], "r");
    if (!cells) return 2;
    unsigned policy = 0, lead = 0, buffer = 0, in_flight = 0;
    double accuracy = 0;
    unsigned long long read_ns = 0, compute_ns = 0, seed = 0;
    while (std::fscanf(cells, "%u %lf %u %u %u %llu %llu %llu", &policy, &accuracy, &lead,
                       &buffer, &in_flight, &read_ns, &compute_ns, &seed) == 8) {
        hbfsim::PrefetchConfig c{};
        c.policy = policy == 0   ? hbfsim::PrefetchPolicy::None
                   : policy == 1 ? hbfsim::PrefetchPolicy::NextPage
                                 : hbfsim::PrefetchPolicy::Accuracy;
        c.accuracy = accuracy;
        c.lead_distance = lead;
        c.buffer_pages = buffer;
        c.max_in_flight = in_flight;
        c.read_latency_ns = read_ns;
        c.compute_ns_per_access = compute_ns;
        c.seed = seed;
        const auto s = hbfsim::simulate_prefetch(pages, c);
        std::printf("%" PRIu64 " %" PRIu64 " %" PRIu64 " %" PRIu64 " %" PRIu64 " %" PRIu64
                    " %" PRIu64 "\n",
                    s.total_ns, s.stall_ns, s.demand_accesses, s.demand_misses, s.prefetch_hits,
                    s.prefetch_issued, s.prefetch_wasted);
    }
    std::fclose(cells);
    return 0;
}
