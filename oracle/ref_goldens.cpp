// ref_goldens.cpp -- golden-vector generator built against the REFERENCE.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this driver together
// with the reference's own sources, where they lie in the HBFSim tree:
//   src/cuda_runtime/device/hbf_device.cuh  (host-compilable constexpr model)
//   src/hybrid/calibrator.cpp               (host fast_service_ns)
//   src/eq3_thermal/thermal.cpp             (backward-Euler RC model)
// The binary lands in oracle/_ref/.  Its output is committed as fixtures under
// tests/golden/ by tests/golden/make_goldens.py.  Nothing here is shipped.
//
// Modes:
//   ref_goldens device          JSON lines of model-function goldens
//   ref_goldens thermal FILE    runs ThermalModel on the network in FILE
#include "cuda_runtime/device/hbf_device.cuh"

#include <hbfsim/eq3_thermal/thermal.hpp>
#include <hbfsim/hybrid_model.hpp>

#include <cinttypes>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

namespace dev = hbfsim::device;

namespace {

struct Rng {
    std::uint64_t s;
    std::uint64_t next()
    {
        std::uint64_t z = (s += 0x9e3779b97f4a7c15ULL);
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
        return z ^ (z >> 31);
    }
    std::uint64_t below(std::uint64_t n) { return n ? next() % n : 0; }
};

void emit_ranges(const std::vector<dev::SharedRangeRecord>& r)
{
    std::printf("{\"kind\":\"ranges\",\"ranges\":[");
    for (std::size_t i = 0; i < r.size(); ++i) {
        std::printf("%s[%" PRIu64 ",%" PRIu64 ",%" PRIu64 ",%u,%u,%u,%" PRIu64 "]",
                    i ? "," : "", r[i].base, r[i].length, r[i].file_offset,
                    r[i].range_id, r[i].mode, r[i].permissions, r[i].page_bytes);
    }
    std::printf("]}\n");
}

// Probe one access against the table with the reference functions.
void emit_probe(const std::vector<dev::SharedRangeRecord>& r, std::uint64_t a,
                std::uint32_t bytes, std::uint32_t op)
{
    const auto count = static_cast<std::uint32_t>(r.size());
    const auto index = dev::find_range_index(r.data(), count, a);
    int supported = -1, media_valid = -1, succ_overlap = -1, touches = -1;
    std::uint64_t logical = 0;
    std::uint32_t media_bytes = 0;
    if (index != count) {
        supported = dev::access_supported(r[index], a, bytes, op) ? 1 : 0;
        const auto m = dev::media_descriptor(r[index], a, bytes, op);
        media_valid = m.valid ? 1 : 0;
        logical = m.logical_address;
        media_bytes = m.bytes;
    }
    const auto successor = index == count ? 0U : index + 1U;
    if (successor < count)
        succ_overlap = dev::range_overlaps(r[successor], a, bytes) ? 1 : 0;
    touches = dev::span_touches_any_range(r.data(), count, a, bytes) ? 1 : 0;
    std::printf("{\"kind\":\"probe\",\"a\":%" PRIu64 ",\"bytes\":%u,\"op\":%u,"
                "\"index\":%u,\"supported\":%d,\"media_valid\":%d,"
                "\"logical\":%" PRIu64 ",\"media_bytes\":%u,"
                "\"succ_overlap\":%d,\"touches\":%d}\n",
                a, bytes, op, index, supported, media_valid, logical,
                media_bytes, succ_overlap, touches);
}

// Empirical burst-curve profile (hbf_device.cuh:959-1140): curve lookups,
// the packed run-length state, the control-header check and the request
// service, all by the reference functions; then traces of the empirical fast
// path (hbf_device.cu:797-838: burst CAS, then the tail CAS with the scaled
// service) with arrivals in place of the globaltimer.
void emit_u64s(const char* name, const std::uint64_t* v, std::size_t n, bool last = false)
{
    std::printf("\"%s\":[", name);
    for (std::size_t i = 0; i < n; ++i) std::printf("%s%" PRIu64, i ? "," : "", v[i]);
    std::printf("]%s", last ? "" : ",");
}

dev::SharedControlHeader empirical_header(const std::uint32_t* pages, const std::uint64_t* cum,
                                          std::uint64_t program)
{
    dev::SharedControlHeader h{};
    h.empirical_flags = 1;
    h.empirical_point_count = 6;
    h.program_latency_ns = program;
    for (int i = 0; i < 6; ++i) {
        h.empirical_breakpoint_pages[i] = pages[i];
        h.empirical_cumulative_ns[i] = cum[i];
    }
    return h;
}

void random_curve(Rng& rng, std::uint32_t* pages, std::uint64_t* cum, std::uint32_t last_max)
{
    std::uint32_t p = 0;
    std::uint64_t c = 0;
    for (int i = 0; i < 6; ++i) {
        const std::uint32_t room = last_max - p - static_cast<std::uint32_t>(5 - i);
        p += 1 + static_cast<std::uint32_t>(rng.below(std::min<std::uint32_t>(room, 300)));
        c += 1 + rng.below(i == 0 ? 20'000 : 4'000'000);
        pages[i] = p;
        cum[i] = c;
    }
}

void empirical_goldens(Rng& rng)
{
    // 7a. curve lookups over every run length the state can hold, and beyond
    struct Curve {
        std::uint32_t pages[6];
        std::uint64_t cum[6];
        std::uint32_t count;
    };
    std::vector<Curve> curves;
    curves.push_back({{1, 4, 16, 64, 256, 512},
                      {11'133, 41'495, 168'606, 2'824'351, 10'767'793, 20'254'374}, 6});
    curves.push_back({{1, 2, 0, 0, 0, 0}, {UINT64_MAX - 1, UINT64_MAX, 0, 0, 0, 0}, 2});
    curves.push_back({{3, 7, 8, 100, 101, 1023}, {5, 9, 10, 1'000'000, 1'000'001, 9'000'000}, 6});
    for (int k = 0; k < 5; ++k) {
        Curve c{};
        c.count = 6;
        random_curve(rng, c.pages, c.cum, 1023);
        curves.push_back(c);
    }
    for (const auto& c : curves) {
        std::vector<std::uint64_t> runs, cumulative, service;
        for (std::uint64_t r = 0; r <= 1100; ++r) runs.push_back(r);
        for (std::uint64_t r : {100'000ULL, 4'294'967'295ULL}) runs.push_back(r);
        for (auto r : runs) {
            const auto run = static_cast<std::uint32_t>(r);
            cumulative.push_back(dev::empirical_cumulative_ns(c.pages, c.cum, c.count, run));
            service.push_back(dev::empirical_service_ns(c.pages, c.cum, c.count, run));
        }
        std::uint64_t pages64[6];
        for (int i = 0; i < 6; ++i) pages64[i] = c.pages[i];
        std::printf("{\"kind\":\"emp_curve\",\"count\":%u,", c.count);
        emit_u64s("pages", pages64, c.count);
        emit_u64s("cum", c.cum, c.count);
        emit_u64s("runs", runs.data(), runs.size());
        emit_u64s("cumulative", cumulative.data(), cumulative.size());
        emit_u64s("service", service.data(), service.size(), true);
        std::printf("}\n");
    }
    // 7b. packed run-length state: chains of updates
    constexpr std::uint64_t kMaxPage = (std::uint64_t{1} << 53) - 2;
    for (int chain = 0; chain < 4; ++chain) {
        std::printf("{\"kind\":\"emp_burst\",\"steps\":[");
        std::uint64_t state = 0;
        std::uint64_t page = chain == 3 ? kMaxPage - 40 : rng.below(1u << 20);
        std::uint32_t op = 0;
        const int steps = chain == 0 ? 1200 : 600;
        for (int i = 0; i < steps; ++i) {
            const auto r = rng.below(100);
            if (chain == 0 || r < 70) page += 1;
            else if (r < 78) page = rng.below(1ULL << 40);
            else if (r < 83) op ^= 1u;
            else if (r < 86) {}  // the same page again
            else if (r < 90) page = page - 1;
            else if (r < 93) page = kMaxPage + rng.below(3);
            else if (r < 95) page = rng.below(64);
            std::uint32_t use_op = op;
            if (chain != 0 && rng.below(60) == 0) use_op = 2 + static_cast<std::uint32_t>(rng.below(3));
            const auto u = dev::update_empirical_burst(state, page, use_op);
            std::printf("%s[%" PRIu64 ",%" PRIu64 ",%u,%" PRIu64 ",%u,%d]", i ? "," : "", state,
                        page, use_op, u.packed, u.run_pages, u.valid ? 1 : 0);
            if (u.valid) state = u.packed;
            if (page > kMaxPage) page = rng.below(1u << 20);
        }
        std::printf("]}\n");
    }
    // 7c. control-header validity
    {
        const std::uint32_t pages[6] = {1, 4, 16, 64, 256, 512};
        const std::uint64_t cum[6] = {11'133, 41'495, 168'606, 2'824'351, 10'767'793, 20'254'374};
        for (int k = 0; k < 40; ++k) {
            auto h = empirical_header(pages, cum, 408'305);
            switch (k % 10) {
            case 0: break;
            case 1: h.empirical_point_count = static_cast<std::uint32_t>(rng.below(12)); break;
            case 2: h.empirical_breakpoint_pages[rng.below(6)] = 0; break;
            case 3: h.empirical_cumulative_ns[rng.below(6)] = 0; break;
            case 4: {
                const auto i = 1 + rng.below(5);
                h.empirical_breakpoint_pages[i] = h.empirical_breakpoint_pages[i - 1];
                break;
            }
            case 5: {
                const auto i = 1 + rng.below(5);
                h.empirical_cumulative_ns[i] = h.empirical_cumulative_ns[i - 1] - rng.below(2);
                break;
            }
            case 6: h.empirical_breakpoint_pages[5] = 1023 + static_cast<std::uint32_t>(rng.below(3)); break;
            case 7: h.empirical_flags = static_cast<std::uint32_t>(rng.below(4)); break;
            case 8: h.program_latency_ns = rng.below(2); break;
            default: {
                std::uint32_t p[6];
                std::uint64_t c[6];
                random_curve(rng, p, c, 1023);
                h = empirical_header(p, c, 1 + rng.below(1'000'000));
            }
            }
            std::uint64_t p64[6];
            for (int i = 0; i < 6; ++i) p64[i] = h.empirical_breakpoint_pages[i];
            std::printf("{\"kind\":\"emp_control\",\"flags\":%u,\"count\":%u,\"program\":%" PRIu64 ",",
                        h.empirical_flags, h.empirical_point_count, h.program_latency_ns);
            emit_u64s("pages", p64, 6);
            emit_u64s("cum", h.empirical_cumulative_ns, 6);
            const auto first = dev::empirical_request_service(h, 0, 5, 0);
            std::printf("\"valid\":%d,\"service\":%" PRIu64 "}\n",
                        dev::empirical_control_valid(h) ? 1 : 0, first.valid ? first.service_ns : 0);
        }
    }
    // 7d. traces of the empirical fast path
    for (int trace = 0; trace < 4; ++trace) {
        std::uint32_t pages[6] = {1, 4, 16, 64, 256, 512};
        std::uint64_t cum[6] = {11'133, 41'495, 168'606, 2'824'351, 10'767'793, 20'254'374};
        std::uint64_t program = 408'305;
        if (trace == 1 || trace == 3) {
            random_curve(rng, pages, cum, trace == 3 ? 1023 : 600);
            program = 1 + rng.below(2'000'000);
        }
        const auto h = empirical_header(pages, cum, program);
        const std::uint32_t scale = trace == 1 ? 7 : 1;
        std::uint64_t tail = trace == 2 ? UINT64_MAX - 50'000'000ULL : 0;
        std::uint64_t arrival = trace == 2 ? UINT64_MAX - 60'000'000ULL : 0;
        std::uint64_t state = 0;
        std::uint64_t pages64[6];
        for (int i = 0; i < 6; ++i) pages64[i] = pages[i];
        std::printf("{\"kind\":\"emp_trace\",\"program\":%" PRIu64 ",\"scale\":%u,\"tail0\":%" PRIu64 ",",
                    program, scale, tail);
        emit_u64s("pages", pages64, 6);
        emit_u64s("cum", cum, 6);
        std::printf("\"steps\":[");
        std::uint64_t page = rng.below(1u << 16);
        std::uint32_t op = 0;
        std::uint64_t streak = 0;
        for (int i = 0; i < 3000; ++i) {
            if (streak == 0) {
                // a new streak: sequential pages of one operation
                const auto r = rng.below(10);
                streak = r < 6 ? 1 + rng.below(8) : r < 9 ? 1 + rng.below(300) : 900 + rng.below(400);
                page = rng.below(1u << 16);
                op = rng.below(12) == 0 ? 1u : 0u;
            }
            --streak;
            arrival = dev::saturating_add(arrival, rng.below(4) == 0 ? rng.below(400'000) : rng.below(30));
            const auto request = dev::empirical_request_service(h, state, page, op);
            std::uint64_t target = 0;
            if (request.valid) {
                state = request.packed_state;
                const auto scaled = dev::saturating_multiply(request.service_ns, scale);
                const auto start = tail > arrival ? tail : arrival;
                target = dev::saturating_add(start, scaled);
                tail = target;
            }
            std::printf("%s[%" PRIu64 ",%" PRIu64 ",%u,%d,%" PRIu64 ",%" PRIu64 ",%u]", i ? "," : "",
                        arrival, page, op, request.valid ? 1 : 0, target, request.service_ns,
                        request.run_pages);
            page += 1;
        }
        std::printf("]}\n");
    }
}

int device_goldens()
{
    Rng rng{12345};
    // 1. The reference unit-test table (tests/cpu/device_helper_abi_test.cpp).
    std::vector<dev::SharedRangeRecord> fixed{
        {.base = 0x1000, .length = 0x1000, .file_offset = 0x8000,
         .range_id = 1, .mode = 1, .permissions = 3, .page_bytes = 0x1000},
        {.base = 0x4000, .length = 0x2000, .file_offset = 0x10'000,
         .range_id = 2, .mode = 1, .permissions = 1, .page_bytes = 0x1000},
        {.base = 0x8000, .length = 0x2000, .file_offset = 0x20'000,
         .range_id = 3, .mode = 2, .permissions = 3, .page_bytes = 0x1000},
    };
    emit_ranges(fixed);
    for (std::uint64_t a = 0x0ff0; a < 0xa010; a += 0x1f8) {
        for (std::uint32_t bytes : {0u, 1u, 8u, 16u, 0x800u, 0x1001u})
            for (std::uint32_t op : {0u, 1u, 2u}) emit_probe(fixed, a, bytes, op);
    }
    // 2. Random sorted, non-overlapping tables.
    for (int table = 0; table < 6; ++table) {
        std::vector<dev::SharedRangeRecord> r;
        const int n = 1 + static_cast<int>(rng.below(40));
        std::uint64_t cursor = 0x10000 + rng.below(1 << 20);
        std::uint64_t file = 0;
        for (int i = 0; i < n; ++i) {
            const std::uint64_t page = 512ULL << rng.below(6);
            const std::uint64_t len = 1 + rng.below(page * 6);
            dev::SharedRangeRecord rec{};
            rec.base = cursor;
            rec.length = len;
            rec.file_offset = file;
            rec.range_id = static_cast<std::uint32_t>(i + 1);
            rec.mode = 1 + static_cast<std::uint32_t>(rng.below(2));
            rec.permissions = 1 + static_cast<std::uint32_t>(rng.below(3));
            rec.page_bytes = page;
            r.push_back(rec);
            file += ((len + page - 1) / page) * page;
            cursor += len + rng.below(3) * rng.below(page * 2);
        }
        emit_ranges(r);
        for (int p = 0; p < 400; ++p) {
            const auto& pick = r[rng.below(r.size())];
            std::uint64_t a;
            switch (rng.below(4)) {
            case 0: a = pick.base + rng.below(pick.length + 64); break;
            case 1: a = pick.base - 1 - rng.below(64); break;
            case 2: a = pick.base + pick.length - 1 - rng.below(64); break;
            default: a = rng.below(cursor + 4096); break;
            }
            const std::uint32_t bytes =
                rng.below(8) == 0 ? 0u
                                  : static_cast<std::uint32_t>(1 + rng.below(9000));
            emit_probe(r, a, bytes, static_cast<std::uint32_t>(rng.below(3)));
        }
    }
    // 3. fast_transfer_ns / fast_service_ns, host == device pin.
    const std::uint64_t bws[] = {1, 7, 1'000'000'000ULL, 8'000'000'000ULL,
                                 128'000'000'000ULL, 512'000'000'000ULL,
                                 1'000'000'000'000ULL, 3'000'000'007ULL};
    const std::uint32_t sizes[] = {0, 1, 128, 512, 1024, 4096, 16384,
                                   1'048'576, 268'435'456, 4'294'967'295U};
    for (auto bw : bws) {
        for (auto b : sizes) {
            const hbfsim::FastModelProfile prof{10'000, 200'000, bw};
            const hbfsim::AccessClass cls{hbfsim::RequestOperation::Read, b, 0, 0};
            std::printf("{\"kind\":\"transfer\",\"bytes\":%u,\"bw\":%" PRIu64
                        ",\"transfer\":%" PRIu64 ",\"service\":%" PRIu64
                        ",\"host_service\":%" PRIu64 "}\n",
                        b, bw, dev::fast_transfer_ns(b, bw),
                        dev::fast_service_ns(10'000, b, bw),
                        hbfsim::fast_service_ns(prof, cls));
        }
    }
    // 4. Saturating arithmetic.
    const std::uint64_t big[] = {0, 1, 2, 1000, UINT64_MAX / 3, UINT64_MAX - 1,
                                 UINT64_MAX};
    for (auto x : big)
        for (auto y : big)
            std::printf("{\"kind\":\"sat\",\"a\":%" PRIu64 ",\"b\":%" PRIu64
                        ",\"add\":%" PRIu64 ",\"mul\":%" PRIu64 "}\n",
                        x, y, dev::saturating_add(x, y),
                        dev::saturating_multiply(
                            x, static_cast<std::uint32_t>(y & 0xffffffffULL)));
    // 5. Hybrid sampler bit.
    for (int k = 0; k < 200; ++k) {
        const std::uint64_t seq = rng.below(5000);
        const std::uint32_t warm = static_cast<std::uint32_t>(rng.below(8));
        const std::uint64_t thr = rng.below(4) == 0 ? 0 : rng.next();
        const std::uint64_t key = rng.next();
        std::printf("{\"kind\":\"hybrid\",\"seq\":%" PRIu64 ",\"warmup\":%u,"
                    "\"threshold\":%" PRIu64 ",\"key\":%" PRIu64
                    ",\"sample\":%d}\n",
                    seq, warm, thr, key,
                    dev::hybrid_reference_sample(seq, warm, thr, key) ? 1 : 0);
    }
    // 6. Fast-model trace: the tail recurrence of hbf_device.cu:883-910 with
    //    the reference's own helpers, arrivals in place of the globaltimer.
    for (int trace = 0; trace < 3; ++trace) {
        const std::uint64_t read_lat = trace == 2 ? 11'133 : 3'000;
        const std::uint64_t prog_lat = 200'000;
        const std::uint64_t bw = trace == 1 ? 512'000'000'000ULL
                                            : 128'000'000'000ULL;
        const std::uint32_t page = trace == 0 ? 16384 : 4096;
        const std::uint32_t scale = trace == 1 ? 100 : 1;
        std::uint64_t tail = trace == 2 ? UINT64_MAX - 5'000'000 : 0;
        std::uint64_t arrival = trace == 2 ? UINT64_MAX - 9'000'000 : 0;
        std::printf("{\"kind\":\"fast_trace\",\"read_lat\":%" PRIu64
                    ",\"prog_lat\":%" PRIu64 ",\"bw\":%" PRIu64
                    ",\"page\":%u,\"scale\":%u,\"tail0\":%" PRIu64
                    ",\"steps\":[",
                    read_lat, prog_lat, bw, page, scale, tail);
        for (int i = 0; i < 1500; ++i) {
            arrival = dev::saturating_add(arrival, rng.below(3) * rng.below(400));
            const std::uint32_t op = rng.below(20) == 0 ? 1 : 0;
            const auto base = op == 0 ? read_lat : prog_lat;
            const auto transfer = dev::fast_transfer_ns(page, bw);
            const auto base_scaled = dev::saturating_multiply(base, scale);
            const auto transfer_scaled = dev::saturating_multiply(transfer, scale);
            const auto start = tail > arrival ? tail : arrival;
            tail = dev::saturating_add(start, transfer_scaled);
            const auto latency_target = dev::saturating_add(arrival, base_scaled);
            const auto target = latency_target > tail ? latency_target : tail;
            std::printf("%s[%" PRIu64 ",%u,%" PRIu64 ",%" PRIu64 "]",
                        i ? "," : "", arrival, op, target,
                        dev::fast_service_ns(base, page, bw));
        }
        std::printf("]}\n");
    }
    empirical_goldens(rng);
    return 0;
}

// Thermal: read "nodes N" then N lines (C G_boundary T_boundary T0 P_static),
// "edges M" then M lines (a b G), "steps K dt" then K lines of N node powers
// (W, constant over the step, applied as one activity per node per step).
int thermal_goldens(const char* path)
{
    std::ifstream in(path);
    if (!in) return 2;
    using namespace hbfsim::eq3_thermal;
    std::string word;
    std::size_t n = 0, m = 0, k = 0;
    double dt = 0;
    ThermalModelConfig cfg;
    in >> word >> n;
    for (std::size_t i = 0; i < n; ++i) {
        ThermalNode node;
        node.id = "n" + std::to_string(i);
        node.physical_type = PhysicalType::Hbf;
        node.logical_role = LogicalRole::CapacityMemory;
        in >> node.heat_capacity_j_per_k >> node.boundary_conductance_w_per_k >>
            node.boundary_temperature_k >> node.initial_temperature_k >>
            node.static_power_w;
        cfg.nodes.push_back(node);
    }
    in >> word >> m;
    for (std::size_t i = 0; i < m; ++i) {
        ThermalEdge e;
        e.kind = ConductanceKind::IntraComponent;
        in >> e.node_a >> e.node_b >> e.conductance_w_per_k;
        cfg.edges.push_back(e);
    }
    in >> word >> k >> dt;
    ThermalModel model(cfg);
    std::uint64_t id = 1;
    for (std::size_t s = 0; s < k; ++s) {
        const double t0 = dt * static_cast<double>(s);
        const double t1 = dt * static_cast<double>(s + 1);
        for (std::size_t i = 0; i < n; ++i) {
            double p = 0;
            in >> p;
            if (p > 0) {
                PhysicalActivity a;
                a.activity_id = id++;
                a.request_id = "step" + std::to_string(s);
                a.kind = ActivityKind::Read;
                a.source = ActivitySource::Demand;
                a.start_time_s = t0;
                a.end_time_s = t1;
                a.completion_time_s = t1;
                a.node_energy.push_back({i, p * (t1 - t0)});
                model.add_activity(a);
            }
        }
        model.advance_to(t1);
        std::printf("step %zu", s);
        for (double t : model.temperatures_k()) std::printf(" %.17g", t);
        std::printf("\n");
    }
    return 0;
}

}  // namespace

int main(int argc, char** argv)
{
    if (argc >= 2 && std::strcmp(argv[1], "device") == 0) return device_goldens();
    if (argc >= 3 && std::strcmp(argv[1], "thermal") == 0)
        return thermal_goldens(argv[2]);
    std::fprintf(stderr, "usage: ref_goldens device | thermal FILE\n");
    return 64;
}
