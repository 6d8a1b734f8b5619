// profile.h -- HBF media profile (configs/profiles/*.json, schema
// configs/schema/hbf-profile.schema.json) as this build reads it.
#pragma once

#include <cstdint>
#include <string>

namespace hbfb {

struct EmpiricalPoint {
    std::uint32_t pages;
    std::uint64_t cumulative_ns;
    std::uint64_t p95_ns;
};

struct Profile {
    std::string name;
    std::uint64_t capacity_bytes = 0;
    std::uint32_t page_bytes = 0;
    std::uint64_t read_latency_ns = 0;
    std::uint64_t program_latency_ns = 0;
    std::uint32_t channels = 0;
    std::uint32_t dies_per_channel = 0;
    std::uint32_t planes_per_die = 0;
    std::uint32_t pages_per_block = 0;
    std::uint32_t channel_width_bits = 0;
    std::uint32_t channel_transfer_rate_mtps = 0;
    std::uint32_t queue_depth = 0;
    std::uint64_t aggregate_bandwidth_bytes_per_s = 0;
    std::uint64_t hbm_cache_bytes = 0;
    double reference_sample_rate = 0;
    std::uint32_t reference_warmup_requests = 0;
    std::uint32_t time_scale = 0;
    std::uint64_t timing_tolerance_ns = 0;
    std::string nand_technology = "SLC";
    std::string plane_allocation_scheme = "CWDP";
    std::uint64_t page_latency[8] = {};  // read lsb/csb/msb/tsb, program ...
    bool has_empirical = false;
    EmpiricalPoint empirical[6] = {};
    std::uint64_t empirical_program_p50_ns = 0;
    std::uint64_t empirical_program_p95_ns = 0;
};

// Loads and validates; returns an empty string on success or the reason.
// The rules follow src/profile/profile.cpp:238-467 of the reference.
std::string load_profile(const std::string& path, Profile* out);
std::string validate_profile(const Profile& p);

// Channel bandwidth in bytes/s: channel_width_bits / 8 * MT/s * 1e6.
std::uint64_t channel_bandwidth(const Profile& p);

}  // namespace hbfb
