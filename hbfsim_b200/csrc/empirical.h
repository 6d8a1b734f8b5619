// empirical.h -- the FAST model with an empirical burst-curve profile
// (empirical.cu).
//
// Reference: src/cuda_runtime/device/hbf_device.cu:797-838 (the empirical
// branch of resolve_fast_or_hybrid) and hbf_device.cuh:959-1140 (curve
// lookup, packed run-length state, control-header check).  One context-wide
// burst state and one context-wide channel tail; every timed access is one
// 4 KiB page whose read service comes from the curve at its run length.
#pragma once

#include "common.h"
#include "timing.h"

namespace hbfb {

constexpr u32 kRunCap = 1023;          // kEmpiricalBurstRunMask
constexpr u32 kEmpMaxCtas = 1024;      // CTAs of one batch (one scan CTA covers them)
constexpr u32 kEmpScratchWords = kEmpMaxCtas * 8 + 8;

struct EmpiricalParams {
    const u64* service;  // device [kRunCap + 1]: unscaled read service per run length
    u64 program_ns;      // unscaled write service (header program_latency_ns)
    u32 time_scale;
    u32 ok;              // control header valid, time_scale and request timeout nonzero
};

struct EmpiricalScratch {
    u64* words;          // kEmpScratchWords: per-CTA summaries and carries
    u32* error;
    u64* last_arrival;
    DevCounters* counters;
    const u64* state_in;  // [0] channel tail, [1] packed burst state
    u64* state_out;
};

// hbf_device.cuh:1107-1128 empirical_control_valid, on the profile's values.
bool empirical_control_valid(u32 flags, u32 count, u64 program_ns, const u32* pages,
                             const u64* cumulative);

// hbf_device.cuh:1021-1032 empirical_service_ns for every run length
// 0 .. kRunCap (out has kRunCap + 1 entries).
void empirical_service_table(const u32* pages, const u64* cumulative, u32 count, u64* out);

// Times one batch (device arrays).  Five launches (burst summaries, burst
// scan, tail summaries, tail scan, replay) unless `force_sequential`, then
// the exact single-thread kernel, which returns at once unless the error word
// asks for it.
cudaError_t launch_empirical(const DecodeParams& dp, const EmpiricalParams& ep,
                             const BatchIO& io, const EmpiricalScratch& s,
                             bool force_sequential, int sm_count, cudaStream_t stream,
                             const LaunchHooks& hooks = {});

}  // namespace hbfb
