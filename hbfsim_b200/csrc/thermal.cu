// thermal.cu -- eq3 layered thermal grid and the refresh / throttle epoch
// controller, on the GPU in fp64.
//
// Grid (reference tools/eq3_layered_export.py:48-114): nz layers of nx*ny
// square cells, each layer one material; lateral edges G = k*dz (square
// cells), vertical edges G = dx*dy / (dz_a/(2 kz_a) + dz_b/(2 kz_b)), Robin
// boundaries on the bottom and top faces g = dx*dy / (dz/(2 kz) + 1/h),
// insulated sides.  Step (ThermalModel::advance_to, src/eq3_thermal/
// thermal.cpp:242-311): backward Euler
//     (C/dt + G_b + L) T+ = C/dt T + P + G_b T_amb.
//
// B200 design: with one material per layer and insulated sides, the lateral
// part of L is G_x,z (L_x (x) I) + G_y,z (I (x) L_y) with the Neumann 1-D
// Laplacians L_x, L_y, which the orthonormal DCT-II diagonalizes exactly
// (eigenvalues 2 - 2 cos(pi p / n)).  So the implicit step is solved
// directly, not iteratively:
//     rhs -> DCT over x and y (two fp64 GEMMs against the cosine matrices)
//         -> one nz-point tridiagonal solve per (p, q) mode (Thomas)
//         -> inverse DCT (two more GEMMs).
// Accuracy is that of the transforms (~1e-14 relative), well inside the
// 1e-9 tolerance against the sparse direct solve of the oracle.  The GEMMs
// run on the double-precision tensor cores.
#include "context.h"

#include <algorithm>
#include <cmath>
#include <vector>

namespace hbfb {

struct ThermalState {
    hbfsim_thermal_config_v1 cfg{};
    int nx = 0, ny = 0, nz = 0;
    std::uint64_t cells = 0;
    std::uint32_t dies_total = 0;   // global dies (channels_total * D)
    // per-layer coefficients (device)
    double* d_cap = nullptr;    // C_z per cell
    double* d_gb = nullptr;     // boundary conductance per cell of layer z
    double* d_tb = nullptr;     // boundary ambient of layer z
    double* d_gx = nullptr;     // lateral x edge conductance of layer z
    double* d_gy = nullptr;
    double* d_gz = nullptr;     // vertical conductance between z and z+1
    double* d_lx = nullptr;     // DCT eigenvalues
    double* d_ly = nullptr;
    double* d_qx = nullptr;     // nx x nx cosine matrix
    double* d_qy = nullptr;
    double* d_t = nullptr;      // temperatures
    double* d_w0 = nullptr;     // work
    double* d_w1 = nullptr;
    int* d_cell_die = nullptr;  // owning global die or -1
    double* d_die_cells = nullptr;
    int* d_die_start = nullptr;  // cells of die d: d_die_list[start[d] .. start[d+1])
    int* d_die_list = nullptr;
    double* d_die_temp = nullptr;
    std::uint32_t* d_level = nullptr;    // throttle level per stack
    std::uint32_t* d_refresh = nullptr;  // per local channel (permille)
    std::uint32_t* d_throttle = nullptr; // per stack (permille)
    std::uint64_t* d_admit = nullptr;    // per stack
    std::uint64_t epoch_end_ns = 0;
    std::uint64_t epochs = 0;
    // bounds of what the controller can write into the channel tables
    std::uint64_t x_bound = 0, op_bound = 0, admit_bound = 0;
};

const double* thermal_die_temperatures(const ThermalState* t) { return t->d_die_temp; }

void thermal_factor_arrays(ThermalState* t, std::uint32_t** refresh, std::uint32_t** throttle,
                           std::uint64_t** admit)
{
    *refresh = t->d_refresh;
    *throttle = t->d_throttle;
    *admit = t->d_admit;
}

void thermal_tick_bounds(const ThermalState* t, std::uint64_t* x, std::uint64_t* op,
                         std::uint64_t* admit)
{
    *x = t->x_bound;
    *op = t->op_bound;
    *admit = t->admit_bound;
}

void thermal_destroy(ThermalState* t)
{
    if (!t) return;
    for (void* p : {static_cast<void*>(t->d_cap), static_cast<void*>(t->d_gb),
                    static_cast<void*>(t->d_tb), static_cast<void*>(t->d_gx),
                    static_cast<void*>(t->d_gy), static_cast<void*>(t->d_gz),
                    static_cast<void*>(t->d_lx), static_cast<void*>(t->d_ly),
                    static_cast<void*>(t->d_qx), static_cast<void*>(t->d_qy),
                    static_cast<void*>(t->d_t), static_cast<void*>(t->d_w0),
                    static_cast<void*>(t->d_w1), static_cast<void*>(t->d_cell_die),
                    static_cast<void*>(t->d_die_cells),
                    static_cast<void*>(t->d_die_start), static_cast<void*>(t->d_die_list),
                    static_cast<void*>(t->d_die_temp), static_cast<void*>(t->d_level),
                    static_cast<void*>(t->d_refresh), static_cast<void*>(t->d_throttle),
                    static_cast<void*>(t->d_admit)})
        if (p) cudaFree(p);
    delete t;
}

namespace {

// C[b] = op(A[b]) * op(B[b]) in fp64 on the double-precision tensor cores
// (mma.sync m8n8k4 .f64; the tcgen05 instructions have no fp64 kind).
// op(X) = X or X^T; row-major storage with leading dimension = columns.
// CTA tile 32 x 32 (enough CTAs for the small transforms of the grid), K
// step 32, four warps of 16 x 16 (2 x 2 MMA tiles).  Fragment layout of
// m8n8k4 .f64 (PTX ISA): lane = 4 g + t holds A(g, t), B(t, g) and C(g, 2t),
// C(g, 2t + 1).
constexpr int kBM = 32, kBN = 32, kBK = 32;

__device__ __forceinline__ void dmma_8x8x4(double& c0, double& c1, double a, double b)
{
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
                 : "+d"(c0), "+d"(c1)
                 : "d"(a), "d"(b));
}

// 8-byte global -> shared copy that zero-fills when `bytes` is 0 (then
// nothing is read at `gmem_src`).  A thread issues all of its copies of a K
// step before it waits, so the step costs one memory round trip.
__device__ __forceinline__ void cp_async8z(void* smem_dst, const void* gmem_src, unsigned bytes)
{
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(dst), "l"(gmem_src),
                 "r"(bytes));
}

__global__ void __launch_bounds__(128) dgemm_kernel(int M, int N, int K, const double* A,
                                                    long long sa, int ta, const double* B,
                                                    long long sb, int tb, double* C, long long sc)
{
    // two K steps in shared memory: the next one streams in while the
    // current one feeds the MMAs
    __shared__ double as[2][kBK][kBM + 1];  // as[.][k][m] = op(A)(m, k)
    __shared__ double bs[2][kBK][kBN + 1];  // bs[.][k][n] = op(B)(k, n)
    const double* a = A + sa * blockIdx.z;
    const double* b = B + sb * blockIdx.z;
    double* c = C + sc * blockIdx.z;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int wm = (warp >> 1) * 16, wn = (warp & 1) * 16;
    // global loads run along the contiguous dimension of each operand
    auto stage = [&](int k0, int buf) {
#pragma unroll
        for (int idx = tid; idx < kBK * kBM; idx += 128) {
            int m, k;
            if (ta) { k = idx / kBM; m = idx % kBM; } else { m = idx / kBK; k = idx % kBK; }
            const int gm = m0 + m, gk = k0 + k;
            const bool in = gm < M && gk < K;
            const double* src = in ? (ta ? a + static_cast<long long>(gk) * M + gm
                                         : a + static_cast<long long>(gm) * K + gk)
                                   : a;
            cp_async8z(&as[buf][k][m], src, in ? 8u : 0u);
        }
#pragma unroll
        for (int idx = tid; idx < kBK * kBN; idx += 128) {
            int n, k;
            if (tb) { n = idx / kBK; k = idx % kBK; } else { k = idx / kBN; n = idx % kBN; }
            const int gn = n0 + n, gk = k0 + k;
            const bool in = gk < K && gn < N;
            const double* src = in ? (tb ? b + static_cast<long long>(gn) * K + gk
                                         : b + static_cast<long long>(gk) * N + gn)
                                   : b;
            cp_async8z(&bs[buf][k][n], src, in ? 8u : 0u);
        }
        asm volatile("cp.async.commit_group;\n" ::);
    };
    double acc[2][2][2];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;
    stage(0, 0);
    for (int k0 = 0, it = 0; k0 < K; k0 += kBK, ++it) {
        const int cur = it & 1;
        if (k0 + kBK < K) {
            stage(k0 + kBK, cur ^ 1);
            asm volatile("cp.async.wait_group 1;\n" ::: "memory");  // the current step landed
        } else {
            asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kBK; kk += 4) {
            double fa[2], fb[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) fa[i] = as[cur][kk + t][wm + i * 8 + g];
#pragma unroll
            for (int j = 0; j < 2; ++j) fb[j] = bs[cur][kk + t][wn + j * 8 + g];
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j) dmma_8x8x4(acc[i][j][0], acc[i][j][1], fa[i], fb[j]);
        }
        __syncthreads();  // every warp is done with `cur` before it is refilled
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int row = m0 + wm + i * 8 + g;
        if (row >= M) continue;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int col = n0 + wn + j * 8 + 2 * t;
            if (col < N) c[static_cast<long long>(row) * N + col] = acc[i][j][0];
            if (col + 1 < N) c[static_cast<long long>(row) * N + col + 1] = acc[i][j][1];
        }
    }
}

void dgemm(int M, int N, int K, const double* A, long long sa, int ta, const double* B,
           long long sb, int tb, double* C, long long sc, int batch, cudaStream_t s)
{
    dim3 grid((N + kBN - 1) / kBN, (M + kBM - 1) / kBM, batch);
    dgemm_kernel<<<grid, 128, 0, s>>>(M, N, K, A, sa, ta, B, sb, tb, C, sc);
}

// rhs = C/dt T + P + G_b T_amb
// with the owning die's power (die_power_kernel's formula) folded in
__global__ void rhs_kernel(const double* t, const int* cell_die,
                           const unsigned long long* rb, const unsigned long long* wr,
                           double idle, double jpb, double jpw, const double* die_cells,
                           const double* cap, const double* gb, const double* tb, int plane,
                           long long cells, double dt, double* rhs)
{
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= cells) return;
    const int z = static_cast<int>(i / plane);
    const int d = cell_die[i];
    double p = 0.0;
    if (d >= 0) {
        const double e = static_cast<double>(rb[d]) * jpb + static_cast<double>(wr[d]) * jpw;
        p = (idle + e / dt) / die_cells[d];
    }
    rhs[i] = cap[z] / dt * t[i] + p + gb[z] * tb[z];
}

// Thomas algorithm along z for every (q, p) mode; nz <= 32.
__global__ void tridiag_kernel(const double* rhs, int nx, int ny, int nz, const double* cap,
                               const double* gb, const double* gx, const double* gy,
                               const double* gz, const double* lx, const double* ly,
                               double dt, double* out)
{
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    const int plane = nx * ny;
    if (m >= plane) return;
    const int q = m / nx, p = m % nx;
    double cp[32], dp[32];
    double prev_c = 0.0, prev_d = 0.0;
    for (int z = 0; z < nz; ++z) {
        const double down = z > 0 ? gz[z - 1] : 0.0;
        const double up = z + 1 < nz ? gz[z] : 0.0;
        const double diag = cap[z] / dt + gb[z] + gx[z] * lx[p] + gy[z] * ly[q] + down + up;
        const double a = -down, c = -up;
        const double r = rhs[static_cast<long long>(z) * plane + m];
        const double denom = diag - a * prev_c;
        const double cz = c / denom;
        const double dz = (r - a * prev_d) / denom;
        cp[z] = cz;
        dp[z] = dz;
        prev_c = cz;
        prev_d = dz;
    }
    double x = dp[nz - 1];
    out[static_cast<long long>(nz - 1) * plane + m] = x;
    for (int z = nz - 2; z >= 0; --z) {
        x = dp[z] - cp[z] * x;
        out[static_cast<long long>(z) * plane + m] = x;
    }
}

// Mean temperature of each global die over its cells (one block per die,
// over the die's own cell list; fixed summation order).
__global__ void die_temp_kernel(const double* t, const int* die_start, const int* die_list,
                                int dies, const double* die_cells, double* mean_out)
{
    const int d = blockIdx.x;
    if (d >= dies) return;
    double s = 0.0;
    for (int k = die_start[d] + threadIdx.x; k < die_start[d + 1]; k += blockDim.x)
        s += t[die_list[k]];
    __shared__ double red[256];
    red[threadIdx.x] = s;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x == 0) mean_out[d] = die_cells[d] > 0 ? red[0] / die_cells[d] : 0.0;
}

struct ControllerArgs {
    const double* die_temp;   // global dies
    int dies;                 // per channel
    int channels_total;
    int stacks;
    int local_channels;
    int shard_rank, shard_count;
    double onset_k, step_k;
    unsigned base_permille, cap_permille;
    double light_k, severe_k, shutdown_k, hysteresis_k;
    unsigned light_permille, severe_permille;
    unsigned long long next_epoch_end;
    std::uint32_t* level;     // per stack, persistent
    std::uint32_t* refresh;   // per local channel
    std::uint32_t* throttle;  // per stack
    std::uint64_t* admit;     // per stack
    // timing tables of the context
    std::uint64_t chan_bw_nominal;
    std::uint64_t* chan_bw;
    i64* t_read;
    i64* t_prog;
    i64* t_admit;
    std::uint64_t read_latency, program_latency;
    unsigned time_scale;
    // this context's die activity, cleared for the next epoch
    unsigned long long* act_read;
    unsigned long long* act_write;
    int act_words;
};

__device__ std::uint64_t sat_mul_dev(std::uint64_t a, std::uint64_t b)
{
    if (a == 0 || b == 0) return 0;
    return a > ~0ull / b ? ~0ull : a * b;
}

// Refresh: a die at T_d refreshes at base * 2^floor((T_d - onset)/step) permille
// (base below the onset); a channel gives up the mean of its dies' shares,
// capped.  Throttle: the hysteresis levels of cpu_service.cpp:221-247 on the
// hottest die of each stack: Light and Severe stretch die op times, Shutdown
// admits nothing before the end of the next epoch.
__global__ void controller_kernel(ControllerArgs a)
{
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (tid < a.stacks) {
        const int s = tid;
        double hot = 0.0;
        for (int g = s; g < a.channels_total; g += a.stacks)
            for (int d = 0; d < a.dies; ++d) hot = fmax(hot, a.die_temp[g * a.dies + d]);
        const double th[3] = {a.light_k, a.severe_k, a.shutdown_k};
        const unsigned applied = a.level[s];
        unsigned desired = 0;
        for (int k = 0; k < 3; ++k)
            if (hot >= th[k]) ++desired;
        if (desired < applied && hot >= th[applied - 1] - a.hysteresis_k) desired = applied;
        a.level[s] = desired;
        a.throttle[s] = desired == 1 ? a.light_permille : desired >= 2 ? a.severe_permille : 1000u;
        a.admit[s] = desired == 3 ? a.next_epoch_end : 0ull;
    }
    __syncthreads();  // single block: stacks done before channels read them
    for (int c = tid; c < a.local_channels; c += blockDim.x * gridDim.x) {
        const int g = c * a.shard_count + a.shard_rank;
        unsigned long long total = 0;
        if (g < a.channels_total) {
            for (int d = 0; d < a.dies; ++d) {
                const double t = a.die_temp[g * a.dies + d];
                unsigned long long share = a.base_permille;
                if (t >= a.onset_k) {
                    const double k = floor((t - a.onset_k) / a.step_k);
                    const int kk = k > 20.0 ? 20 : static_cast<int>(k);
                    share <<= kk;
                }
                total += share;
            }
            total /= static_cast<unsigned long long>(a.dies);
        }
        const unsigned r = static_cast<unsigned>(total < a.cap_permille ? total : a.cap_permille);
        a.refresh[c] = r;
        std::uint64_t eff = static_cast<std::uint64_t>(
            (static_cast<unsigned __int128>(a.chan_bw_nominal) * (1000u - r)) / 1000u);
        a.chan_bw[c] = eff ? eff : 1;
        const int stack = g < a.channels_total ? g % a.stacks : 0;
        const unsigned thr = a.throttle[stack];
        const std::uint64_t tr = (static_cast<unsigned __int128>(a.read_latency) * thr + 999) / 1000;
        const std::uint64_t tp = (static_cast<unsigned __int128>(a.program_latency) * thr + 999) / 1000;
        a.t_read[c] = static_cast<i64>(sat_mul_dev(tr, a.time_scale));
        a.t_prog[c] = static_cast<i64>(sat_mul_dev(tp, a.time_scale));
        a.t_admit[c] = static_cast<i64>(a.admit[stack]);
    }
    for (int k = tid; k < a.act_words; k += blockDim.x * gridDim.x) {
        a.act_read[k] = 0;
        a.act_write[k] = 0;
    }
}

template <typename T>
cudaError_t alloc(T** p, std::uint64_t n)
{
    return cudaMalloc(reinterpret_cast<void**>(p), sizeof(T) * (n ? n : 1));
}

bool finite_pos(double v) { return std::isfinite(v) && v > 0.0; }

}  // namespace
}  // namespace hbfb

using namespace hbfb;

namespace {

int advance(hbfsim_context* c, double epoch_s, const unsigned long long* rb,
            const unsigned long long* wr, cudaStream_t s)
{
    ThermalState* t = c->thermal;
    if (!t) return HBFSIM_INVALID_ARGUMENT;
    if (!(epoch_s > 0.0) || !std::isfinite(epoch_s)) return HBFSIM_INVALID_ARGUMENT;
    const double dt = epoch_s;
    const int plane = t->nx * t->ny;
    const auto& cfg = t->cfg;
    auto hooks = c->hooks();
    hooks(kSlotThermal, 0, s);
    rhs_kernel<<<static_cast<unsigned>((t->cells + 255) / 256), 256, 0, s>>>(
        t->d_t, t->d_cell_die, rb, wr, cfg.die_idle_w, cfg.read_j_per_byte,
        cfg.write_j_per_access, t->d_die_cells, t->d_cap, t->d_gb, t->d_tb, plane,
        static_cast<long long>(t->cells), dt, t->d_w0);
    // forward: W1 = W0 Qx (rows = nz*ny), then W0_z = Qy^T W1_z
    dgemm(t->nz * t->ny, t->nx, t->nx, t->d_w0, 0, 0, t->d_qx, 0, 0, t->d_w1, 0, 1, s);
    dgemm(t->ny, t->nx, t->ny, t->d_qy, 0, 1, t->d_w1, plane, 0, t->d_w0, plane, t->nz, s);
    tridiag_kernel<<<(plane + 127) / 128, 128, 0, s>>>(t->d_w0, t->nx, t->ny, t->nz, t->d_cap,
                                                       t->d_gb, t->d_gx, t->d_gy, t->d_gz,
                                                       t->d_lx, t->d_ly, dt, t->d_w1);
    // inverse: W0_z = Qy W1_z, then T = W0 Qx^T
    dgemm(t->ny, t->nx, t->ny, t->d_qy, 0, 0, t->d_w1, plane, 0, t->d_w0, plane, t->nz, s);
    dgemm(t->nz * t->ny, t->nx, t->nx, t->d_w0, 0, 0, t->d_qx, 0, 1, t->d_t, 0, 1, s);
    die_temp_kernel<<<t->dies_total, 256, 0, s>>>(t->d_t, t->d_die_start, t->d_die_list,
                                                   static_cast<int>(t->dies_total),
                                                   t->d_die_cells, t->d_die_temp);
    hooks(kSlotThermal, 1, s);
    t->epoch_end_ns += static_cast<std::uint64_t>(std::llround(epoch_s * 1e9));
    ++t->epochs;
    ControllerArgs a{};
    a.die_temp = t->d_die_temp;
    a.dies = static_cast<int>(c->D);
    a.channels_total = static_cast<int>(c->channels_total);
    a.stacks = static_cast<int>(c->stacks);
    a.local_channels = static_cast<int>(c->C);
    a.shard_rank = static_cast<int>(c->shard_rank);
    a.shard_count = static_cast<int>(c->shard_count);
    a.onset_k = cfg.refresh_onset_k;
    a.step_k = cfg.refresh_step_k;
    a.base_permille = cfg.refresh_base_permille;
    a.cap_permille = cfg.refresh_cap_permille;
    a.light_k = cfg.light_k;
    a.severe_k = cfg.severe_k;
    a.shutdown_k = cfg.shutdown_k;
    a.hysteresis_k = cfg.hysteresis_k;
    a.light_permille = cfg.light_permille;
    a.severe_permille = cfg.severe_permille;
    a.next_epoch_end = t->epoch_end_ns + static_cast<std::uint64_t>(std::llround(epoch_s * 1e9));
    a.level = t->d_level;
    a.refresh = t->d_refresh;
    a.throttle = t->d_throttle;
    a.admit = t->d_admit;
    a.chan_bw_nominal = channel_bandwidth(c->profile);
    a.chan_bw = c->d_chan_bw;
    a.t_read = c->d_t_read;
    a.t_prog = c->d_t_prog;
    a.t_admit = c->d_admit;
    a.read_latency = c->profile.read_latency_ns;
    a.program_latency = c->profile.program_latency_ns;
    a.time_scale = c->profile.time_scale;
    a.act_read = c->d_die_read_bytes;
    a.act_write = c->d_die_writes;
    a.act_words = static_cast<int>(static_cast<std::uint64_t>(c->C) * std::max(1u, c->D));
    hooks(kSlotController, 0, s);
    controller_kernel<<<1, 1024, 0, s>>>(a);
    hooks(kSlotController, 1, s);
    // the admission tick bound used by the host's path choice
    t->admit_bound = std::max<std::uint64_t>(t->admit_bound, a.next_epoch_end);
    c->admit_max = std::max<std::uint64_t>(c->admit_max, t->admit_bound);
    return cudaGetLastError() == cudaSuccess ? HBFSIM_OK : HBFSIM_CUDA_ERROR;
}

struct TGuard {
    explicit TGuard(hbfsim_context* c) : lock(c->mu) { cudaSetDevice(c->device); }
    std::lock_guard<std::mutex> lock;
};

}  // namespace

extern "C" {

int hbfsim_thermal_configure_v1(hbfsim_context* c, const hbfsim_thermal_config_v1* cfg)
{
    if (!c || !cfg || cfg->struct_size != sizeof(hbfsim_thermal_config_v1) ||
        cfg->version != HBFSIM_THERMAL_CONFIG_V1_VERSION)
        return HBFSIM_INVALID_ARGUMENT;
    if (c->mode != HBFSIM_MODEL_DIE_V1) return HBFSIM_UNSUPPORTED;
    const auto& f = *cfg;
    if (f.nx == 0 || f.ny == 0 || f.nx > 4096 || f.ny > 4096 || f.layer_count == 0 ||
        f.layer_count > HBFSIM_THERMAL_MAX_LAYERS || !finite_pos(f.cell_m) ||
        !finite_pos(f.initial_k) || !finite_pos(f.bottom_ambient_k) ||
        !finite_pos(f.top_ambient_k) || !(f.bottom_h_w_m2_k >= 0) || !(f.top_h_w_m2_k >= 0) ||
        !(f.die_idle_w >= 0) || !(f.read_j_per_byte >= 0) || !(f.write_j_per_access >= 0) ||
        !finite_pos(f.refresh_step_k) || f.refresh_cap_permille > 999 ||
        f.light_permille < 1000 || f.severe_permille < 1000 || !(f.hysteresis_k >= 0) ||
        !f.die_z0 || !f.die_z_count || !f.die_x0 || !f.die_x1 || !f.die_y0 || !f.die_y1)
        return HBFSIM_INVALID_ARGUMENT;
    for (std::uint32_t z = 0; z < f.layer_count; ++z) {
        const auto& l = f.layers[z];
        if (!finite_pos(l.thickness_m) || !finite_pos(l.cv_j_m3_k) ||
            !finite_pos(l.k_xyz_w_m_k[0]) || !finite_pos(l.k_xyz_w_m_k[1]) ||
            !finite_pos(l.k_xyz_w_m_k[2]))
            return HBFSIM_INVALID_ARGUMENT;
    }
    TGuard g(c);
    const int nx = static_cast<int>(f.nx), ny = static_cast<int>(f.ny),
              nz = static_cast<int>(f.layer_count);
    const std::uint64_t plane = static_cast<std::uint64_t>(nx) * ny;
    const std::uint64_t cells = plane * nz;
    const std::uint32_t dies = c->channels_total * c->D;
    // floorplan -> cell owner map
    std::vector<int> owner(cells, -1);
    std::vector<double> die_cells(dies, 0.0);
    for (std::uint32_t d = 0; d < dies; ++d) {
        const std::uint32_t z0 = f.die_z0[d], zc = f.die_z_count[d];
        if (zc == 0 || z0 + zc > f.layer_count || f.die_x0[d] >= f.die_x1[d] ||
            f.die_y0[d] >= f.die_y1[d] || f.die_x1[d] > f.nx || f.die_y1[d] > f.ny)
            return HBFSIM_INVALID_ARGUMENT;
        for (std::uint32_t z = z0; z < z0 + zc; ++z)
            for (std::uint32_t y = f.die_y0[d]; y < f.die_y1[d]; ++y)
                for (std::uint32_t x = f.die_x0[d]; x < f.die_x1[d]; ++x) {
                    int& o = owner[z * plane + static_cast<std::uint64_t>(y) * nx + x];
                    if (o >= 0) return HBFSIM_INVALID_ARGUMENT;  // overlapping dies
                    o = static_cast<int>(d);
                    die_cells[d] += 1.0;
                }
    }
    // coefficients, as tools/eq3_layered_export.py:92-114 builds them
    const double cell = f.cell_m;
    std::vector<double> cap(nz), gb(nz), tb(nz), gx(nz), gy(nz);
    std::vector<double> gzv(static_cast<std::size_t>(nz > 1 ? nz - 1 : 1), 0.0);
    for (int z = 0; z < nz; ++z) {
        const auto& l = f.layers[z];
        const double dz = l.thickness_m;
        cap[z] = (cell * cell * dz) * l.cv_j_m3_k;
        // lateral: area (cell*dz) / (cell/(2k) + cell/(2k))
        gx[z] = (cell * dz) / (cell / (2 * l.k_xyz_w_m_k[0]) + cell / (2 * l.k_xyz_w_m_k[0]));
        gy[z] = (cell * dz) / (cell / (2 * l.k_xyz_w_m_k[1]) + cell / (2 * l.k_xyz_w_m_k[1]));
        if (z + 1 < nz) {
            const auto& u = f.layers[z + 1];
            gzv[z] = (cell * cell) / (dz / (2 * l.k_xyz_w_m_k[2]) +
                                      u.thickness_m / (2 * u.k_xyz_w_m_k[2]));
        }
        double conductance = 0.0, heat = 0.0;
        const double sides[2][2] = {{f.bottom_h_w_m2_k, f.bottom_ambient_k},
                                    {f.top_h_w_m2_k, f.top_ambient_k}};
        const bool on[2] = {z == 0, z == nz - 1};
        for (int k = 0; k < 2; ++k) {
            if (!on[k]) continue;
            const double h = sides[k][0];
            const double gg = h == 0 ? 0.0 : cell * cell / (dz / (2 * l.k_xyz_w_m_k[2]) + 1 / h);
            conductance += gg;
            heat += gg * sides[k][1];
        }
        gb[z] = conductance;
        tb[z] = conductance != 0.0 ? heat / conductance : f.initial_k;
    }
    // orthonormal DCT-II matrices Q[j][p] = s_p cos(pi p (j + 1/2) / n)
    auto dct = [](int n, std::vector<double>& q, std::vector<double>& lam) {
        q.assign(static_cast<std::size_t>(n) * n, 0.0);
        lam.assign(n, 0.0);
        const double pi = 3.14159265358979323846;
        for (int p = 0; p < n; ++p) {
            const double s = p == 0 ? std::sqrt(1.0 / n) : std::sqrt(2.0 / n);
            for (int j = 0; j < n; ++j) q[static_cast<std::size_t>(j) * n + p] =
                s * std::cos(pi * p * (j + 0.5) / n);
            lam[p] = 2.0 - 2.0 * std::cos(pi * p / n);
        }
    };
    std::vector<double> qx, qy, lx, ly;
    dct(nx, qx, lx);
    dct(ny, qy, ly);
    if (cudaDeviceSynchronize() != cudaSuccess) return HBFSIM_CUDA_ERROR;
    if (c->thermal) thermal_destroy(c->thermal);
    auto* t = new ThermalState();
    c->thermal = t;
    t->cfg = f;
    t->nx = nx;
    t->ny = ny;
    t->nz = nz;
    t->cells = cells;
    t->dies_total = dies;
    std::vector<double> t0(cells, f.initial_k);
    bool ok = !alloc(&t->d_cap, nz) && !alloc(&t->d_gb, nz) && !alloc(&t->d_tb, nz) &&
              !alloc(&t->d_gx, nz) && !alloc(&t->d_gy, nz) && !alloc(&t->d_gz, gzv.size()) &&
              !alloc(&t->d_lx, nx) && !alloc(&t->d_ly, ny) &&
              !alloc(&t->d_qx, static_cast<std::uint64_t>(nx) * nx) &&
              !alloc(&t->d_qy, static_cast<std::uint64_t>(ny) * ny) && !alloc(&t->d_t, cells) &&
              !alloc(&t->d_w0, cells) && !alloc(&t->d_w1, cells) &&
              !alloc(&t->d_cell_die, cells) && !alloc(&t->d_die_cells, dies) &&
              !alloc(&t->d_die_start, dies + 1ull) && !alloc(&t->d_die_list, cells) &&
              !alloc(&t->d_die_temp, dies) &&
              !alloc(&t->d_level, c->stacks) && !alloc(&t->d_refresh, c->C) &&
              !alloc(&t->d_throttle, c->stacks) && !alloc(&t->d_admit, c->stacks);
    auto up = [&](void* dst, const void* src, std::size_t bytes) {
        ok = ok && cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice) == cudaSuccess;
    };
    if (ok) {
        up(t->d_cap, cap.data(), 8 * nz);
        up(t->d_gb, gb.data(), 8 * nz);
        up(t->d_tb, tb.data(), 8 * nz);
        up(t->d_gx, gx.data(), 8 * nz);
        up(t->d_gy, gy.data(), 8 * nz);
        up(t->d_gz, gzv.data(), 8 * gzv.size());
        up(t->d_lx, lx.data(), 8 * nx);
        up(t->d_ly, ly.data(), 8 * ny);
        up(t->d_qx, qx.data(), 8 * qx.size());
        up(t->d_qy, qy.data(), 8 * qy.size());
        up(t->d_t, t0.data(), 8 * cells);
        up(t->d_cell_die, owner.data(), sizeof(int) * cells);
        // per-die cell lists, ascending cell index
        std::vector<int> start(dies + 1, 0), list;
        list.reserve(cells);
        for (std::uint64_t i = 0; i < cells; ++i)
            if (owner[i] >= 0) ++start[owner[i] + 1];
        for (std::uint32_t d = 0; d < dies; ++d) start[d + 1] += start[d];
        list.assign(static_cast<std::size_t>(start[dies]), 0);
        std::vector<int> fill(start.begin(), start.end() - 1);
        for (std::uint64_t i = 0; i < cells; ++i)
            if (owner[i] >= 0) list[fill[owner[i]]++] = static_cast<int>(i);
        up(t->d_die_start, start.data(), sizeof(int) * (dies + 1));
        if (!list.empty()) up(t->d_die_list, list.data(), sizeof(int) * list.size());
        up(t->d_die_cells, die_cells.data(), 8 * dies);
        ok = ok && cudaMemset(t->d_level, 0, 4 * c->stacks) == cudaSuccess &&
             cudaMemset(t->d_die_temp, 0, 8 * dies) == cudaSuccess;
        // the factors in force until the first epoch closes
        up(t->d_refresh, c->refresh_permille.data(), 4ull * c->C);
        up(t->d_throttle, c->throttle_permille.data(), 4ull * c->stacks);
        up(t->d_admit, c->admit_after.data(), 8ull * c->stacks);
    }
    if (!ok) {
        thermal_destroy(t);
        c->thermal = nullptr;
        return HBFSIM_CUDA_ERROR;
    }
    // worst-case factor bounds for the host's choice of the parallel path
    const std::uint64_t bw = channel_bandwidth(c->profile);
    std::uint64_t eff = static_cast<std::uint64_t>(
        static_cast<unsigned __int128>(bw) * (1000u - f.refresh_cap_permille) / 1000u);
    if (!eff) eff = 1;
    const unsigned __int128 xnum =
        static_cast<unsigned __int128>(c->profile.page_bytes) * 1000000000ull;
    const std::uint64_t xw = static_cast<std::uint64_t>((xnum + eff - 1) / eff) *
                             c->profile.time_scale;
    const std::uint32_t thr = std::max(f.light_permille, f.severe_permille);
    const std::uint64_t tw =
        (static_cast<unsigned __int128>(std::max(c->profile.read_latency_ns,
                                                 c->profile.program_latency_ns)) * thr + 999) /
        1000 * c->profile.time_scale;
    t->x_bound = xw;
    t->op_bound = tw;
    c->x_max = std::max(c->x_max, xw);
    c->t_max = std::max(c->t_max, tw);
    return HBFSIM_OK;
}

int hbfsim_advance_epoch_v1(hbfsim_context* c, double epoch_s, void* stream)
{
    if (!c) return HBFSIM_INVALID_ARGUMENT;
    TGuard g(c);
    if (!c->thermal) return HBFSIM_INVALID_ARGUMENT;
    if (c->shard_count != 1) return HBFSIM_INVALID_ARGUMENT;  // needs the global activity
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    return advance(c, epoch_s, c->d_die_read_bytes, c->d_die_writes, s);
}

int hbfsim_advance_epoch_global_v1(hbfsim_context* c, double epoch_s, const uint64_t* read_bytes,
                                   const uint64_t* writes, void* stream)
{
    if (!c || !read_bytes || !writes) return HBFSIM_INVALID_ARGUMENT;
    TGuard g(c);
    if (!c->thermal) return HBFSIM_INVALID_ARGUMENT;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    return advance(c, epoch_s, reinterpret_cast<const unsigned long long*>(read_bytes),
                   reinterpret_cast<const unsigned long long*>(writes), s);
}

int hbfsim_copy_die_activity_v1(hbfsim_context* c, uint64_t* read_bytes, uint64_t* writes,
                                void* stream)
{
    if (!c || !read_bytes || !writes) return HBFSIM_INVALID_ARGUMENT;
    TGuard g(c);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    const std::uint64_t n = 8ull * c->C * std::max(1u, c->D);
    if (cudaMemcpyAsync(read_bytes, c->d_die_read_bytes, n, cudaMemcpyDeviceToDevice, s) ||
        cudaMemcpyAsync(writes, c->d_die_writes, n, cudaMemcpyDeviceToDevice, s))
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

int hbfsim_get_temperatures_v1(hbfsim_context* c, double* out, uint64_t count)
{
    if (!c || !out) return HBFSIM_INVALID_ARGUMENT;
    TGuard g(c);
    if (!c->thermal || count != c->thermal->cells) return HBFSIM_INVALID_ARGUMENT;
    if (cudaDeviceSynchronize() ||
        cudaMemcpy(out, c->thermal->d_t, 8 * count, cudaMemcpyDeviceToHost))
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

int hbfsim_get_die_temperatures_v1(hbfsim_context* c, double* out, uint64_t count)
{
    if (!c || !out) return HBFSIM_INVALID_ARGUMENT;
    TGuard g(c);
    if (!c->thermal || count != c->thermal->dies_total) return HBFSIM_INVALID_ARGUMENT;
    if (cudaDeviceSynchronize() ||
        cudaMemcpy(out, c->thermal->d_die_temp, 8 * count, cudaMemcpyDeviceToHost))
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

int hbfsim_get_thermal_factors_v1(hbfsim_context* c, uint32_t* refresh_permille,
                                  uint32_t* throttle_permille, uint64_t* admit_after_ns,
                                  uint32_t* levels)
{
    if (!c) return HBFSIM_INVALID_ARGUMENT;
    TGuard g(c);
    ThermalState* t = c->thermal;
    if (!t) return HBFSIM_INVALID_ARGUMENT;
    if (cudaDeviceSynchronize()) return HBFSIM_CUDA_ERROR;
    if ((refresh_permille &&
         cudaMemcpy(refresh_permille, t->d_refresh, 4ull * c->C, cudaMemcpyDeviceToHost)) ||
        (throttle_permille &&
         cudaMemcpy(throttle_permille, t->d_throttle, 4ull * c->stacks, cudaMemcpyDeviceToHost)) ||
        (admit_after_ns &&
         cudaMemcpy(admit_after_ns, t->d_admit, 8ull * c->stacks, cudaMemcpyDeviceToHost)) ||
        (levels && cudaMemcpy(levels, t->d_level, 4ull * c->stacks, cudaMemcpyDeviceToHost)))
        return HBFSIM_CUDA_ERROR;
    return HBFSIM_OK;
}

}  // extern "C"
