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
    double* d_qxt = nullptr;    // their transposes (row operands of the fused step)
    double* d_qyt = nullptr;
    unsigned* d_bar = nullptr;  // grid barrier word of the fused step
    bool fused = false;         // one cooperative kernel per epoch (thermal_epoch_kernel)
    int fused_grid = 0;
    std::uint32_t fused_smem = 0;
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

// After a wait error of the fused step, with no kernel running: a barrier
// that a CTA left early may hold stray arrivals.
void thermal_reset_barrier(ThermalState* t)
{
    if (t && t->d_bar) cudaMemset(t->d_bar, 0, 8);
}

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
                    static_cast<void*>(t->d_qxt), static_cast<void*>(t->d_qyt),
                    static_cast<void*>(t->d_bar),
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

// Power per cell of die d over the epoch: idle plus the epoch's read and
// write energy over dt, spread evenly over the die's cells.
__device__ __forceinline__ double cell_power(int d, const unsigned long long* rb,
                                             const unsigned long long* wr, double idle,
                                             double jpb, double jpw, double dt,
                                             const double* die_cells)
{
    const double e = static_cast<double>(rb[d]) * jpb + static_cast<double>(wr[d]) * jpw;
    return (idle + e / dt) / die_cells[d];
}

// rhs = C/dt T + P + G_b T_amb, from the layer's C/dt and G_b T_amb
__device__ __forceinline__ double rhs_value(double cdt, double t, double p, double gbtb)
{
    return cdt * t + p + gbtb;
}

__global__ void rhs_kernel(const double* t, const int* cell_die,
                           const unsigned long long* rb, const unsigned long long* wr,
                           double idle, double jpb, double jpw, const double* die_cells,
                           const double* cap, const double* gb, const double* tb, int plane,
                           long long cells, double dt, double* rhs)
{
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= cells) return;
    const int z = static_cast<int>(static_cast<unsigned>(i) / static_cast<unsigned>(plane));
    const int d = cell_die[i];
    const double p = d >= 0 ? cell_power(d, rb, wr, idle, jpb, jpw, dt, die_cells) : 0.0;
    rhs[i] = rhs_value(cap[z] / dt, t[i], p, gb[z] * tb[z]);
}

// Thomas algorithm along z for mode m = q * nx + p; nz <= 32.  base[z] =
// C_z/dt + G_b,z (the layer's diagonal before the lateral and vertical
// terms).
__device__ __forceinline__ void tridiag_mode(int m, const double* rhs, int nx, int ny, int nz,
                                             const double* base, const double* gx,
                                             const double* gy, const double* gz,
                                             const double* lx, const double* ly, double* out,
                                             bool transposed)
{
    const int plane = nx * ny;
    const int q = m / nx, p = m % nx;
    double cp[32], dp[32];
    // the mode's right-hand side first, several loads in flight
#pragma unroll 8
    for (int z = 0; z < nz; ++z) dp[z] = rhs[static_cast<long long>(z) * plane + m];
    const double lxp = lx[p], lyq = ly[q];
    double prev_c = 0.0, prev_d = 0.0;
    for (int z = 0; z < nz; ++z) {
        const double down = z > 0 ? gz[z - 1] : 0.0;
        const double up = z + 1 < nz ? gz[z] : 0.0;
        const double diag = base[z] + gx[z] * lxp + gy[z] * lyq + down + up;
        const double a = -down, c = -up;
        const double denom = diag - a * prev_c;
        const double cz = c / denom;
        const double dz = (dp[z] - a * prev_d) / denom;
        cp[z] = cz;
        dp[z] = dz;
        prev_c = cz;
        prev_d = dz;
    }
    const int at = transposed ? p * ny + q : m;  // [z][p][q] or [z][q][p]
    double x = dp[nz - 1];
    out[static_cast<long long>(nz - 1) * plane + at] = x;
    for (int z = nz - 2; z >= 0; --z) {
        x = dp[z] - cp[z] * x;
        out[static_cast<long long>(z) * plane + at] = x;
    }
}

__global__ void tridiag_kernel(const double* rhs, int nx, int ny, int nz, const double* cap,
                               const double* gb, const double* gx, const double* gy,
                               const double* gz, const double* lx, const double* ly,
                               double dt, double* out)
{
    __shared__ double base[32];
    if (threadIdx.x < nz) base[threadIdx.x] = cap[threadIdx.x] / dt + gb[threadIdx.x];
    __syncthreads();
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= nx * ny) return;
    tridiag_mode(m, rhs, nx, ny, nz, base, gx, gy, gz, lx, ly, out, false);
}

// Mean temperature of global die d over its own cell list, by one warp
// (fixed summation order: lane-strided partial sums, then a shuffle tree).
__device__ __forceinline__ void die_mean(int d, const double* t, const int* die_start,
                                         const int* die_list, const double* die_cells,
                                         double* mean_out)
{
    const int lane = threadIdx.x & 31;
    double s = 0.0;
    for (int k = die_start[d] + lane; k < die_start[d + 1]; k += 32) s += t[die_list[k]];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
    if (lane == 0) mean_out[d] = die_cells[d] > 0 ? s / die_cells[d] : 0.0;
}

constexpr int kDieWarps = 4;  // warps (dies) per CTA of die_temp_kernel

__global__ void __launch_bounds__(kDieWarps * 32) die_temp_kernel(const double* t,
                                                                const int* die_start,
                                                                const int* die_list, int dies,
                                                                const double* die_cells,
                                                                double* mean_out)
{
    const int d = blockIdx.x * kDieWarps + (threadIdx.x >> 5);
    if (d < dies) die_mean(d, t, die_start, die_list, die_cells, mean_out);
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
// One CTA (any block size) runs the whole controller.
__device__ __forceinline__ void controller_body(const ControllerArgs& a)
{
    const int tid = threadIdx.x, step = blockDim.x;
    // one warp per stack: the lanes take the stack's dies, then a max
    // across the warp (exact in any order)
    const int lane = tid & 31, warps = step >> 5;
    for (int s = tid >> 5; s < a.stacks; s += warps) {
        const int count = (a.channels_total - s + a.stacks - 1) / a.stacks * a.dies;
        double hot = 0.0;
        for (int k = lane; k < count; k += 32)
            hot = fmax(hot, a.die_temp[(s + (k / a.dies) * a.stacks) * a.dies + k % a.dies]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) hot = fmax(hot, __shfl_xor_sync(0xffffffffu, hot, o));
        if (lane) continue;
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
    __syncthreads();  // stacks done before channels read them
    for (int c = tid; c < a.local_channels; c += step) {
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
    for (int k = tid; k < a.act_words; k += step) {
        a.act_read[k] = 0;
        a.act_write[k] = 0;
    }
}

__global__ void controller_kernel(ControllerArgs a) { controller_body(a); }

// ------------------------------------------------------------ fused step
// The whole epoch close in one cooperative kernel (all CTAs resident): the
// right-hand side, the four DCT GEMMs, the tridiagonal solves, the die
// means and the controller, as phases separated by a grid barrier.  A GEMM
// tile (32 x 32 of C) stages its operands with bulk copies (cp.async.bulk,
// completion on an mbarrier): 32 rows of A and 32 columns of B, each a
// K-contiguous run in global memory, into padded shared rows; then the same
// m8n8k4 fp64 MMAs in the same k order as dgemm_kernel, so the two paths
// give the same bits.  For every operand to be K-contiguous the forward
// x-transform stores its result transposed per layer ([z][p][y]) and so
// does the tridiagonal solve ([z][p][q]); the cosine matrices come with
// their transposes.
// Waits are bounded: a barrier or an mbarrier that gives up records a wait
// error in the context's counters; the CTA then skips its remaining work but
// still arrives at every grid barrier, and its copies in flight are waited
// for (bounded) before it exits.
constexpr int kEpochThreads = 128;
constexpr u32 kWaitSpins = 1u << 24;              // polls, a second bound
constexpr unsigned long long kWaitNs = 1000000000ull;  // 1 s of device time

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

struct EpochArgs {
    // grid and coefficients
    int nx, ny, nz;
    long long cells;
    double dt;
    const double* cap; const double* gb; const double* tb;
    const double* gx; const double* gy; const double* gz;
    const double* lx; const double* ly;
    const double* qx; const double* qy; const double* qxt; const double* qyt;
    double* t; double* w0; double* w1;
    // power
    const int* cell_die;
    const unsigned long long* rb; const unsigned long long* wr;
    double idle, jpb, jpw;
    const double* die_cells;
    // die means
    const int* die_start; const int* die_list; int dies; double* die_temp;
    // barrier and errors
    unsigned* bar;
    DevCounters* counters;
    ControllerArgs ctl;
};

constexpr unsigned long long kErrWaitBit = kErrWait;

// Grid-wide barrier over gridDim.x CTAs on one word: every CTA adds 1
// except CTA 0, which adds 2^31 - (gridDim.x - 1), so each barrier flips
// the top bit once and leaves the low bits as they were; a CTA waits for the
// flip of the word it added to.  Bounded: `failed` (shared) is set when the
// wait gives up and skips the wait of later barriers (the CTA still adds).
__device__ __forceinline__ void grid_barrier(unsigned* bar, int* failed)
{
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned inc = blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1) : 1u;
        unsigned old;
        __threadfence();
        asm volatile("atom.add.release.gpu.u32 %0, [%1], %2;\n"
                     : "=r"(old) : "l"(bar), "r"(inc) : "memory");
        if (!*failed) {
            const unsigned long long t0 = global_ns();
            for (u32 spins = 0;; ++spins) {
                unsigned cur;
                asm volatile("ld.acquire.gpu.u32 %0, [%1];\n" : "=r"(cur) : "l"(bar) : "memory");
                if ((cur ^ old) & 0x80000000u) break;
                if (spins >= kWaitSpins || ((spins & 1023u) == 0 && global_ns() - t0 > kWaitNs)) {
                    *failed = 1;
                    break;
                }
            }
        }
    }
    __syncthreads();
}

__device__ __forceinline__ unsigned smem_u32(const void* p)
{
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes,
                                         unsigned long long* mbar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(mbar))
        : "memory");
}

__device__ __forceinline__ void mbar_expect(unsigned long long* mbar, unsigned bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n"
                 ::"r"(smem_u32(mbar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_wait(unsigned long long* mbar, unsigned parity)
{
    const unsigned long long t0 = global_ns();
    for (u32 i = 0; i < kWaitSpins && global_ns() - t0 <= kWaitNs; ++i) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done) : "r"(smem_u32(mbar)), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}

// Padded shared row of a staged A row (doubles): a stride of 4 mod 8
// doubles keeps the fragment loads free of bank conflicts.
__host__ __device__ inline int a_row(int K) { return K % 8 == 0 ? K + 4 : K + 8; }

struct EpochGemm {
    int M, N, K, batch;
    const double* A; long long sa;   // [M][K] per batch entry
    const double* Bt; long long sb;  // B transposed: [N][K]
    double* C; long long sc;
    int mz; long long mstride;       // transposed store: C(m, n) at
    bool transposed;                 //   (m / mz) * mstride + n * mz + m % mz, else m * N + n
    bool const_a;                    // A (else Bt) is a cosine matrix, the same for each entry
};

struct EpochTile {
    int z, m0, n0, rows, cols;
};

__device__ __forceinline__ int epoch_tiles(const EpochGemm& g)
{
    return ((g.M + kBM - 1) / kBM) * ((g.N + kBN - 1) / kBN) * g.batch;
}

__device__ __forceinline__ EpochTile epoch_tile(const EpochGemm& g, int tile)
{
    const int tm = (g.M + kBM - 1) / kBM, tn = (g.N + kBN - 1) / kBN;
    EpochTile t;
    t.z = tile / (tm * tn);
    const int r = tile % (tm * tn);
    t.m0 = (r / tn) * kBM;
    t.n0 = (r % tn) * kBN;
    t.rows = min(kBM, g.M - t.m0);
    t.cols = min(kBN, g.N - t.n0);
    return t;
}

// Threads 0..n-1 each copy one K-contiguous row of the tile's constant
// (cosine) panel or of its data panel into padded shared rows.
__device__ __forceinline__ void copy_panel(const EpochGemm& g, const EpochTile& t, bool constant,
                                           double* slot, unsigned long long* bar, int thread)
{
    const bool is_a = constant == g.const_a;
    const int n = is_a ? t.rows : t.cols;
    if (thread < 0 || thread >= n) return;
    const double* src = is_a ? g.A + g.sa * t.z + static_cast<long long>(t.m0 + thread) * g.K
                             : g.Bt + g.sb * t.z + static_cast<long long>(t.n0 + thread) * g.K;
    asm volatile("fence.proxy.async.global;\n" ::: "memory");
    bulk_g2s(slot + static_cast<long long>(thread) * a_row(g.K), src, 8u * g.K, bar);
}

__device__ __forceinline__ int panel_rows(const EpochGemm& g, const EpochTile& t, bool constant)
{
    return constant == g.const_a ? t.rows : t.cols;
}

struct EpochSync {
    unsigned long long* cbar;  // one-shot barrier of this phase's prefetched constant panel
    unsigned long long* dbar;  // data barrier
    unsigned* dphase;          // completions of dbar so far
    int* pending;              // copies on dbar in flight
    int* cpend;                // bit p: the constant panel of phase p in flight
    int bit;
    int* failed;
};

// C = A B over all tiles, CTA-strided.  The CTA's first tile finds its
// constant panel in `cslot`, prefetched at the kernel's start; later tiles
// copy it there with the data panel.
__device__ void epoch_gemm(const EpochGemm& g, double* cslot, double* dslot, const EpochSync& y)
{
    const int tiles = epoch_tiles(g);
    const int SA = a_row(g.K);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gg = lane >> 2, t4 = lane & 3;
    const int wm = (warp >> 1) * 16, wn = (warp & 1) * 16;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        if (*y.failed) return;
        const EpochTile t = epoch_tile(g, tile);
        const bool first = tile == static_cast<int>(blockIdx.x);
        if (tid == 0) {
            *y.pending = 1;
            const int n = panel_rows(g, t, false) + (first ? 0 : panel_rows(g, t, true));
            mbar_expect(y.dbar, static_cast<unsigned>(8 * g.K * n));
        }
        copy_panel(g, t, false, dslot, y.dbar, tid);
        if (!first) copy_panel(g, t, true, cslot, y.dbar, tid - kBM);
        bool ok = true;
        if (first) {
            ok = mbar_wait(y.cbar, 0u);
            if (ok && tid == 0) *y.cpend &= ~(1 << y.bit);
        }
        ok = mbar_wait(y.dbar, *y.dphase & 1u) && ok;
        if (!ok) *y.failed = 1;  // benign race: every writer stores 1
        __syncthreads();
        if (*y.failed) return;  // the kernel's end waits out these copies
        if (tid == 0) *y.pending = 0;
        ++*y.dphase;
        const double* as = g.const_a ? cslot : dslot;
        const double* bs = g.const_a ? dslot : cslot;
        double acc[2][2][2];
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int j = 0; j < 2; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;
        const double* pa = as + (wm + gg) * SA + t4;
        const double* pb = bs + (wn + gg) * SA + t4;
        for (int kk = 0; kk < g.K; kk += 4) {
            double fa[2], fb[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) fa[i] = pa[i * 8 * SA + kk];
#pragma unroll
            for (int j = 0; j < 2; ++j) fb[j] = pb[j * 8 * SA + kk];
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j) dmma_8x8x4(acc[i][j][0], acc[i][j][1], fa[i], fb[j]);
        }
        double* c = g.C + g.sc * t.z;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int row = wm + i * 8 + gg;
            if (row >= t.rows) continue;
            const int m = t.m0 + row;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int col = wn + j * 8 + 2 * t4 + h;
                    if (col >= t.cols) continue;
                    const int n = t.n0 + col;
                    const long long at = g.transposed
                        ? static_cast<long long>(m / g.mz) * g.mstride +
                              static_cast<long long>(n) * g.mz + m % g.mz
                        : static_cast<long long>(m) * g.N + n;
                    c[at] = acc[i][j][h];
                }
            }
        }
        __syncthreads();  // every warp is done with the staged panels before the next copies
    }
}

// dynamic shared memory of thermal_epoch_kernel: the per-die cell power,
// then 4 constant panels and 1 data panel of 32 padded rows
__host__ __device__ inline std::uint64_t epoch_power_words(int dies) { return (dies + 1) & ~1; }
__host__ __device__ inline std::uint64_t epoch_smem_bytes(int dies, int kmax)
{
    return 8 * (epoch_power_words(dies) + 5ull * kBM * a_row(kmax));
}

__global__ void __launch_bounds__(kEpochThreads) thermal_epoch_kernel(const EpochArgs e)
{
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ unsigned long long dbar, cbar[4];
    __shared__ int failed, pending, cpend;
    __shared__ double cdt[32], gbtb[32], base[32];  // per layer
    const int tid = threadIdx.x;
    const int Kmax = e.nx > e.ny ? e.nx : e.ny;
    const int panel = kBM * a_row(Kmax);
    double* power = reinterpret_cast<double*>(smem);
    double* cslot = power + epoch_power_words(e.dies);
    double* dslot = cslot + 4 * panel;
    const int plane = e.nx * e.ny;
    const EpochGemm gemm[4] = {
        // 1. W1T_z = (W0 Qx)^T per z: rows (z, y), columns p, stored [z][p][y]
        {e.nz * e.ny, e.nx, e.nx, 1, e.w0, 0, e.qxt, 0, e.w1, 0, e.ny, plane, true, false},
        // 2. W0_z = Qy^T W1_z  (B^T = W1T_z), stored [z][q][p]
        {e.ny, e.nx, e.ny, e.nz, e.qyt, 0, e.w1, plane, e.w0, plane, 0, 0, false, true},
        // 4. W0_z = Qy W1_z  (B^T = the transposed solution), stored [z][y][p]
        {e.ny, e.nx, e.ny, e.nz, e.qy, 0, e.w1, plane, e.w0, plane, 0, 0, false, true},
        // 5. T = W0 Qx^T  (B^T = Qx)
        {e.nz * e.ny, e.nx, e.nx, 1, e.w0, 0, e.qx, 0, e.t, 0, 0, 0, false, false}};
    if (tid == 0) {
        failed = 0;
        pending = 0;
        cpend = 0;
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_u32(&dbar)) : "memory");
        for (int p = 0; p < 4; ++p)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_u32(&cbar[p]))
                         : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    // the constant panels of this CTA's first tile of each GEMM, in flight
    // during the right-hand side
    for (int p = 0; p < 4; ++p) {
        if (static_cast<int>(blockIdx.x) >= epoch_tiles(gemm[p])) continue;
        const EpochTile t = epoch_tile(gemm[p], blockIdx.x);
        if (tid == 0) {
            cpend |= 1 << p;
            mbar_expect(&cbar[p], static_cast<unsigned>(8 * gemm[p].K *
                                                        panel_rows(gemm[p], t, true)));
        }
        copy_panel(gemm[p], t, true, cslot + p * panel, &cbar[p], tid);
    }
    // per-layer terms and per-die power
    if (tid < e.nz) {
        cdt[tid] = e.cap[tid] / e.dt;
        gbtb[tid] = e.gb[tid] * e.tb[tid];
        base[tid] = e.cap[tid] / e.dt + e.gb[tid];
    }
    for (int d = tid; d < e.dies; d += kEpochThreads)
        power[d] = cell_power(d, e.rb, e.wr, e.idle, e.jpb, e.jpw, e.dt, e.die_cells);
    __syncthreads();
    unsigned dphase = 0;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long gtid = static_cast<long long>(blockIdx.x) * blockDim.x + tid;
    auto fence_out = [] { asm volatile("fence.proxy.async.global;\n" ::: "memory"); };
    auto sync_of = [&](int p) {
        return EpochSync{&cbar[p], &dbar, &dphase, &pending, &cpend, p, &failed};
    };
    // 0. right-hand side into w0
#pragma unroll 4
    for (long long i = gtid; i < e.cells; i += stride) {
        const int z = static_cast<int>(static_cast<unsigned>(i) / static_cast<unsigned>(plane));
        const int d = e.cell_die[i];
        e.w0[i] = rhs_value(cdt[z], e.t[i], d >= 0 ? power[d] : 0.0, gbtb[z]);
    }
    fence_out();
    grid_barrier(e.bar, &failed);
    epoch_gemm(gemm[0], cslot, dslot, sync_of(0));
    fence_out();
    grid_barrier(e.bar, &failed);
    epoch_gemm(gemm[1], cslot + panel, dslot, sync_of(1));
    grid_barrier(e.bar, &failed);
    // 3. one tridiagonal solve along z per mode, into w1 stored [z][p][q]
    if (!failed)
        for (long long m = gtid; m < plane; m += stride)
            tridiag_mode(static_cast<int>(m), e.w0, e.nx, e.ny, e.nz, base, e.gx, e.gy, e.gz,
                         e.lx, e.ly, e.w1, true);
    fence_out();
    grid_barrier(e.bar, &failed);
    epoch_gemm(gemm[2], cslot + 2 * panel, dslot, sync_of(2));
    fence_out();
    grid_barrier(e.bar, &failed);
    epoch_gemm(gemm[3], cslot + 3 * panel, dslot, sync_of(3));
    grid_barrier(e.bar, &failed);
    // 6. die means
    if (!failed) {
        const int warps = kEpochThreads / 32;
        for (int d = blockIdx.x * warps + (tid >> 5); d < e.dies; d += gridDim.x * warps)
            die_mean(d, e.t, e.die_start, e.die_list, e.die_cells, e.die_temp);
    }
    grid_barrier(e.bar, &failed);
    // 7. the controller, on CTA 0
    if (blockIdx.x == 0 && !failed) controller_body(e.ctl);
    __syncthreads();
    if (failed) {
        // copies still in flight may land: wait for them (bounded)
        if (tid == 0) {
            if (pending) mbar_wait(&dbar, dphase & 1u);
            for (int p = 0; p < 4; ++p)
                if (cpend & (1 << p)) mbar_wait(&cbar[p], 0u);
            atomicAdd(&e.counters->errors, 1ull);
            atomicOr(&e.counters->error_code, kErrWaitBit);
        }
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

// The controller's arguments for the epoch that closes now (the factors it
// derives hold until the end of the next one).
ControllerArgs controller_args(hbfsim_context* c, ThermalState* t, double epoch_s)
{
    const auto& cfg = t->cfg;
    const std::uint64_t epoch_ns = static_cast<std::uint64_t>(std::llround(epoch_s * 1e9));
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
    a.next_epoch_end = t->epoch_end_ns + 2 * epoch_ns;
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
    return a;
}

// Host bookkeeping of a launched epoch close.
void commit_epoch(hbfsim_context* c, ThermalState* t, const ControllerArgs& a, double epoch_s)
{
    t->epoch_end_ns += static_cast<std::uint64_t>(std::llround(epoch_s * 1e9));
    ++t->epochs;
    // the admission tick bound used by the host's path choice
    t->admit_bound = std::max<std::uint64_t>(t->admit_bound, a.next_epoch_end);
    c->admit_max = std::max<std::uint64_t>(c->admit_max, t->admit_bound);
}

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
    ControllerArgs a = controller_args(c, t, epoch_s);
    if (t->fused) {
        EpochArgs e{};
        e.nx = t->nx;
        e.ny = t->ny;
        e.nz = t->nz;
        e.cells = static_cast<long long>(t->cells);
        e.dt = dt;
        e.cap = t->d_cap;
        e.gb = t->d_gb;
        e.tb = t->d_tb;
        e.gx = t->d_gx;
        e.gy = t->d_gy;
        e.gz = t->d_gz;
        e.lx = t->d_lx;
        e.ly = t->d_ly;
        e.qx = t->d_qx;
        e.qy = t->d_qy;
        e.qxt = t->d_qxt;
        e.qyt = t->d_qyt;
        e.t = t->d_t;
        e.w0 = t->d_w0;
        e.w1 = t->d_w1;
        e.cell_die = t->d_cell_die;
        e.rb = rb;
        e.wr = wr;
        e.idle = cfg.die_idle_w;
        e.jpb = cfg.read_j_per_byte;
        e.jpw = cfg.write_j_per_access;
        e.die_cells = t->d_die_cells;
        e.die_start = t->d_die_start;
        e.die_list = t->d_die_list;
        e.dies = static_cast<int>(t->dies_total);
        e.die_temp = t->d_die_temp;
        e.bar = t->d_bar;
        e.counters = c->d_counters;
        e.ctl = a;
        cudaLaunchConfig_t lc{};
        lc.gridDim = dim3(static_cast<unsigned>(t->fused_grid));
        lc.blockDim = dim3(kEpochThreads);
        lc.dynamicSmemBytes = t->fused_smem;
        lc.stream = s;
        cudaLaunchAttribute attr{};
        attr.id = cudaLaunchAttributeCooperative;
        attr.val.cooperative = 1;
        lc.attrs = &attr;
        lc.numAttrs = 1;
        hooks(kSlotThermal, 0, s);
        const cudaError_t le = cudaLaunchKernelEx(&lc, thermal_epoch_kernel, e);
        hooks(kSlotThermal, 1, s);
        if (le != cudaSuccess) return HBFSIM_CUDA_ERROR;
        commit_epoch(c, t, a, epoch_s);
        return HBFSIM_OK;
    }
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
    die_temp_kernel<<<(t->dies_total + kDieWarps - 1) / kDieWarps, kDieWarps * 32, 0, s>>>(
        t->d_t, t->d_die_start, t->d_die_list, static_cast<int>(t->dies_total), t->d_die_cells,
        t->d_die_temp);
    hooks(kSlotThermal, 1, s);
    hooks(kSlotController, 0, s);
    controller_kernel<<<1, 1024, 0, s>>>(a);
    hooks(kSlotController, 1, s);
    commit_epoch(c, t, a, epoch_s);
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
              !alloc(&t->d_qy, static_cast<std::uint64_t>(ny) * ny) &&
              !alloc(&t->d_qxt, static_cast<std::uint64_t>(nx) * nx) &&
              !alloc(&t->d_qyt, static_cast<std::uint64_t>(ny) * ny) && !alloc(&t->d_bar, 2) &&
              !alloc(&t->d_t, cells) &&
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
        auto transpose = [](const std::vector<double>& q, int n) {
            std::vector<double> r(q.size());
            for (int i = 0; i < n; ++i)
                for (int j = 0; j < n; ++j)
                    r[static_cast<std::size_t>(j) * n + i] = q[static_cast<std::size_t>(i) * n + j];
            return r;
        };
        const std::vector<double> qxt = transpose(qx, nx), qyt = transpose(qy, ny);
        up(t->d_qxt, qxt.data(), 8 * qxt.size());
        up(t->d_qyt, qyt.data(), 8 * qyt.size());
        ok = ok && cudaMemset(t->d_bar, 0, 8) == cudaSuccess;
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
    // the fused epoch close: one cooperative grid of one CTA per SM, when the
    // grid's sides are multiples of 4 (whole MMA k steps, 16-byte bulk rows),
    // its panels and per-die power fit shared memory (sides up to about 150
    // cells) and the device co-schedules the grid
    {
        const int kmax = std::max(nx, ny);
        const std::uint64_t smem64 = epoch_smem_bytes(static_cast<int>(dies), kmax);
        const std::uint32_t smem = static_cast<std::uint32_t>(smem64);
        int coop = 0, sms = 0, per_sm = 0;
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c->device);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->device);
        const bool shape = nx % 4 == 0 && ny % 4 == 0 && smem64 <= 220 * 1024;
        if (coop && shape &&
            cudaFuncSetAttribute(thermal_epoch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)) == cudaSuccess &&
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, thermal_epoch_kernel,
                                                          kEpochThreads, smem) == cudaSuccess &&
            per_sm >= 1 && sms > 0) {
            t->fused = true;
            t->fused_grid = sms;
            t->fused_smem = smem;
        }
        cudaGetLastError();  // a refused attribute leaves the multi-kernel path
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
