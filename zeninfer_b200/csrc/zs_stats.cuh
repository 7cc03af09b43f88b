// zs_stats.cuh -- the display numbers of zeninfer's `logits` command
// (src/main.cpp:473-503) for a batch of rows: min and max of the row (as double,
// from the reference's -1e30 / 1e30 starts, NaN ignored), Z = sum over the row of
// exp(x - max) in f64, and p = exp(x - max) / Z for the top-N ids (the top-N
// itself comes from the select kernels).  Three small launches, all of them
// deterministic: per-chunk min/max, per-chunk f64 sums, then one thread per row
// adds the chunk sums in chunk order.
#pragma once

#include <math.h>
#include <stdint.h>

namespace zs {

constexpr int kStatsThreads = 256;
constexpr int kStatsChunk = 16384;  // columns per CTA

struct StatsArgs {
    const float* logits;
    int64_t ld;
    int32_t B;
    int32_t n;
    int32_t nchunk;
    float2* part_mm;   // [B][nchunk] (min, max) of each chunk, f32
    double* part_z;    // [B][nchunk]
    const int32_t* top_ids;  // [B][top_ld], the first topn of a row filled
    int32_t topn;
    int32_t top_ld;
    double* out_min;
    double* out_max;
    double* out_z;
    double* top_p;     // [B][top_ld]
};

__device__ __forceinline__ float stats_block_reduce(float v, bool is_max, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float t = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? fmaxf(v, t) : fminf(v, t);
    }
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float r = red[0];
        for (int w = 1; w < kStatsThreads / 32; ++w) r = is_max ? fmaxf(r, red[w]) : fminf(r, red[w]);
        red[kStatsThreads / 32] = r;
    }
    __syncthreads();
    const float r = red[kStatsThreads / 32];
    __syncthreads();
    return r;
}

// grid (nchunk, B): f32 min and max of each chunk (fminf/fmaxf skip NaN; a chunk
// of NaN only gives NaN, which the next step reads as "no value").
__global__ void __launch_bounds__(kStatsThreads) zs_stats_minmax_kernel(const StatsArgs a) {
    __shared__ float red[kStatsThreads / 32 + 1];
    const int c = blockIdx.x;
    for (int row = blockIdx.y; row < a.B; row += gridDim.y) {
        const float* x = a.logits + (int64_t)row * a.ld;
        const int i0 = c * kStatsChunk, i1 = min(a.n, i0 + kStatsChunk);
        float mn = __int_as_float(0x7fc00000), mx = __int_as_float(0x7fc00000);
        for (int i = i0 + threadIdx.x; i < i1; i += kStatsThreads) {
            const float v = x[i];
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
        }
        mn = stats_block_reduce(mn, false, red);
        mx = stats_block_reduce(mx, true, red);
        if (threadIdx.x == 0) a.part_mm[(int64_t)row * a.nchunk + c] = make_float2(mn, mx);
    }
}

// The row's max as the reference computes it: the largest value, or -1e30 when
// no value exceeds that start (NaN never does).  Likewise the min from 1e30.
__device__ __forceinline__ void stats_row_minmax(const StatsArgs& a, int row, double& mn,
                                                 double& mx) {
    mn = 1e30;
    mx = -1e30;
    for (int c = 0; c < a.nchunk; ++c) {
        const float2 p = a.part_mm[(int64_t)row * a.nchunk + c];
        if ((double)p.x < mn) mn = (double)p.x;  // false for NaN
        if ((double)p.y > mx) mx = (double)p.y;
    }
}

// grid (nchunk, B): f64 sum of exp(x - max) over each chunk, a fixed tree order.
__global__ void __launch_bounds__(kStatsThreads) zs_stats_z_kernel(const StatsArgs a) {
    __shared__ double red[kStatsThreads / 32];
    const int c = blockIdx.x;
    for (int row = blockIdx.y; row < a.B; row += gridDim.y) {
        double mn, mx;
        stats_row_minmax(a, row, mn, mx);
        const float* x = a.logits + (int64_t)row * a.ld;
        const int i0 = c * kStatsChunk, i1 = min(a.n, i0 + kStatsChunk);
        double s = 0.0;
        for (int i = i0 + threadIdx.x; i < i1; i += kStatsThreads) s += exp((double)x[i] - mx);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int w = 0; w < kStatsThreads / 32; ++w) t += red[w];
            a.part_z[(int64_t)row * a.nchunk + c] = t;
        }
        __syncthreads();
    }
}

// grid B, one warp: Z in chunk order, then the top-N probabilities.
__global__ void __launch_bounds__(32) zs_stats_final_kernel(const StatsArgs a) {
    const int lane = threadIdx.x;
    for (int row = blockIdx.x; row < a.B; row += gridDim.x) {
        double mn, mx;
        stats_row_minmax(a, row, mn, mx);
        double z = 0.0;
        if (lane == 0) {
            for (int c = 0; c < a.nchunk; ++c) z += a.part_z[(int64_t)row * a.nchunk + c];
            a.out_min[row] = mn;
            a.out_max[row] = mx;
            a.out_z[row] = z;
        }
        z = __shfl_sync(0xffffffffu, z, 0);
        const float* x = a.logits + (int64_t)row * a.ld;
        for (int i = lane; i < a.topn; i += 32) {
            const int32_t id = a.top_ids[(int64_t)row * a.top_ld + i];
            a.top_p[(int64_t)row * a.top_ld + i] =
                (id >= 0 && id < a.n) ? exp((double)x[id] - mx) / z : 0.0;
        }
    }
}

}  // namespace zs
