// td_probe.cuh -- measurement kernel: the rate at which all SMs gather random rows out of L2.
//
// The sampler and the fused kernel are bound by gathers of short rows (64-byte head slices, 512-byte memory rows)
// from an L2-resident buffer, so their roofline is an L2 random-row rate, which no plain copy measures. This kernel
// reads `visits` pseudo-random rows of `row_bytes` from `buf` the way the sampler reads corner rows: G lanes per row
// (16-byte loads, or 32-byte loads with kWide), kBatch rows in flight per lane, no arithmetic beyond an integer
// hash per row and an XOR fold that keeps every load live. bench.py times it with CUDA events (--l2-peak).
#pragma once

#include "td_sampler.cuh"

namespace td {

struct ProbeArgs {
    const unsigned char* buf;
    unsigned long long rows;  // rows in buf
    long long visits;         // rows read in total: a multiple of (warps in the grid) * (32 / G) * kBatch
    int row_bytes;            // power of two, 16 .. 512 (kWide: 32 .. 512)
    unsigned seed;
    uint4* sink;              // one 16-byte word per thread of the grid
};

constexpr int kProbeThreads = 256;

template <bool kWide>
__global__ void __launch_bounds__(kProbeThreads) row_gather_probe_kernel(const ProbeArgs a) {
    constexpr int kWords = kWide ? 2 : 1;
    constexpr int kBatch = kWide ? 4 : 8;
    const int word = 16 * kWords;
    const int G = a.row_bytes / word, CG = 32 / G;
    const int lane = threadIdx.x & 31, cg = lane / G, v = lane - cg * G;
    const long long warp = ((long long)blockIdx.x * kProbeThreads + threadIdx.x) >> 5;
    const long long n_warps = ((long long)gridDim.x * kProbeThreads) >> 5;
    const long long chunk = (long long)CG * kBatch;
    uint4 fold = {0u, 0u, 0u, 0u};
    for (long long base = warp * chunk; base < a.visits; base += n_warps * chunk) {
        uint4 raw[kBatch][kWords];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            // row = floor(hash(visit) * rows / 2^32) < rows
            unsigned h = unsigned(base + u * CG + cg) * 2654435761u ^ a.seed;
            h ^= h >> 15;
            h *= 2246822519u;
            h ^= h >> 13;
            const unsigned long long r = ((unsigned long long)h * a.rows) >> 32;
            ld_corner<false>(a.buf + r * (unsigned long long)a.row_bytes + v * word, raw[u]);
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
#pragma unroll
            for (int k = 0; k < kWords; ++k) {
                fold.x ^= raw[u][k].x;
                fold.y ^= raw[u][k].y;
                fold.z ^= raw[u][k].z;
                fold.w ^= raw[u][k].w;
            }
        }
    }
    a.sink[(long long)blockIdx.x * kProbeThreads + threadIdx.x] = fold;
}

}  // namespace td
