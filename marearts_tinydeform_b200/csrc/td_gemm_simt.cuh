// td_gemm_simt.cuh -- value projection on CUDA cores: value = memory @ W^T + b (the nn.Linear of the project order).
//
// Replaces the F.linear call of upstream marearts_tinydeform/__init__.py:77 for float32 (TF32 off), float64 and
// shapes the tcgen05 GEMM does not take. A 128 x 64 output tile per 256-thread CTA, 8 x 4 outputs per thread,
// K staged through shared memory in steps of 16, accumulation in float32 (float64 for float64).
// The epilogue adds the bias and writes either the nn.Linear layout [B*N, HD] or the head-major [B, H, N, D].
#pragma once

#include "td_common.cuh"
#include "td_ptx.cuh"

namespace td {

template <typename T>
struct ProjArgs {
    const T* memory;  // [M, C], M = B * N
    const T* weight;  // [HD, C]
    const T* bias;    // [HD] or null
    T* value;
    long long M, n_tok;  // M = B * N
    int C, HD, H, D;
    int head_major;
};

constexpr int kGemmBM = 128, kGemmBN = 64, kGemmBK = 16;
constexpr int kGemmThreads = 256;

// Output element (row m, column j) goes to value at this offset.
__device__ __forceinline__ long long proj_offset(long long m, int j, long long n_tok, int HD, int H, int D,
                                                  int head_major) {
    if (!head_major) return m * HD + j;
    const long long b = m / n_tok, n = m - b * n_tok;
    const int h = j / D, d = j - h * D;
    return ((b * H + h) * n_tok + n) * D + d;
}

template <typename T>
__global__ void __launch_bounds__(kGemmThreads) proj_simt_kernel(const ProjArgs<T> a) {
    using A = typename Elem<T>::acc;
    __shared__ A sa[kGemmBK][kGemmBM + 4];
    __shared__ A sb[kGemmBK][kGemmBN + 4];
    grid_dependency_wait();  // launched with programmatic dependent launch in the project order
    launch_dependents();
    const long long m0 = (long long)blockIdx.x * kGemmBM;
    const int n0 = blockIdx.y * kGemmBN;
    const int tid = threadIdx.x;
    const int tm = tid / 16, tn = tid % 16;  // 16 x 16 threads, 8 x 4 outputs each
    A acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = A(0);

    for (int k0 = 0; k0 < a.C; k0 += kGemmBK) {
        // A tile: 128 rows x 16 k (8 per thread); B tile: 64 rows x 16 k (4 per thread)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = tid + i * kGemmThreads, r = e / kGemmBK, k = e % kGemmBK;
            const long long gm = m0 + r;
            const int gk = k0 + k;
            sa[k][r] = (gm < a.M && gk < a.C) ? to_acc(a.memory[gm * a.C + gk]) : A(0);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e = tid + i * kGemmThreads, r = e / kGemmBK, k = e % kGemmBK;
            const int gn = n0 + r, gk = k0 + k;
            sb[k][r] = (gn < a.HD && gk < a.C) ? to_acc(a.weight[(long long)gn * a.C + gk]) : A(0);
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kGemmBK; ++k) {
            A av[8], bv[4];
#pragma unroll
            for (int i = 0; i < 8; ++i) av[i] = sa[k][tm + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = sb[k][tn + 16 * j];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const long long gm = m0 + tm + 16 * i;
        if (gm >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tn + 16 * j;
            if (gn >= a.HD) continue;
            A v = acc[i][j];
            if (a.bias != nullptr) v += to_acc(a.bias[gn]);
            a.value[proj_offset(gm, gn, a.n_tok, a.HD, a.H, a.D, a.head_major)] = from_acc<T>(v);
        }
    }
}

}  // namespace td
