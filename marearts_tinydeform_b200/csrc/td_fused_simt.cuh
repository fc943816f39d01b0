// td_fused_simt.cuh -- fused order on CUDA cores: gather C-wide memory rows, then project per head.
//
// For one (batch, query, head) row, bilinear sampling and the attention-weighted sum are linear in value, so
//   out[d] = sum_s w_s * (W[hD+d] . memory[t_s] + b[hD+d]) = W[hD+d] . m + b[hD+d] * sum_s w_s,
//   m = sum_s w_s * memory[t_s]                       (upstream csrc/ma_deform_fused.cu:4-14, :151-210).
// One CTA takes R consecutive queries of one (batch, head): the R x C matrix m is built in shared memory
// (warps over rows, lanes over 16-byte channel vectors), then each warp projects it with a group of 4 of the
// head's value_weight rows held in registers, so every weight element is read once per CTA.
// This is the float32 / float64 / odd-shape path; float16 / bfloat16 with tensor-core friendly shapes take the
// tcgen05 kernel in td_fused_tc.cuh.
#pragma once

#include "td_common.cuh"
#include "td_ptx.cuh"

namespace td {

template <typename T>
struct FusedArgs {
    const T* memory;
    const T* weight;
    const T* bias;  // may be null
    const T* loc;
    const T* attn;
    T* out;
    const int64_t* shapes;
    const int64_t* starts;
    long long n_tok;  // N
    const uint8_t* mask;  // value padding mask [B, N] (nonzero = padded) or null
    int B, Q, C, H, D, L, P;
    int R;            // queries per CTA (<= kFusedMaxRows)
    int q_tiles;      // ceil(Q / R)
    int vec;          // 1: memory rows are read as 16-byte vectors
};

constexpr int kFusedThreads = 256;
constexpr int kFusedWarps = kFusedThreads / 32;
constexpr int kFusedMaxRows = 16;
constexpr int kFusedDimGroup = 4;

// Dynamic shared memory: m [R][C] (accumulator type), tok [R][S], wt [R][S], wsum [R].
template <typename T>
__host__ __device__ inline size_t fused_simt_smem(int R, int C, int S) {
    using A = typename Elem<T>::acc;
    using CT = typename Coord<T>::type;
    size_t bytes = size_t(R) * C * sizeof(A);
    bytes = (bytes + 15) / 16 * 16 + size_t(R) * S * sizeof(int);
    bytes = (bytes + 15) / 16 * 16 + size_t(R) * S * sizeof(CT);
    bytes = (bytes + 15) / 16 * 16 + size_t(R) * sizeof(A);
    return bytes;
}

template <typename T>
__global__ void __launch_bounds__(kFusedThreads) fused_simt_kernel(const FusedArgs<T> a) {
    using A = typename Elem<T>::acc;
    using CT = typename Coord<T>::type;
    constexpr int V = Elem<T>::kVec;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ Level lv[kMaxLevels];

    const int LP = a.L * a.P, S = 4 * LP, C = a.C, R = a.R;
    A* m = reinterpret_cast<A*>(smem_raw);
    size_t off = (size_t(R) * C * sizeof(A) + 15) / 16 * 16;
    int* tok = reinterpret_cast<int*>(smem_raw + off);
    off = (off + size_t(R) * S * sizeof(int) + 15) / 16 * 16;
    CT* wt = reinterpret_cast<CT*>(smem_raw + off);
    off = (off + size_t(R) * S * sizeof(CT) + 15) / 16 * 16;
    A* wsum = reinterpret_cast<A*>(smem_raw + off);

    grid_dependency_wait();  // launched with programmatic dependent launch: every global access comes after this
    launch_dependents();
    // block -> (b, q-tile, h), heads fastest: the heads of one query sample around the same point, so CTAs that
    // run together read overlapping memory rows from L2.
    const int h = int(blockIdx.x % a.H);
    const long long bq = blockIdx.x / a.H;
    const int qt = int(bq % a.q_tiles), b = int(bq / a.q_tiles);
    const int q0 = qt * R;
    const int rows = min(R, a.Q - q0);

    load_levels(a.shapes, a.starts, a.L, lv);
    __syncthreads();

    // 1. corners of every (row, sample) of the tile
    for (int i = threadIdx.x; i < R * LP; i += kFusedThreads) {
        const int r = i / LP, j = i - r * LP;
        int* tk = tok + r * S + 4 * j;
        CT* w = wt + r * S + 4 * j;
        if (r < rows) {
            const long long bqh = ((long long)b * a.Q + q0 + r) * a.H + h;
            row_corners(a.loc, a.attn, lv, LP, a.P, a.n_tok, bqh, j, tk, w,
                        a.mask != nullptr ? a.mask + (long long)b * a.n_tok : nullptr);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) { tk[k] = -1; w[k] = CT(0); }
        }
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // 2. weight sums (for the bias term) and the gathered rows m
    for (int r = warp; r < R; r += kFusedWarps) {
        A s = A(0);
        for (int i = lane; i < S; i += 32) s += A(wt[r * S + i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) wsum[r] = s;
    }
    const T* mb = a.memory + (long long)b * a.n_tok * C;
    if (a.vec) {
        const int nv = C / V;
        for (int r = warp; r < rows; r += kFusedWarps) {
            const int* tk = tok + r * S;
            const CT* w = wt + r * S;
            for (int cv = lane; cv < nv; cv += 32) {
                A acc[V];
#pragma unroll
                for (int i = 0; i < V; ++i) acc[i] = A(0);
#pragma unroll 8
                for (int s = 0; s < S; ++s) {
                    int t = tk[s];
                    TD_BOUNDS_TOKEN(t, a.n_tok);
                    if (t >= 0) {
                        A x[V];
                        load16<T>(mb + (long long)t * C + cv * V, x);
                        const A ws = A(w[s]);
#pragma unroll
                        for (int i = 0; i < V; ++i) acc[i] = fma(ws, x[i], acc[i]);
                    }
                }
#pragma unroll
                for (int i = 0; i < V; ++i) m[r * C + cv * V + i] = acc[i];
            }
        }
    } else {
        for (int r = warp; r < rows; r += kFusedWarps) {
            const int* tk = tok + r * S;
            const CT* w = wt + r * S;
            for (int c = lane; c < C; c += 32) {
                A acc = A(0);
                for (int s = 0; s < S; ++s) {
                    int t = tk[s];
                    TD_BOUNDS_TOKEN(t, a.n_tok);
                    if (t >= 0) acc = fma(A(w[s]), to_acc(mb[(long long)t * C + c]), acc);
                }
                m[r * C + c] = acc;
            }
        }
    }
    __syncthreads();

    // 3. projection: warp w owns output dims [4g, 4g + 4) for g = w, w + 8, ...; lanes stride over C
    const T* wh = a.weight + (long long)h * a.D * C;
    for (int d0 = warp * kFusedDimGroup; d0 < a.D; d0 += kFusedWarps * kFusedDimGroup) {
        A acc[kFusedMaxRows][kFusedDimGroup];
#pragma unroll
        for (int r = 0; r < kFusedMaxRows; ++r)
#pragma unroll
            for (int i = 0; i < kFusedDimGroup; ++i) acc[r][i] = A(0);
        for (int c = lane; c < C; c += 32) {
            A wv[kFusedDimGroup];
#pragma unroll
            for (int i = 0; i < kFusedDimGroup; ++i)
                wv[i] = d0 + i < a.D ? to_acc(wh[(long long)(d0 + i) * C + c]) : A(0);
#pragma unroll
            for (int r = 0; r < kFusedMaxRows; ++r) {
                if (r < rows) {
                    const A mv = m[r * C + c];
#pragma unroll
                    for (int i = 0; i < kFusedDimGroup; ++i) acc[r][i] = fma(wv[i], mv, acc[r][i]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kFusedMaxRows; ++r) {
#pragma unroll
            for (int i = 0; i < kFusedDimGroup; ++i) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[r][i] += __shfl_xor_sync(0xffffffffu, acc[r][i], o);
            }
        }
        // every lane now holds every sum; lane (r * 4 + i) % 32 writes output (r, d0 + i)
#pragma unroll
        for (int r = 0; r < kFusedMaxRows; ++r) {
#pragma unroll
            for (int i = 0; i < kFusedDimGroup; ++i) {
                const int d = d0 + i;
                if (r < rows && d < a.D && ((r * kFusedDimGroup + i) & 31) == lane) {
                    A v = acc[r][i];
                    if (a.bias != nullptr) v = fma(to_acc(a.bias[h * a.D + d]), wsum[r], v);
                    const long long bqh = ((long long)b * a.Q + q0 + r) * a.H + h;
                    a.out[bqh * a.D + d] = from_acc<T>(v);
                }
            }
        }
    }
}

}  // namespace td
