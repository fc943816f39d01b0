// td_backward.cuh -- gradients of the sampling half: d out / d (value, sampling_locations, attention_weights).
//
// For out[b,q,h,:] = sum over (l, p) of a * sum over corners c of w_c * value[b, tok_c, h, :] (bilinear weights
// w_c = (dx ? fx : 1 - fx) * (dy ? fy : 1 - fy) of x = loc_x * w_l - 0.5 clamped to [-2, w_l + 1], zero outside the
// map and on padded tokens) and g = grad_out[b,q,h,:], with d_c = <g, value[b, tok_c, h, :]>:
//   grad_value[b, tok_c, h, :] += a * w_c * g                            (scatter: float atomics)
//   grad_attention_weights     = sum_c w_c * d_c
//   grad_sampling_locations.x  = a * w_l * sum_c (dx ? 1 : -1) * (dy ? fy : 1 - fy) * d_c      (d x / d loc = w_l)
//   grad_sampling_locations.y  = a * h_l * sum_c (dy ? 1 : -1) * (dx ? fx : 1 - fx) * d_c
// which is what autograd computes through upstream's reference (reference.py:29-40: grid_sample with
// align_corners=False, zero padding). Upstream's CUDA operator has no backward.
//
// Unlike the forward, nothing here sums over a row's points: every point's gradients depend on its own four corners
// only. The vector kernel therefore gives each point a group of G lanes (G = D * sizeof(T) / 16, one 16-byte slice
// of a D-row each); the scatter into grad_value (float32 -- float64 for float64 inputs -- [B, N, H * D]) uses
// 16-byte vector atomics. The generic kernel (any D or alignment) keeps one warp per (b, q, h) row with lanes over
// D, the row's corners in shared memory, and one warp-wide sum per corner row.
#pragma once

#include "td_common.cuh"
#include "td_ptx.cuh"
#include "td_sampler.cuh"

namespace td {

template <typename T>
struct BackArgs {
    const T* value;                       // element (b, token, head, d) at b*s_img + token*s_tok + head*s_head + d
    long long s_img, s_tok, s_head;
    const T* loc;                         // [B, Q, H, L, P, 2]
    const T* attn;                        // [B, Q, H, L, P]
    const T* grad_out;                    // [B, Q, H * D]
    typename Coord<T>::type* grad_value;  // [B, N, H * D], accumulated
    T* grad_loc;                          // [B, Q, H, L, P, 2]
    T* grad_attn;                         // [B, Q, H, L, P]
    const int64_t* shapes;
    const int64_t* starts;
    const uint8_t* mask;                  // value padding mask [B, N] or null
    long long rows;                       // B * Q * H
    long long n_tok;
    int Q, H, D, L, P;
    int G;                                // lanes per corner row (vector kernel)
};

constexpr int kBackWarps = 8;

// per warp: S corner tokens, S bilinear weights, S scatter coefficients (a * w), S dot products
template <typename T>
__host__ __device__ inline size_t backward_smem(int L, int P) {
    return size_t(kBackWarps) * 4 * L * P * (sizeof(int) + 3 * sizeof(typename Coord<T>::type));
}

// The corners of point j of row `row` (bilinear weights without the attention weight) into s_tok / s_wt, the
// scatter coefficients a * w into s_coef; returns the point's attention weight and fractions for the last step.
template <typename T>
__device__ __forceinline__ void backward_point(const BackArgs<T>& a, long long row, int j, const uint8_t* mask_b,
                                               int* s_tok, typename Coord<T>::type* s_wt,
                                               typename Coord<T>::type* s_coef, typename Coord<T>::type& att,
                                               typename Coord<T>::type& fx, typename Coord<T>::type& fy,
                                               Level& lv) {
    using CT = typename Coord<T>::type;
    const int LP = a.L * a.P;
    lv = level_at(a.shapes, a.starts, level_of(j, a.P));
    const long long i = row * LP + j;
    const CT lx = CT(to_acc(a.loc[2 * i])), ly = CT(to_acc(a.loc[2 * i + 1]));
    att = CT(to_acc(a.attn[i]));
    corners4<CT>(lx, ly, CT(1), lv, a.n_tok, &s_tok[4 * j], &s_wt[4 * j], mask_b);
    // the same clamped pixel coordinates as corners4
    const CT x = cmin(cmax(lx * CT(lv.w) - CT(0.5), CT(-2)), CT(lv.w) + CT(1));
    const CT y = cmin(cmax(ly * CT(lv.h) - CT(0.5), CT(-2)), CT(lv.h) + CT(1));
    fx = x - cfloor(x);
    fy = y - cfloor(y);
#pragma unroll
    for (int c = 0; c < 4; ++c) s_coef[4 * j + c] = att * s_wt[4 * j + c];
}

// The two small gradients of point j from its four dot products (corner c = dx + 2 dy).
template <typename T>
__device__ __forceinline__ void backward_finish(const BackArgs<T>& a, long long row, int j,
                                                const typename Coord<T>::type* s_wt,
                                                const typename Coord<T>::type* s_dot, typename Coord<T>::type att,
                                                typename Coord<T>::type fx, typename Coord<T>::type fy,
                                                const Level& lv) {
    using CT = typename Coord<T>::type;
    const CT d0 = s_dot[4 * j], d1 = s_dot[4 * j + 1], d2 = s_dot[4 * j + 2], d3 = s_dot[4 * j + 3];
    const CT ga = s_wt[4 * j] * d0 + s_wt[4 * j + 1] * d1 + s_wt[4 * j + 2] * d2 + s_wt[4 * j + 3] * d3;
    const CT gfx = (CT(1) - fy) * (d1 - d0) + fy * (d3 - d2);
    const CT gfy = (CT(1) - fx) * (d2 - d0) + fx * (d3 - d1);
    const long long i = row * (a.L * a.P) + j;
    a.grad_attn[i] = from_acc<T>(typename Elem<T>::acc(ga));
    a.grad_loc[2 * i] = from_acc<T>(typename Elem<T>::acc(att * CT(lv.w) * gfx));
    a.grad_loc[2 * i + 1] = from_acc<T>(typename Elem<T>::acc(att * CT(lv.h) * gfy));
}

// Add V accumulators into grad_value (16-byte aligned): float4 vector atomics, or one atomic per double.
__device__ __forceinline__ void scatter_add(float* p, const float* v, int n) {
    for (int i = 0; i < n; i += 4)
        atomicAdd(reinterpret_cast<float4*>(p + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
}
__device__ __forceinline__ void scatter_add(double* p, const double* v, int n) {
    for (int i = 0; i < n; ++i) atomicAdd(p + i, v[i]);
}

// Vector kernel: D * sizeof(T) % 16 == 0, <= 512 bytes, G a power of two; value, grad_out 16-byte aligned with
// 16-byte strides; grad_value rows 16-byte aligned. The gradients of different points are independent, so here a
// group of G lanes owns one point from start to end, with no shared memory: each lane of the group loads the
// point's location and weight (one broadcast transaction per group) and its 16-byte slice of grad_out, computes the
// four corners, loads its slice of the four corner rows at once, and the group sums the four dot products by xor
// shuffles; every lane scatters its slice of a * w_c * g, and the group's first lane writes the two small
// gradients. A warp covers 32 / G consecutive points: two memory round trips per point, and many warps in flight.
template <typename T>
__global__ void __launch_bounds__(kBackWarps * 32) sample_backward_vec_kernel(const BackArgs<T> a) {
    using A = typename Elem<T>::acc;
    using CT = typename Coord<T>::type;
    constexpr int V = Elem<T>::kVec;
    grid_dependency_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.G, CG = 32 / G, cg = lane / G, v = lane - cg * G;
    const int LP = a.L * a.P;
    const long long pt = ((long long)blockIdx.x * kBackWarps + warp) * CG + cg;  // point: row * LP + j
    const bool live = pt < a.rows * LP;
    const long long row = live ? pt / LP : 0;
    const int j = int(pt - row * LP);
    const long long b = row / ((long long)a.Q * a.H);
    const int h = int(row % a.H);
    // the point's geometry, location, weight and grad_out slice, all loads issued together
    const Level lv = level_at(a.shapes, a.starts, live ? level_of(j, a.P) : 0);
    const long long i = row * LP + (live ? j : 0);
    const CT lx = live ? CT(to_acc(a.loc[2 * i])) : CT(-1e4), ly = live ? CT(to_acc(a.loc[2 * i + 1])) : CT(-1e4);
    const CT att = live ? CT(to_acc(a.attn[i])) : CT(0);
    A g[V];
    unpack16<T>(live ? *reinterpret_cast<const uint4*>(a.grad_out + row * a.D + v * V) : g_zero16, g);
    const uint8_t* mask_b = a.mask != nullptr ? a.mask + b * a.n_tok : nullptr;
    int tok[4];
    CT wt[4];
    corners4<CT>(lx, ly, CT(1), lv, a.n_tok, tok, wt, mask_b);  // a dead group's point lies outside every map
#pragma unroll
    for (int c = 0; c < 4; ++c) TD_BOUNDS_TOKEN(tok[c], a.n_tok);
    const CT x = cmin(cmax(lx * CT(lv.w) - CT(0.5), CT(-2)), CT(lv.w) + CT(1));
    const CT y = cmin(cmax(ly * CT(lv.h) - CT(0.5), CT(-2)), CT(lv.h) + CT(1));
    const CT fx = x - cfloor(x), fy = y - cfloor(y);
    // the four corner rows' slices, then the four dot products summed over the group
    const T* vb = a.value + b * a.s_img + (long long)h * a.s_head + v * V;
    uint4 raw[4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
        raw[c] = __ldg(tok[c] < 0 ? &g_zero16 : reinterpret_cast<const uint4*>(vb + (long long)tok[c] * a.s_tok));
    CT d[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        A xs[V];
        unpack16<T>(raw[c], xs);
        A dp = A(0);
#pragma unroll
        for (int k = 0; k < V; ++k) dp = fma(g[k], xs[k], dp);
        for (int o = G >> 1; o > 0; o >>= 1) dp += __shfl_xor_sync(0xffffffffu, dp, o);
        d[c] = CT(dp);
    }
    // scatter a * w_c * g into the corner rows of grad_value
    CT* gb = a.grad_value + b * (a.n_tok * (long long)a.H * a.D) + (long long)h * a.D + v * V;
    const long long g_tok = (long long)a.H * a.D;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        if (tok[c] < 0) continue;
        const CT coef = att * wt[c];
        CT add[V];
#pragma unroll
        for (int k = 0; k < V; ++k) add[k] = coef * CT(g[k]);
        scatter_add(gb + (long long)tok[c] * g_tok, add, V);
    }
    if (!live || v != 0) return;
    const CT ga = wt[0] * d[0] + wt[1] * d[1] + wt[2] * d[2] + wt[3] * d[3];
    const CT gfx = (CT(1) - fy) * (d[1] - d[0]) + fy * (d[3] - d[2]);
    const CT gfy = (CT(1) - fx) * (d[2] - d[0]) + fx * (d[3] - d[1]);
    a.grad_attn[i] = from_acc<T>(typename Elem<T>::acc(ga));
    a.grad_loc[2 * i] = from_acc<T>(typename Elem<T>::acc(att * CT(lv.w) * gfx));
    a.grad_loc[2 * i + 1] = from_acc<T>(typename Elem<T>::acc(att * CT(lv.h) * gfy));
}

// Generic kernel: lanes over D, scalar loads and atomics, one warp-wide sum per corner row.
template <typename T>
__global__ void __launch_bounds__(kBackWarps * 32) sample_backward_generic_kernel(const BackArgs<T> a) {
    using A = typename Elem<T>::acc;
    using CT = typename Coord<T>::type;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    grid_dependency_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long row = (long long)blockIdx.x * kBackWarps + warp;
    if (row >= a.rows) return;
    const int LP = a.L * a.P, S = 4 * LP;
    int* s_tok = reinterpret_cast<int*>(smem_raw) + warp * S;
    CT* s_wt = reinterpret_cast<CT*>(smem_raw + kBackWarps * S * sizeof(int)) + warp * S;
    CT* s_coef = s_wt + kBackWarps * S;
    CT* s_dot = s_coef + kBackWarps * S;
    const long long b = row / ((long long)a.Q * a.H);
    const int h = int(row % a.H);
    const uint8_t* mask_b = a.mask != nullptr ? a.mask + b * a.n_tok : nullptr;
    CT att[2], fx[2], fy[2];
    Level lv[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int j = lane + 32 * k;
        if (j < LP) backward_point<T>(a, row, j, mask_b, s_tok, s_wt, s_coef, att[k], fx[k], fy[k], lv[k]);
    }
    __syncwarp();
    const T* vb = a.value + b * a.s_img + (long long)h * a.s_head;
    CT* gb = a.grad_value + b * (a.n_tok * (long long)a.H * a.D) + (long long)h * a.D;
    const long long g_tok = (long long)a.H * a.D;
    const T* go = a.grad_out + row * a.D;
    for (int s = 0; s < S; ++s) {
        int t = s_tok[s];
        TD_BOUNDS_TOKEN(t, a.n_tok);
        A dp = A(0);
        if (t >= 0) {
            const CT coef = s_coef[s];
            for (int d = lane; d < a.D; d += 32) {
                const A gd = to_acc(go[d]);
                dp = fma(gd, to_acc(vb[(long long)t * a.s_tok + d]), dp);
                atomicAdd(gb + (long long)t * g_tok + d, coef * CT(gd));
            }
        }
        for (int o = 16; o > 0; o >>= 1) dp += __shfl_xor_sync(0xffffffffu, dp, o);
        if (lane == 0) s_dot[s] = CT(dp);
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int j = lane + 32 * k;
        if (j < LP) backward_finish<T>(a, row, j, s_wt, s_dot, att[k], fx[k], fy[k], lv[k]);
    }
}

// One pass over the float32 grad_value accumulator [rows, HD]: its rounding to the dtype (out, or none for float32)
// and its column sums, the value bias gradient (added into bias_acc, zeroed by the host). 256 threads a CTA: a
// thread owns 4 columns (HD / 4 <= 256 of them) of every (256 / (HD / 4))-th row of the CTA's block of rows;
// the CTA's partial sums meet in shared memory and leave with one atomic per column.
constexpr int kFinishThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kFinishThreads) grad_value_finish_kernel(const float* __restrict__ acc,
                                                                           T* __restrict__ out,
                                                                           float* __restrict__ bias_acc,
                                                                           long long rows, int HD,
                                                                           long long rows_per_cta) {
    __shared__ float4 s_sum[kFinishThreads];
    const int groups = HD >> 2;  // 4-column groups
    const int lanes_per_row = groups, row_step = kFinishThreads / groups;
    const int gcol = threadIdx.x % lanes_per_row, r0 = threadIdx.x / lanes_per_row;
    const bool active = r0 < row_step;
    const long long first = (long long)blockIdx.x * rows_per_cta;
    const long long last = min(first + rows_per_cta, rows);
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    if (active) {
        for (long long r = first + r0; r < last; r += row_step) {
            const float4 v = __ldcs(reinterpret_cast<const float4*>(acc + r * HD) + gcol);  // read once: streaming
            sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
            if constexpr (!std::is_same<T, float>::value) {  // four 16-bit values: one 8-byte store
                const T q[4] = {from_acc<T>(v.x), from_acc<T>(v.y), from_acc<T>(v.z), from_acc<T>(v.w)};
                *reinterpret_cast<uint2*>(out + r * HD + 4 * gcol) = *reinterpret_cast<const uint2*>(q);
            }
        }
    }
    s_sum[threadIdx.x] = sum;
    __syncthreads();
    if (bias_acc == nullptr || threadIdx.x >= groups) return;
    float4 t = s_sum[threadIdx.x];
    for (int k = 1; k < row_step; ++k) {
        const float4 u = s_sum[threadIdx.x + k * lanes_per_row];
        t.x += u.x; t.y += u.y; t.z += u.z; t.w += u.w;
    }
    atomicAdd(reinterpret_cast<float4*>(bias_acc) + threadIdx.x, t);
}

}  // namespace td
