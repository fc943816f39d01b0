// td_fused_warp.cuh -- fused order, one warp per (batch, head, query) row: gather, project, store.
//
// Computes what upstream's fused_vec computes (csrc/ma_deform_fused.cu:151-210):
//   m_r = sum_s w_s * memory[b, t_s, :]  (C wide),   out[b, q, hD + d] = W[hD + d] . m_r + bias[hD + d] * sum_s w_s
// The order's cost is the gather of C-wide corner rows out of L2 (48 rows of 512 bytes per row at the RT-DETR
// shapes in float16): its roofline is the L2 random-row gather rate, about 127 GB/s per SM on B200 for 512-byte rows
// (td_probe_row_gather). A row's work is independent of every other row's, so each warp owns one row from start to
// end, with nothing shared and no barrier beyond its own lanes:
//   * corners: lanes over the row's L x P points (one round trip for locations, weights and level geometry), the
//     4 corners of each into the warp's shared-memory list;
//   * gather: lanes over the C channels, 16-byte vectors (CV per lane: C * sizeof(T) = 512 * CV bytes), kB corner
//     rows in flight per lane (16 at CV = 1), accumulated in float32 registers -- the warp keeps 8 KB of loads in
//     flight, so the 20 warps an SM holds keep the 128+ KB in flight that the L2 rate needs;
//   * projection on CUDA cores: lane l multiplies its channels of m_r by the same channels of the head's D weight
//     rows (16-byte loads, L1-resident after the head's first row on the SM: rows are numbered head-major), giving D
//     partial sums per lane, eight outputs at a time, which three halving steps and two butterfly steps over the warp
//     (9 shuffles per eight outputs) turn into D / 32 finished outputs per lane; + bias * sum_s w_s, stored.
// The projection is 8 K multiply-adds per row at D = 32, C = 256: an eighth of the issue slots the gather's bytes
// take at the L2 rate, so the tensor cores would buy nothing here, while staging rows for them would put barriers
// back into the gather.
// CTAs are small (kFwWarps warps) so that the block scheduler spreads the rows evenly: at batch 1 every SM gets
// 16 or 17 rows in one wave.
#pragma once

#include <type_traits>

#include "td_common.cuh"
#include "td_ptx.cuh"

namespace td {

template <typename T>
struct FusedWarpArgs {
    const T* memory;
    const T* weight;
    const T* bias;  // may be null
    const T* loc;
    const T* attn;
    T* out;
    const int64_t* shapes;
    const int64_t* starts;
    const uint8_t* mask;  // value padding mask [B, N] (nonzero = padded) or null
    long long n_tok;
    long long rows;       // B * H * Q, numbered head-major: row = (b * H + h) * Q + q
    int Q, C, H, L, P;
};

constexpr int kFwWarps = 2;

// 16-byte read-only load without L1 allocation: the gathered rows are read about once per SM, while the weight rows
// the projection reads next are read by every row of the head (c2: 6.15 -> 5.94 us per call, c1h 10.04 -> 9.93).
// Used for 512-byte rows only: on 1024-byte rows (float32 C = 256, float16 C = 512) the L1-allocating load measured
// faster (c5 float16 B1 Q50: 24.7 against 43.9 us).
__device__ __forceinline__ uint4 ld_nc_no_l1(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// What a corner outside the map reads: zeros, as many bytes as the widest row the kernel takes.
__device__ __align__(16) const uint4 g_fw_zero_row[128] = {};

// CV: 16-byte vectors per lane per corner row (C * sizeof(T) = 512 * CV, CV = 1, 2 or 4). DW: outputs per lane
// (D = 32 * DW). 96 registers a thread at 10 CTAs per SM, no spills. kDeep (512-byte rows, grids of at most 8 rows
// per SM): 24 corner rows in flight per lane instead of 16, at 6 CTAs per SM -- with few rows an SM the kernel is a
// chain of gather round trips, and 48 corners then take two instead of three (B200, float16, batch 1 with 100
// queries: 6.19 -> 5.61 us per call); with more rows it measured slower (2,400 rows: 9.2 -> 10.4 us).
template <typename T, int CV, int DW, bool kDeep = false>
__global__ void __launch_bounds__(kFwWarps * 32, kDeep ? 6 : 10) fused_warp_kernel(const FusedWarpArgs<T> a) {
    static_assert(!kDeep || CV == 1, "the deep batch is for 512-byte rows");
    constexpr int V = Elem<T>::kVec;      // elements per 16-byte vector
    constexpr int D = 32 * DW;
    constexpr int kB = kDeep ? 24 : (CV == 4 ? 2 : 16 / CV);  // corner rows in flight per lane
    constexpr int kRowBytes = 512 * CV;
    constexpr int kSlots = (kMaxCorners + kB - 1) / kB * kB;   // the longest padded list
    // per corner: the address of its memory row (or of the zero row) and its weight; the list is padded with
    // zero-weight entries on the zero row to a multiple of kB, so the gather loop needs no bounds test
    __shared__ const unsigned char* s_ptr[kFwWarps][kSlots];
    __shared__ float s_wt[kFwWarps][kSlots];

    grid_dependency_wait();
    launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long row = (long long)blockIdx.x * kFwWarps + warp;
    if (row >= a.rows) return;
    const int q = int(row % a.Q);
    const long long bh = row / a.Q;
    const int h = int(bh % a.H);
    const long long b = bh / a.H;
    const int LP = a.L * a.P, S = 4 * LP, S_pad = (S + kB - 1) / kB * kB;
    const unsigned char** ptr = s_ptr[warp];
    float* wt = s_wt[warp];
    const unsigned char* zero = reinterpret_cast<const unsigned char*>(g_fw_zero_row);

    // 1. corners of the row's points (loc / attn are [B, Q, H, L, P])
    {
        const uint8_t* mask_b = a.mask != nullptr ? a.mask + b * a.n_tok : nullptr;
        const unsigned char* mb = reinterpret_cast<const unsigned char*>(a.memory + b * a.n_tok * a.C);
        const long long base = ((b * a.Q + q) * a.H + h) * LP;
        for (int j = lane; j < LP; j += 32) {
            const Level lv = level_at(a.shapes, a.starts, level_of(j, a.P));
            const long long i = base + j;
            int tk[4];
            float w4[4];
            corners4<float>(to_acc(a.loc[2 * i]), to_acc(a.loc[2 * i + 1]), to_acc(a.attn[i]), lv, a.n_tok, tk, w4,
                            mask_b);
#pragma unroll
            for (int k = 0; k < 4; ++k) TD_BOUNDS_TOKEN(tk[k], a.n_tok);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                ptr[4 * j + k] = tk[k] >= 0 ? mb + (long long)tk[k] * kRowBytes : zero;
                wt[4 * j + k] = w4[k];
            }
        }
        for (int s = S + lane; s < S_pad; s += 32) {
            ptr[s] = zero;
            wt[s] = 0.f;
        }
    }
    __syncwarp();

    // 2. gather: lane holds channels [(lane + 32 v) * V, + V) of m_r, v < CV
    float acc[CV][V];
#pragma unroll
    for (int v = 0; v < CV; ++v)
#pragma unroll
        for (int i = 0; i < V; ++i) acc[v][i] = 0.f;
    for (int s0 = 0; s0 < S_pad; s0 += kB) {
        uint4 raw[kB][CV];
        // every load of the batch is issued before the first is used
#pragma unroll
        for (int u = 0; u < kB; ++u) {
            const uint4* src = reinterpret_cast<const uint4*>(ptr[s0 + u]) + lane;
#pragma unroll
            for (int v = 0; v < CV; ++v)
                raw[u][v] = CV == 1 ? ld_nc_no_l1(src + 32 * v) : __ldg(src + 32 * v);
        }
#pragma unroll
        for (int u = 0; u < kB; ++u) {
            const float w = wt[s0 + u];
#pragma unroll
            for (int v = 0; v < CV; ++v) {
                float x[V];
                unpack16<T>(raw[u][v], x);
#pragma unroll
                for (int i = 0; i < V; ++i) acc[v][i] = fmaf(w, x[i], acc[v][i]);
            }
        }
    }

    // 3. the bias term's weight sum
    float wsum = 0.f;
    if (a.bias != nullptr) {
        for (int s = lane; s < S; s += 32) wsum += wt[s];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
    }

    T* orow = a.out + ((b * a.Q + q) * a.H + h) * D;
    {
        // 4. projection on CUDA cores, eight outputs at a time: p[k] = sum over this lane's channels c of
        // W[hD + d0 + k, c] * m_r[c]; three halving steps (lanes 16, 8, 4 apart) leave each lane one output of the
        // eight, d0 + (lane >> 2), summed over 8 lanes, and two butterfly steps finish the sum over all 32. Lane l
        // keeps output (l & 3) * 8 + (l >> 2) of every 32 (chunk l & 3 of each group of four chunks).
        const T* wh = a.weight + (long long)h * D * (kRowBytes / int(sizeof(T))) + lane * V;
        float mine[DW];
#pragma unroll
        for (int c8 = 0; c8 < D / 8; ++c8) {
            float p[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) p[k] = 0.f;
#pragma unroll
            for (int v = 0; v < CV; ++v) {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    float wv[V];
                    load16<T>(wh + (c8 * 8 + k) * (kRowBytes / int(sizeof(T))) + 32 * v * V, wv);
#pragma unroll
                    for (int i = 0; i < V; ++i) p[k] = fmaf(wv[i], acc[v][i], p[k]);
                }
            }
#pragma unroll
            for (int o = 16, n = 4; o >= 4; o >>= 1, n >>= 1) {
                const bool upper = (lane & o) != 0;
#pragma unroll
                for (int i = 0; i < n; ++i) {
                    const float send = upper ? p[i] : p[i + n];
                    const float keep = upper ? p[i + n] : p[i];
                    p[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            p[0] += __shfl_xor_sync(0xffffffffu, p[0], 2);
            p[0] += __shfl_xor_sync(0xffffffffu, p[0], 1);
            if ((c8 & 3) == (lane & 3)) mine[c8 >> 2] = p[0];
        }
        // 5. + bias * sum of weights, stored: out[b, q, h * D + d]
#pragma unroll
        for (int k = 0; k < DW; ++k) {
            const int d = 32 * k + (lane & 3) * 8 + (lane >> 2);
            float v = mine[k];
            if (a.bias != nullptr) v = fmaf(to_acc(a.bias[h * D + d]), wsum, v);
            orow[d] = from_acc<T>(v);
        }
    }
}

}  // namespace td
