// td_producer.cuh -- the producer of sampling_locations / attention_weights from the decoder's query projection.
//
// The standard multi-scale deformable attention layer (Deformable-DETR's MSDeformAttn, RT-DETR's decoder) computes,
// per query, proj = query @ [W_off; W_att]^T + [b_off; b_att] (one projection-kernel launch) and then, per
// (batch, query, head) row:
//   attention_weights[l, p] = softmax over the L * P logits of the row
//   sampling_locations[l, p] = ref[l] + offset[l, p] / (w_l, h_l)                 (2-d reference points)
//                            = ref[l].xy + offset[l, p] / P * ref[l].wh * 0.5       (4-d reference boxes)
// proj row layout: the 2 * H * L * P offsets (head, level, point, xy), then the H * L * P logits (head, level * point).
// One warp per row, lanes over the row's L * P <= 64 points (two per lane); the softmax max and sum are warp
// shuffles. produce_row is shared by the standalone producer kernel (which writes both tensors) and the sampler,
// which runs it in its corner prologue and never writes them out.
#pragma once

#include "td_common.cuh"
#include "td_ptx.cuh"

namespace td {

// The producer's inputs as the sampler carries them (proj == nullptr: the sampler reads sampling_locations and
// attention_weights instead).
template <typename T>
struct ProducerIn {
    const T* proj = nullptr;  // [B * Q, 3 * H * L * P]
    const T* ref = nullptr;   // [B, Q, L, ref_dim]
    int ref_dim = 2;
    // proj is written by the kernel right before this one (launched with programmatic serialization): wait for it
    // (griddepcontrol.wait) between the loads of the reference points and those of proj
    int wait_first = 0;
};

// Locations (lx, ly) and softmax weight w of the points j = lane + kLanes k (k = 0, 1) of row `row` = (b * Q + q) * H
// + h; a lane with j >= L * P gets w = 0. The row takes kLanes lanes: 32, or 16 when a warp holds two rows (lane is
// then the index within the row's half, and L * P <= 32). Every lane of the warp must call it (the softmax is a
// reduction over the row's lanes by xor shuffles; for L * P <= 16 the two widths give the same sums bit for bit, as
// the upper half only adds -inf to the max and exact zeros to the sum). All global loads of the row are issued before
// the first shuffle (with wait_first, the reference points and level sizes before the grid dependency wait, proj
// after it).
template <typename T, typename A, int kLanes = 32>
__device__ __forceinline__ void produce_row(const ProducerIn<T>& in, const int64_t* __restrict__ shapes,
                                            long long row, int H, int L, int P, int lane, A (&lx)[2], A (&ly)[2],
                                            A (&w)[2]) {
    const int LP = L * P;
    const long long bq = row / H;
    const int h = int(row - bq * H);
    const T* __restrict__ base = in.proj + bq * 3LL * H * LP;
    const T* __restrict__ off = base + (long long)h * LP * 2;
    const T* __restrict__ logit = base + 2LL * H * LP + (long long)h * LP;
    A x[2], ox[2], oy[2], rx[2], ry[2], sx[2], sy[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int j = lane + kLanes * k;
        const bool on = j < LP;
        const int l = on ? j / P : 0;
        const T* __restrict__ r = in.ref + (bq * L + l) * in.ref_dim;
        rx[k] = on ? to_acc(r[0]) : A(0);
        ry[k] = on ? to_acc(r[1]) : A(0);
        if (in.ref_dim == 2) {  // offset normaliser (w_l, h_l)
            sx[k] = on ? A(shapes[2 * l + 1]) : A(1);
            sy[k] = on ? A(shapes[2 * l]) : A(1);
        } else {                // box width and height
            sx[k] = on ? to_acc(r[2]) : A(0);
            sy[k] = on ? to_acc(r[3]) : A(0);
        }
    }
    if (in.wait_first) grid_dependency_wait();
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int j = lane + kLanes * k;
        const bool on = j < LP;
        x[k] = on ? to_acc(logit[j]) : A(-INFINITY);
        ox[k] = on ? to_acc(off[2 * j]) : A(0);
        oy[k] = on ? to_acc(off[2 * j + 1]) : A(0);
    }
    A m = x[0] > x[1] ? x[0] : x[1];
#pragma unroll
    for (int o = kLanes / 2; o > 0; o >>= 1) {
        const A y = __shfl_xor_sync(0xffffffffu, m, o);
        m = y > m ? y : m;
    }
    A e[2], sum = A(0);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        e[k] = lane + kLanes * k < LP ? exp(x[k] - m) : A(0);
        sum += e[k];
    }
#pragma unroll
    for (int o = kLanes / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        w[k] = e[k] / sum;
        if (in.ref_dim == 2) {
            lx[k] = rx[k] + ox[k] / sx[k];
            ly[k] = ry[k] + oy[k] / sy[k];
        } else {
            lx[k] = rx[k] + ox[k] / A(P) * sx[k] * A(0.5);
            ly[k] = ry[k] + oy[k] / A(P) * sy[k] * A(0.5);
        }
    }
}

template <typename T>
struct ProducerArgs {
    ProducerIn<T> in;
    const int64_t* shapes;    // [L, 2] (height, width)
    T* loc;                   // [B, Q, H, L, P, 2]
    T* attn;                  // [B, Q, H, L, P]
    long long rows;           // B * Q * H
    int H, L, P;
};

constexpr int kProducerWarps = 8;

// The standalone producer: writes sampling_locations and attention_weights. Launched with programmatic dependent
// launch behind the projection kernel (its reads of proj come after the grid dependency wait).
template <typename T>
__global__ void __launch_bounds__(kProducerWarps * 32) sampling_producer_kernel(const ProducerArgs<T> a) {
    using A = typename Elem<T>::acc;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long row = (long long)blockIdx.x * kProducerWarps + warp;
    grid_dependency_wait();  // proj is the output of the kernel before this one
    launch_dependents();
    if (row >= a.rows) return;  // warp-uniform
    A lx[2], ly[2], w[2];
    produce_row<T, A>(a.in, a.shapes, row, a.H, a.L, a.P, lane, lx, ly, w);
    const int LP = a.L * a.P;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int j = lane + 32 * k;
        if (j >= LP) continue;
        const long long i = row * LP + j;
        a.loc[2 * i] = from_acc<T>(lx[k]);
        a.loc[2 * i + 1] = from_acc<T>(ly[k]);
        a.attn[i] = from_acc<T>(w[k]);
    }
}

// ---- backward ------------------------------------------------------------------------------------------------
// Gradients of the producer, given those of its two outputs (either may be absent: zero):
//   logits:  g_x[j] = w[j] * (g_w[j] - sum_k w[k] g_w[k])                       (softmax over the row's L * P points)
//   offsets: 2-d reference points: g_off = g_loc / (w_l, h_l);  4-d boxes: g_off = g_loc * wh / P * 0.5
//   reference points (summed over the query's heads and each level's points):
//            g_ref.xy += g_loc;  4-d boxes also g_ref.wh += g_loc * off / P * 0.5
// One CTA per (batch, query), warp w taking heads w, w + kProducerWarps, ... with lanes over the L * P points (two
// per lane, as the forward); the reference-point gradient is then summed over the warps and each level's points
// through shared memory, in a fixed order (no atomics: bitwise reproducible).
template <typename T>
struct ProducerBwdArgs {
    const T* proj;            // [B * Q, 3 * H * L * P]: offsets (head, level, point, xy), then logits (head, L * P)
    const T* ref;             // [B, Q, L, ref_dim]
    const int64_t* shapes;    // [L, 2] (height, width)
    const T* g_loc;           // [B, Q, H, L, P, 2] or null
    const T* g_attn;          // [B, Q, H, L, P] or null
    T* g_proj;                // [B * Q, 3 * H * L * P]
    T* g_ref;                 // [B, Q, L, ref_dim] or null
    long long bq;             // B * Q
    int ref_dim, H, L, P;
};

template <typename T>
__global__ void __launch_bounds__(kProducerWarps * 32) sampling_producer_backward_kernel(const ProducerBwdArgs<T> a) {
    using A = typename Elem<T>::acc;
    // per warp and point: the point's reference-gradient terms summed over the warp's heads (x, y, w, h)
    __shared__ A s_sum[kProducerWarps][kMaxLevelPoints][4];
    grid_dependency_wait();
    launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long bq = blockIdx.x;
    const int LP = a.L * a.P;
    const long long row_len = 3LL * a.H * LP;
    const T* __restrict__ base = a.proj + bq * row_len;
    T* __restrict__ gbase = a.g_proj + bq * row_len;
    const A inv_p_half = A(0.5) / A(a.P);
    A sx[2], sy[2], acc[2][4];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int j = lane + 32 * k;
        const bool on = j < LP;
        const int l = on ? level_of(j, a.P) : 0;
        if (a.ref_dim == 2) {  // the offset normaliser (w_l, h_l)
            sx[k] = on ? A(a.shapes[2 * l + 1]) : A(1);
            sy[k] = on ? A(a.shapes[2 * l]) : A(1);
        } else {               // the box's width and height
            const T* r = a.ref + (bq * a.L + l) * 4;
            sx[k] = on ? to_acc(r[2]) : A(0);
            sy[k] = on ? to_acc(r[3]) : A(0);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[k][c] = A(0);
    }
    for (int h = warp; h < a.H; h += kProducerWarps) {
        const T* __restrict__ off = base + (long long)h * LP * 2;
        const T* __restrict__ logit = base + 2LL * a.H * LP + (long long)h * LP;
        const long long pt0 = (bq * a.H + h) * LP;  // this head's first point in loc / attn
        A x[2], ox[2], oy[2], gx[2], gy[2], gw[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int j = lane + 32 * k;
            const bool on = j < LP;
            x[k] = on ? to_acc(logit[j]) : A(-INFINITY);
            ox[k] = on ? to_acc(off[2 * j]) : A(0);
            oy[k] = on ? to_acc(off[2 * j + 1]) : A(0);
            gx[k] = on && a.g_loc != nullptr ? to_acc(a.g_loc[2 * (pt0 + j)]) : A(0);
            gy[k] = on && a.g_loc != nullptr ? to_acc(a.g_loc[2 * (pt0 + j) + 1]) : A(0);
            gw[k] = on && a.g_attn != nullptr ? to_acc(a.g_attn[pt0 + j]) : A(0);
        }
        // the forward's softmax again
        A m = x[0] > x[1] ? x[0] : x[1];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const A y = __shfl_xor_sync(0xffffffffu, m, o);
            m = y > m ? y : m;
        }
        A e[2], sum = A(0);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            e[k] = lane + 32 * k < LP ? exp(x[k] - m) : A(0);
            sum += e[k];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        A w[2], dot = A(0);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            w[k] = e[k] / sum;
            dot += w[k] * gw[k];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        T* __restrict__ g_off = gbase + (long long)h * LP * 2;
        T* __restrict__ g_logit = gbase + 2LL * a.H * LP + (long long)h * LP;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int j = lane + 32 * k;
            if (j >= LP) continue;
            g_logit[j] = from_acc<T>(w[k] * (gw[k] - dot));
            if (a.ref_dim == 2) {
                g_off[2 * j] = from_acc<T>(gx[k] / sx[k]);
                g_off[2 * j + 1] = from_acc<T>(gy[k] / sy[k]);
            } else {
                g_off[2 * j] = from_acc<T>(gx[k] * sx[k] * inv_p_half);
                g_off[2 * j + 1] = from_acc<T>(gy[k] * sy[k] * inv_p_half);
                acc[k][2] += gx[k] * ox[k] * inv_p_half;
                acc[k][3] += gy[k] * oy[k] * inv_p_half;
            }
            acc[k][0] += gx[k];
            acc[k][1] += gy[k];
        }
    }
    if (a.g_ref == nullptr) return;  // uniform over the CTA
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int j = lane + 32 * k;
        if (j < LP) {
#pragma unroll
            for (int c = 0; c < 4; ++c) s_sum[warp][j][c] = acc[k][c];
        }
    }
    __syncthreads();
    // output i (threads over L * ref_dim): level i / ref_dim, coordinate i % ref_dim, summed over the warps that held
    // heads, then the level's points, in order
    const int warps = a.H < kProducerWarps ? a.H : kProducerWarps;
    for (int i = threadIdx.x; i < a.L * a.ref_dim; i += kProducerWarps * 32) {
        const int l = i / a.ref_dim, c = i - l * a.ref_dim;
        A v = A(0);
        for (int ww = 0; ww < warps; ++ww)
            for (int p = 0; p < a.P; ++p) v += s_sum[ww][l * a.P + p][c];
        a.g_ref[(bq * a.L + l) * a.ref_dim + c] = from_acc<T>(v);
    }
}

}  // namespace td
