// td_sample_outproj.cuh -- project order, sampling half with the decoder's output_proj in the same kernel:
//   y[b, q, :] = Wo . attn[b, q, :] + bo,   attn[b, q, h*D + d] = sum_s w_s * value[b, tok_s, h, d]  (rounded to T)
//
// The attention half is sample_vec_kernel's (one or two (batch, query, head) rows a warp, corners before the grid
// dependency wait, one L2 round trip for the row's corner rows). What a chained output_proj costs at batch 1 is a
// kernel boundary and a second grid, not arithmetic (300 x 256 x 256 at the RT-DETR shape). A CTA here holds whole
// queries (kSampleWarps rows, or 2 x kSampleWarps with two rows a warp under the sampler's rule: rows / H queries),
// and its cluster of CS = 8 CTAs splits the output columns: after the gather every CTA writes its queries' attention
// rows (rounded to T, as the operator returns them) into its shared memory, the cluster synchronises, each CTA
// copies the cluster's rows of one query slot out of its peers' shared memory (distributed shared memory, one
// 16-byte load per lane: each row crosses the cluster once) and computes its C_out / CS output columns for the
// slot's CS queries. Each CTA thus reads 1 / CS of Wo (16 KB at
// C_out = HD = 256 in 16-bit types), where a CTA computing every column of its own queries would read all 128 KB of
// it -- the cost that sank a per-CTA epilogue (39 MB of L2 reads at c1h).
// The product: 16-bit types as warp-level tensor-core tiles (mma.sync m16n8k16, float32 accumulation; the slot's
// queries are A's rows, a warp takes an 8-column tile); float32 / float64 on CUDA cores (a lane per 16-byte chunk of
// K, a reduce-scatter over the warp). At 8 queries per cluster a 64- or 128-row tcgen05 tile would be mostly padding.
// In 16- and 32-bit types the kernel keeps to 64 registers (both row forms), so two of its CTAs still become
// resident beside a running projection CTA.
// Requirements (the host checks them, else output_proj is chained): kSampleWarps % H == 0; HD * sizeof(T) = 512
// (one 16-byte vector of K per lane: H * D = 256 in 16-bit types, 128 in float32); C_out <= 256; the sampler's
// vector-kernel conditions; Wo 16-byte aligned.
#pragma once

#include <type_traits>

#include "td_sampler.cuh"

namespace td {

constexpr int kOpCluster = 8;      // CTAs per cluster (the portable maximum; clusters of 4 and 16 measured slower)
constexpr int kOpColsPerWarp = 4;  // CUDA-core path: output columns per warp and query pass

template <typename T>
struct OutProjArgs {
    const T* weight;    // Wo [C_out, HD], row-major, 16-byte aligned
    const T* bias;      // bo [C_out] or null
    T* out;             // y [B * Q, C_out]
    long long queries;  // B * Q
    int C_out, HD;
    int cols;           // output columns per CTA: ceil(C_out / cluster size), at most 32 (CUDA cores) or 64 (MMA)
};

constexpr int kOpPad = 32;         // s_all row padding in elements: rows of 576 bytes in 16-bit types start 16 banks
                                   // apart, so the two rows of each 8-lane phase of a 16-byte fragment load do not
                                   // share a bank

// Queries per CTA: rw x kSampleWarps rows (one or two a warp) of H heads each.
__host__ __device__ inline int qpc_of(int H, int rw = 1) { return rw * kSampleWarps / H; }

// The corner lists' bytes: a row a warp (sample_vec_smem), or two rows a warp of S_pad slots (S_pad > 0).
template <typename T>
__host__ __device__ inline size_t sample_outproj_lists(int L, int P, int S_pad) {
    return S_pad > 0 ? size_t(kSampleWarps) * 2 * S_pad * (sizeof(int) + sizeof(typename Coord<T>::type))
                     : sample_vec_smem<T>(L, P);
}

// Dynamic shared memory: the sampler's corner lists, the CTA's attention rows [queries per CTA][HD] and the
// cluster's rows of one query slot [CS][HD + kOpPad], both of T.
template <typename T>
__host__ __device__ inline size_t sample_outproj_smem(int L, int P, int H, int HD, int CS, int S_pad = 0) {
    return sample_outproj_lists<T>(L, P, S_pad) +
           (size_t(qpc_of(H, S_pad > 0 ? 2 : 1)) * size_t(HD) + size_t(CS) * size_t(HD + kOpPad)) * sizeof(T);
}

// D (+)= A * B for one m16n8k16 tile of 16-bit inputs with float32 accumulation (warp-level tensor-core MMA): A 16 x 16
// row-major in a0..a3, B 16 x 8 column-major in b0, b1, D 16 x 8 in d (the PTX ISA's fragment layouts).
template <typename T>
__device__ __forceinline__ void mma_m16n8k16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    if constexpr (std::is_same<T, __half>::value) {
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                     "{%8, %9}, {%0, %1, %2, %3};"
                     : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                     : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                     "{%8, %9}, {%0, %1, %2, %3};"
                     : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                     : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

// kRW rows a warp: 1, or 2 (sample_vec_kernel's two-row form: both rows' corner prologues in one pass, a row per
// half-warp), so a CTA holds kRW x kSampleWarps rows = qpc_of(H, kRW) whole queries.
template <typename T, bool kWide, bool kNoAlloc, int CS, int kBatch, int kRW = 1>
__global__ void __launch_bounds__(kSampleWarps * 32) sample_outproj_kernel(const SampleArgs<T> a,
                                                                           const OutProjArgs<T> o) {
    using A = typename Elem<T>::acc;
    using CT = typename Coord<T>::type;
    constexpr int V = Elem<T>::kVec;
    constexpr int kWords = kWide ? 2 : 1;
    extern __shared__ __align__(16) unsigned char smem_raw[];

    launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = kRW == 1 ? 4 * a.L * a.P : a.S_pad;  // list slots a row
    int* s_tok = reinterpret_cast<int*>(smem_raw) + warp * kRW * S;
    CT* s_wt = reinterpret_cast<CT*>(smem_raw + kSampleWarps * kRW * S * sizeof(int)) + warp * kRW * S;
    T* s_att = reinterpret_cast<T*>(smem_raw + sample_outproj_lists<T>(a.L, a.P, kRW == 1 ? 0 : a.S_pad));

    // the rows' attention values, rounded to T, into s_att[query of the CTA][h * D + d]
    if constexpr (kRW == 1) {
        const long long row = (long long)blockIdx.x * kSampleWarps + warp;
        const bool live = row < a.rows;
        if (live) sample_row_corners<T>(a, row, lane, s_tok, s_wt);
        __syncwarp();
        grid_dependency_wait();
        A acc[kWords * V];
        if (live) {
            sample_row_sum<T, kWide, kNoAlloc, kBatch>(a, row, lane, s_tok, s_wt, acc);
        } else {
#pragma unroll
            for (int i = 0; i < kWords * V; ++i) acc[i] = A(0);
        }
        const int qi = warp / a.H, h = warp - qi * a.H;
        if (lane < a.G) {
#pragma unroll
            for (int k = 0; k < kWords; ++k)
                store16<T>(s_att + qi * o.HD + h * a.D + (lane * kWords + k) * V, acc + k * V);
        }
    } else {
        static_assert(kRW == 2, "one or two rows a warp");
        const long long row0 = ((long long)blockIdx.x * kSampleWarps + warp) * 2;
        sample_pair_corners<T>(a, row0, lane, s_tok, s_wt);  // rows past the end sample nothing: zero rows
        __syncwarp();
        grid_dependency_wait();
        const int r = lane >> 4, hl = lane & 15;
        A acc[kWords * V];
        sample_row_sum<T, kWide, kNoAlloc, kBatch, 16, true>(a, row0 + r, hl, s_tok + r * S, s_wt + r * S, acc);
        const int lr = 2 * warp + r, qi = lr / a.H, h = lr - qi * a.H;  // the row within the CTA
        if (hl < a.G) {
#pragma unroll
            for (int k = 0; k < kWords; ++k)
                store16<T>(s_att + qi * o.HD + h * a.D + (hl * kWords + k) * V, acc + k * V);
        }
    }

    cluster_arrive();  // this CTA's attention rows are written (release)

    const uint32_t rank = cluster_ctarank();
    const int c0 = int(rank) * o.cols;                               // this CTA's first output column
    const int qpc = qpc_of(a.H, kRW);
    const long long first_q = ((long long)blockIdx.x - rank) * qpc;  // the cluster's first query
    T* s_all = s_att + qpc * o.HD;                                   // [CS][HD + kOpPad]
    const int HDP = o.HD + kOpPad;

    // Per query slot qi: warp r copies rank r's row of the slot into s_all[r] (one 16-byte distributed-shared-memory
    // load per lane, so each row crosses the cluster once), the CTA synchronises, and the slot's CS queries x
    // this CTA's columns are computed from s_all. Between the cluster barrier's halves each thread loads the weights
    // it needs (an L2 round trip that then overlaps the wait for the other CTAs).
    auto copy_slot = [&](int qi) {
        if (qi > 0) __syncthreads();  // every warp is done with the previous slot's s_all
        for (int r = warp; r < CS; r += kSampleWarps) {
            const uint4 v = ld_cluster_v4(cluster_map(smem_addr(s_att + qi * o.HD + lane * V), uint32_t(r)));
            *reinterpret_cast<uint4*>(s_all + r * HDP + lane * V) = v;
        }
        // this CTA has read its peers' rows for the last time (the loads have returned: nothing to order)
        if (qi == qpc - 1) cluster_arrive_relaxed();
        __syncthreads();
    };

    if constexpr (sizeof(T) == 2) {
        // 16-bit types (H * D = 256): warp w < ceil(cols / 8) computes columns c0 + 8w .. + 7 as m16n8k16 tensor-core
        // products over the slot's CS queries (A rows 0 .. CS - 1, the other rows zero), 16 K steps. Lane
        // (g, t) = (lane / 4, lane % 4) supplies rows g and g + 8 of A and column g of B, and receives D[g][2t, 2t + 1]
        // and D[g + 8][2t, 2t + 1]: columns c0 + 8w + 2t and + 1 of queries g and g + 8 of the slot.
        // K order: the product is a sum over K, so any order serves that A and B share. Here the K steps 2kp and
        // 2kp + 1 of lane t take the 8 consecutive elements [32 kp + 8 t, + 8) -- {a0, a2} of step 2kp, then {a0, a2}
        // of step 2kp + 1 (b0, b1 likewise) -- so each lane reads its A row and its Wo row with one 16-byte load per
        // pair of steps.
        static_assert(CS <= 16, "the A tile holds at most 16 queries");
        constexpr int kPairs = 8;  // pairs of K steps: 256 = 8 x 32
        const int g = lane >> 2, t = lane & 3;
        const bool row0 = g < CS, row1 = g + 8 < CS;
        const bool mma_warp = warp < (o.cols + 7) / 8;
        const int col_b = 8 * warp + g;  // this lane's B column (tile column g)
        const bool b_ok = mma_warp && col_b < o.cols && c0 + col_b < o.C_out;
        const uint4* wrow = reinterpret_cast<const uint4*>(o.weight + (long long)(b_ok ? c0 + col_b : 0) * 256) + t;
        uint4 bf[kPairs];
#pragma unroll
        for (int kp = 0; kp < kPairs; ++kp) bf[kp] = b_ok ? __ldg(wrow + 4 * kp) : make_uint4(0u, 0u, 0u, 0u);
        const int col_d = 8 * warp + 2 * t;  // this lane's first output column (tile column 2t)
        const bool d0_ok = mma_warp && col_d < o.cols && c0 + col_d < o.C_out;
        const bool d1_ok = mma_warp && col_d + 1 < o.cols && c0 + col_d + 1 < o.C_out;
        const float b_lo = d0_ok && o.bias != nullptr ? to_acc(o.bias[c0 + col_d]) : 0.f;
        const float b_hi = d1_ok && o.bias != nullptr ? to_acc(o.bias[c0 + col_d + 1]) : 0.f;
        cluster_wait();  // every CTA's attention rows are in its shared memory (acquire)
        for (int qi = 0; qi < qpc; ++qi) {
            copy_slot(qi);
            if (!mma_warp) continue;
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            const uint4* a0p = reinterpret_cast<const uint4*>(s_all + (row0 ? g : 0) * HDP) + t;
            const uint4* a1p = reinterpret_cast<const uint4*>(s_all + (row1 ? g + 8 : 0) * HDP) + t;
#pragma unroll
            for (int kp = 0; kp < kPairs; ++kp) {
                const uint4 x0 = row0 ? a0p[4 * kp] : make_uint4(0u, 0u, 0u, 0u);
                const uint4 x1 = row1 ? a1p[4 * kp] : make_uint4(0u, 0u, 0u, 0u);
                mma_m16n8k16<T>(d, x0.x, x1.x, x0.y, x1.y, bf[kp].x, bf[kp].y);
                mma_m16n8k16<T>(d, x0.z, x1.z, x0.w, x1.w, bf[kp].z, bf[kp].w);
            }
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int gr = g + 8 * half;
                const long long gq = first_q + (long long)gr * qpc + qi;
                if ((half ? row1 : row0) && gq < o.queries) {
                    T* y = o.out + gq * o.C_out + c0 + col_d;
                    if (d0_ok) y[0] = from_acc<T>(d[2 * half] + b_lo);
                    if (d1_ok) y[1] = from_acc<T>(d[2 * half + 1] + b_hi);
                }
            }
        }
    } else {
        static_assert(CS == 8, "the CUDA-core path takes its ranks in two halves of four");
        // float32 / float64 (H * D = 128 / 64): CUDA cores, a lane owning one 16-byte chunk of K; columns
        // c0 + warp + kSampleWarps * j per warp, in two halves of four ranks: 16 partials per lane (rank r % 4,
        // column j at (r % 4) * 4 + j), which a reduce-scatter over the warp turns into finished outputs
        uint4 wv[kOpColsPerWarp];
        A bj[kOpColsPerWarp];
#pragma unroll
        for (int j = 0; j < kOpColsPerWarp; ++j) {
            const int cl = warp + kSampleWarps * j;
            const bool on = cl < o.cols && c0 + cl < o.C_out;
            wv[j] = on ? __ldg(reinterpret_cast<const uint4*>(o.weight + (long long)(c0 + cl) * o.HD) + lane)
                       : make_uint4(0u, 0u, 0u, 0u);
            bj[j] = on && o.bias != nullptr ? to_acc(o.bias[c0 + cl]) : A(0);
        }
        cluster_wait();  // every CTA's attention rows are in its shared memory (acquire)
        for (int qi = 0; qi < qpc; ++qi) {
            copy_slot(qi);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                A p[16];
#pragma unroll
                for (int rr = 0; rr < 4; ++rr) {
                    A x[V];
                    unpack16<T>(*reinterpret_cast<const uint4*>(s_all + (half * 4 + rr) * HDP + lane * V), x);
#pragma unroll
                    for (int j = 0; j < kOpColsPerWarp; ++j) {
                        A w[V];
                        unpack16<T>(wv[j], w);
                        A sum = A(0);
#pragma unroll
                        for (int i = 0; i < V; ++i) sum = fma(w[i], x[i], sum);
                        p[rr * kOpColsPerWarp + j] = sum;
                    }
                }
                // reduce-scatter: after the steps 16, 8, 4, 2 lane l holds partial (l >> 1) & 15 summed over the 16
                // lanes of its parity, and the step 1 adds the other parity's
#pragma unroll
                for (int off = 16, n = 8; off >= 2; off >>= 1, n >>= 1) {
                    const bool upper = (lane & off) != 0;
#pragma unroll
                    for (int i = 0; i < n; ++i) {
                        const A send = upper ? p[i] : p[i + n];
                        const A keep = upper ? p[i + n] : p[i];
                        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                    }
                }
                p[0] += __shfl_xor_sync(0xffffffffu, p[0], 1);
                const int pi = (lane >> 1) & 15, rr = pi >> 2, j = pi & 3;
                const int cl = warp + kSampleWarps * j;
                const long long gq = first_q + (long long)(half * 4 + rr) * qpc + qi;
                A bias_j = bj[0];
#pragma unroll
                for (int jj = 1; jj < kOpColsPerWarp; ++jj)
                    if (j == jj) bias_j = bj[jj];
                if ((lane & 1) == 0 && gq < o.queries && cl < o.cols && c0 + cl < o.C_out)
                    o.out[gq * o.C_out + c0 + cl] = from_acc<T>(p[0] + bias_j);
            }
        }
    }
    cluster_wait();  // no CTA leaves while a peer may still read its shared memory
}

}  // namespace td
