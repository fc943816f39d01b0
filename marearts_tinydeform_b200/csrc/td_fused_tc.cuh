// td_fused_tc.cuh -- fused order with the per-head projection on tcgen05 tensor cores (float16 / bfloat16).
//
// Computes what upstream's fused_vec computes (csrc/ma_deform_fused.cu:151-210):
//   m_r = sum_s w_s * memory[b, t_s, :]  (C wide),   out[b, q_r, hD + d] = W[hD + d] . m_r + bias[hD + d] * sum_s w_s
// The kernel is bounded by the L2 gather of C-wide corner rows (about 108 GB/s per SM on B200 with enough loads in
// flight), so it is built to give every SM the same share of that gather and to keep 100+ KB of it in flight:
//   * one persistent CTA of 16 warps per SM; rows r = (b, h, q) are numbered head-major (r = (b*H + h)*Q + q) and
//     CTA c owns the contiguous range [c*R/G, (c+1)*R/G) of the R = B*H*Q rows (+-1 row per SM);
//   * the range is walked in passes of at most kFtcPassRows rows spanning at most two (b, h) segments; each segment
//     needs one head's weight rows W[hD : hD + D, :], loaded by TMA (K-major, 128-byte swizzle) into its own slot;
//   * a pass computes its n x L x P bilinear corners into shared memory (one memory round trip), then splits its
//     K = n * S corners (S = L * P * 4) into 16 equal contiguous ranges, one per warp. A warp reads its corner rows 16
//     at a time (lanes over the C channels, 16-byte loads) and writes one float32 partial sum per row piece into its
//     own slot; a row straddling several warps' ranges is completed by adding their slots in warp order, so results
//     do not depend on timing;
//   * finished rows are rounded to T into the MMA's A operand (K-major, 128-byte swizzle: 16-byte chunk j of row r
//     sits at chunk j ^ (r & 7)), each segment starting on an 8-row boundary; one thread issues C/16 tcgen05.mma
//     (M = 128, N = D, K = 16) per segment into D float32 TMEM columns of its own; warp 0 reads the accumulator rows
//     (TMEM lane = row), adds bias * sum_s w_s and stores.
// The A operand is followed by the partial-sum slots, so the MMA's rows past the pass's rows read the next K block
// or those slots; they only produce accumulator rows that are never read. Rounding m to 16 bits before the MMA adds
// about half an ulp of relative error per channel.
#pragma once

#include <type_traits>

#include "td_common.cuh"
#include "td_ptx.cuh"

namespace td {

template <typename T>
struct FusedTcArgs {
    const T* memory;
    const T* bias;  // may be null
    const T* loc;
    const T* attn;
    T* out;
    const int64_t* shapes;
    const int64_t* starts;
    long long n_tok;
    const uint8_t* mask;  // value padding mask [B, N] (nonzero = padded) or null
    long long rows;  // B * H * Q
    int B, Q, C, H, D, L, P;
    int pieces;      // row pieces one warp's corner range can touch in a pass
};

constexpr int kFtcWarps = 16;
constexpr int kFtcThreads = kFtcWarps * 32;
constexpr int kFtcPassRows = 24;                  // rows per pass (<= 32: warp 0 reads them all from TMEM)
constexpr int kFtcARows = kFtcPassRows + 8;       // A rows: the second segment starts on an 8-row boundary
constexpr int kFtcSegs = 2;                       // (b, h) segments per pass

struct FusedTcLayout {
    uint32_t w_off, a_off, part_off, tok_off, wt_off, wsum_off, bias_off, bar_off, slot_off, bytes;
    __host__ __device__ FusedTcLayout(int C, int D, int S, int pieces) {
        const uint32_t kb = uint32_t(C / 64);
        w_off = 0;                                                    // kFtcSegs weight slots
        a_off = w_off + uint32_t(kFtcSegs) * kb * uint32_t(D) * 128u;
        part_off = a_off + kb * uint32_t(kFtcARows) * 128u;
        // the partial-sum slots double as the MMA's read-past slack: up to 127 rows of 128 bytes past a segment start
        uint32_t part_bytes = uint32_t(kFtcWarps * pieces * C) * 4u;
        if (part_bytes < 128u * 128u) part_bytes = 128u * 128u;
        tok_off = part_off + part_bytes;
        wt_off = tok_off + uint32_t(kFtcPassRows * S) * 4u;
        wsum_off = wt_off + uint32_t(kFtcPassRows * S) * 4u;
        bias_off = wsum_off + uint32_t(kFtcPassRows) * 4u;
        bar_off = (bias_off + uint32_t(kFtcSegs * D) * 4u + 7u) & ~7u;  // wbar[2], mbar
        slot_off = bar_off + 24u;
        bytes = slot_off + 16u + 1024u;  // + slack to align the base to 1024 bytes
    }
};

__host__ __device__ inline uint32_t tmem_cols_for(int n) {
    uint32_t c = 32;
    while (c < uint32_t(n)) c <<= 1;
    return c;
}

// Row pieces a warp's contiguous corner range can touch: its range is at most ceil(rows * S / warps) corners.
__host__ __device__ inline int fused_tc_pieces(int S) {
    const int span = (kFtcPassRows * S + kFtcWarps - 1) / kFtcWarps;
    return (span + S - 1) / S + 1;
}

// CV = 16-byte channel vectors per lane per corner row (C <= 256 * CV).
template <typename T, int CV>
__global__ void __launch_bounds__(kFtcThreads, 1)
    fused_tc_kernel(const __grid_constant__ CUtensorMap map_w, const FusedTcArgs<T> a) {
    constexpr int NW = kFtcWarps;
    constexpr int kB = 16 / CV;  // corner rows per batch (16-byte loads in flight per lane)
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);

    const int LP = a.L * a.P, S = 4 * LP, C = a.C, D = a.D, PC = a.pieces;
    const FusedTcLayout lay(C, D, S, PC);
    unsigned char* w_tile = smem + lay.w_off;
    unsigned char* a_tile = smem + lay.a_off;
    float* part = reinterpret_cast<float*>(smem + lay.part_off);
    int* tok = reinterpret_cast<int*>(smem + lay.tok_off);
    float* wt = reinterpret_cast<float*>(smem + lay.wt_off);
    float* wsum = reinterpret_cast<float*>(smem + lay.wsum_off);
    float* sbias = reinterpret_cast<float*>(smem + lay.bias_off);
    uint64_t* wbar = reinterpret_cast<uint64_t*>(smem + lay.bar_off);  // [2]
    uint64_t* mbar = wbar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + lay.slot_off);  // [0] TMEM base, [1] MMA skipped
    __shared__ int warp_first[kFtcWarps], row_wlo[kFtcPassRows], row_whi[kFtcPassRows];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kblocks = C / 64, nvec = C / 8;
    const uint32_t w_bytes = uint32_t(kblocks) * uint32_t(D) * 128u;
    const uint32_t tmem_cols = tmem_cols_for(kFtcSegs * D);
    const long long r_begin = a.rows * blockIdx.x / gridDim.x, r_end = a.rows * (blockIdx.x + 1) / gridDim.x;

    if (tid == 0) {
        mbar_init(&wbar[0], 1);
        mbar_init(&wbar[1], 1);
        mbar_init(mbar, 1);
        mbar_fence_init();
        tma_prefetch_desc(&map_w);
        tmem_slot[1] = 0u;
    }
    __syncwarp();
    if (warp == 0) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot[0];
    // Only shared memory and TMEM so far: under programmatic dependent launch this prologue overlaps the previous
    // kernel in the stream, and every global access comes after this wait.
    grid_dependency_wait();
    launch_dependents();

    int slot_h[kFtcSegs] = {-1, -1};       // head whose weights each slot holds
    int slot_loads[kFtcSegs] = {0, 0};     // completed phases of each slot's barrier
    bool slot_pending[kFtcSegs] = {false, false};
    int passes = 0;
    for (long long p0 = r_begin; p0 < r_end;) {
        // the pass: up to kFtcPassRows rows in at most two (b, h) segments
        const long long seg0 = p0 / a.Q;
        const long long e0 = min(r_end, min((seg0 + 1) * (long long)a.Q, p0 + kFtcPassRows));
        long long p1 = e0;
        if (p1 < r_end && p1 - p0 < kFtcPassRows)
            p1 = min(r_end, min((seg0 + 2) * (long long)a.Q, p0 + kFtcPassRows));
        const int n = int(p1 - p0), n0 = int(e0 - p0), nseg = p1 > e0 ? 2 : 1;
        const int a1 = (n0 + 7) & ~7;  // A row where segment 1 starts
        const int b0 = int(seg0 / a.H), h0 = int(seg0 - (long long)b0 * a.H), q00 = int(p0 - seg0 * a.Q);
        const int b1 = h0 + 1 == a.H ? b0 + 1 : b0, h1 = h0 + 1 == a.H ? 0 : h0 + 1;  // segment seg0 + 1

        // 1. weight rows: segment g uses slot g (reloaded when its head changed; the slot's previous MMA has
        // completed, since the previous pass's epilogue waited for it)
#pragma unroll
        for (int g = 0; g < kFtcSegs; ++g) {
            const int hg = g ? h1 : h0;
            if (g < nseg && hg != slot_h[g]) {
                if (tid == 0) {
                    mbar_arrive_expect_tx(&wbar[g], w_bytes);
                    for (int kb = 0; kb < kblocks; ++kb)
                        tma_load_2d(w_tile + (g * kblocks + kb) * D * 128, &map_w, &wbar[g], kb * 64, hg * D,
                                    l2_evict_last());
                }
                for (int d = tid; d < D; d += kFtcThreads)
                    sbias[g * D + d] = a.bias != nullptr ? to_acc(a.bias[hg * D + d]) : 0.f;
                slot_h[g] = hg;
                slot_pending[g] = true;
            }
        }
        // 2. corners of the pass's rows (row i of the pass is in segment i >= n0)
        for (int i = tid; i < n * LP; i += kFtcThreads) {
            const int r = i / LP, j = i - r * LP;
            const bool g = r >= n0;
            const int q = g ? r - n0 : q00 + r;
            const Level lv = level_at(a.shapes, a.starts, level_of(j, a.P));
            const int bimg = g ? b1 : b0;
            const long long k = (((long long)bimg * a.Q + q) * a.H + (g ? h1 : h0)) * LP + j;
            corners4<float>(to_acc(a.loc[2 * k]), to_acc(a.loc[2 * k + 1]), to_acc(a.attn[k]), lv, a.n_tok,
                            tok + r * S + 4 * j, wt + r * S + 4 * j,
                            a.mask != nullptr ? a.mask + (long long)bimg * a.n_tok : nullptr);
        }
        __syncthreads();

        // which warps hold pieces of which rows: warp w's corners are [K*w/NW, K*(w+1)/NW); row r is completed by
        // warps row_wlo[r] .. row_whi[r] (the largest w with K*w/NW <= r*S, resp. <= (r+1)*S - 1)
        const int K = n * S;
        if (tid < NW) {
            const int kb = K * tid / NW, ke = K * (tid + 1) / NW;
            warp_first[tid] = kb < ke ? kb / S : -1;
        } else if (tid >= 32 && tid < 32 + n) {
            const int r = tid - 32;
            row_wlo[r] = ((r * S + 1) * NW - 1) / K;
            row_whi[r] = ((r + 1) * S * NW - 1) / K;
        }
        // weight sums for the bias term
        for (int r = warp; r < n; r += NW) {
            float s = 0.f;
            for (int i = lane; i < S; i += 32) s += wt[r * S + i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) wsum[r] = s;
        }

        // 3. gather: warp w takes the corners [k_begin, k_end)
        {
            const int k_begin = K * warp / NW, k_end = K * (warp + 1) / NW;
            const int r_first = k_begin / S;
            for (int r = r_first; r * S < k_end; ++r) {
                const T* mb = a.memory + (long long)(r >= n0 ? b1 : b0) * a.n_tok * C;
                const int s_lo = max(k_begin - r * S, 0), s_hi = min(k_end - r * S, S);
                const int* tk = tok + r * S;
                const float* wr = wt + r * S;
                float acc[CV][8];
#pragma unroll
                for (int v = 0; v < CV; ++v)
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[v][i] = 0.f;
                for (int s0 = s_lo; s0 < s_hi; s0 += kB) {
                    uint4 raw[kB][CV];
                    float w[kB];
#pragma unroll
                    for (int u = 0; u < kB; ++u) {
                        const int s = s0 + u;
                        int t = s < s_hi ? tk[s] : -1;
                        TD_BOUNDS_TOKEN(t, a.n_tok);
                        w[u] = s < s_hi ? wr[s] : 0.f;
#pragma unroll
                        for (int v = 0; v < CV; ++v) {
                            const int cv = lane + 32 * v;
                            raw[u][v] = (t >= 0 && cv < nvec)
                                            ? __ldg(reinterpret_cast<const uint4*>(mb + (long long)t * C) + cv)
                                            : make_uint4(0, 0, 0, 0);
                        }
                    }
#pragma unroll
                    for (int u = 0; u < kB; ++u) {
#pragma unroll
                        for (int v = 0; v < CV; ++v) {
                            float x[8];
                            unpack16<T>(raw[u][v], x);
#pragma unroll
                            for (int i = 0; i < 8; ++i) acc[v][i] = fmaf(w[u], x[i], acc[v][i]);
                        }
                    }
                }
                float* slot = part + (warp * PC + (r - r_first)) * C;
#pragma unroll
                for (int v = 0; v < CV; ++v) {
                    const int cv = lane + 32 * v;
                    if (cv < nvec) {
                        reinterpret_cast<float4*>(slot)[2 * cv] = make_float4(acc[v][0], acc[v][1], acc[v][2], acc[v][3]);
                        reinterpret_cast<float4*>(slot)[2 * cv + 1] =
                            make_float4(acc[v][4], acc[v][5], acc[v][6], acc[v][7]);
                    }
                }
            }
        }
        __syncthreads();

        // 4. each row = its pieces added in warp order -> A operand (segment 1 from row a1), rounded and swizzled
        for (int i = tid; i < n * nvec; i += kFtcThreads) {
            const int r = i / nvec, cv = i - r * nvec;
            float v8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int w = row_wlo[r]; w <= row_whi[r]; ++w) {
                if (warp_first[w] < 0) continue;  // empty range
                const float* slot = part + (w * PC + (r - warp_first[w])) * C;
                const float4 lo = reinterpret_cast<const float4*>(slot)[2 * cv];
                const float4 hi = reinterpret_cast<const float4*>(slot)[2 * cv + 1];
                v8[0] += lo.x; v8[1] += lo.y; v8[2] += lo.z; v8[3] += lo.w;
                v8[4] += hi.x; v8[5] += hi.y; v8[6] += hi.z; v8[7] += hi.w;
            }
            const int ar = r < n0 ? r : a1 + (r - n0);
            store16<T>(reinterpret_cast<T*>(a_tile + (cv >> 3) * kFtcARows * 128 + ar * 128 +
                                            (((cv & 7) ^ (ar & 7)) << 4)),
                       v8);
        }

        // 5. the projections on the tensor cores: segment g -> TMEM columns [g*D, (g+1)*D)
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            const uint32_t idesc = idesc_f16(std::is_same<T, __nv_bfloat16>::value, 128, D);
#pragma unroll
            for (int g = 0; g < kFtcSegs; ++g) {
                if (g >= nseg) break;
                bool w_ready = true;
                if (slot_pending[g]) w_ready = mbar_wait(&wbar[g], uint32_t(slot_loads[g] & 1), kErrTmaWait);
                if (!w_ready) {
                    tmem_slot[1] = 1u;  // tell warp 0 not to store
                    continue;
                }
                const uint32_t sa = smem_addr(a_tile) + uint32_t(g ? a1 : 0) * 128u;
                const uint32_t sw = smem_addr(w_tile) + uint32_t(g * kblocks * D * 128);
                for (int kb = 0; kb < kblocks; ++kb) {
                    const uint64_t da = sdesc_sw128(sa + kb * kFtcARows * 128), dw = sdesc_sw128(sw + kb * D * 128);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        mma_f16(tmem + uint32_t(g * D), da + uint64_t(2 * k), dw + uint64_t(2 * k), idesc,
                                (kb | k) != 0);
                }
            }
            mma_commit(mbar);
        }
#pragma unroll
        for (int g = 0; g < kFtcSegs; ++g) {
            if (g < nseg && slot_pending[g]) {
                ++slot_loads[g];
                slot_pending[g] = false;
            }
        }

        // 6. epilogue: warp 0; segment 0 rows are TMEM lanes 0..n0-1 (columns 0..D-1), segment 1 rows are lanes
        // 0..n-n0-1 of columns D..2D-1
        if (warp == 0) {
            const bool ready = mbar_wait(mbar, uint32_t(passes & 1), kErrMmaWait);
            tc_fence_after();
            __syncwarp();
            const bool store = ready && tmem_slot[1] == 0u;
#pragma unroll
            for (int g = 0; g < kFtcSegs; ++g) {
                if (g >= nseg) break;
                const int rows_g = g ? n - n0 : n0, r = g ? n0 + lane : lane;
                const float ws = lane < rows_g ? wsum[r] : 0.f;
                const int q = g ? lane : q00 + lane;
                T* orow = a.out + (((long long)(g ? b1 : b0) * a.Q + q) * a.H + (g ? h1 : h0)) * D;
                for (int d0 = 0; d0 < D; d0 += 16) {
                    uint32_t v[16];
                    tmem_ld_32x32b_x16(tmem + uint32_t(g * D + d0), v);
                    tmem_ld_wait();
                    if (store && lane < rows_g) {
                        float o[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) o[i] = fmaf(sbias[g * D + d0 + i], ws, __uint_as_float(v[i]));
                        store16<T>(orow + d0, o);
                        store16<T>(orow + d0 + 8, o + 8);
                    }
                }
            }
        }
        ++passes;
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        p0 = p1;
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols);
    }
}

}  // namespace td
