// td_fused_tc.cuh -- fused order with the per-head projection on tcgen05 tensor cores (float16 / bfloat16).
//
// Computes what upstream's fused_vec computes (csrc/ma_deform_fused.cu:151-210):
//   m_r = sum_s w_s * memory[b, t_s, :]  (C wide),   out[b, q_r, hD + d] = W[hD + d] . m_r + bias[hD + d] * sum_s w_s
// but for a tile of RQ queries of one (batch, head) at once, so the projection is one [RQ x C] x [C x D] product:
//   1. thread 0 starts the TMA load of the head's weight rows W[hD : hD + D, :] (K-major, 128-byte swizzle), while
//      the CTA computes the bilinear corners of its RQ x L x P sampling points into shared memory;
//   2. gather: warp w takes rows w, w + 8, ...; its 32 lanes cover 256 channels with one 16-byte vector each and
//      keep up to 16 corner rows in flight; the float32 sums are rounded to the input type and written straight
//      into the MMA's A operand (K-major, 128-byte swizzle: 16-byte chunk j of row r sits at chunk j ^ (r & 7));
//   3. thread 0 issues C/16 tcgen05.mma (M = 128, N = D, K = 16) into a D-column float32 accumulator in TMEM;
//   4. epilogue: warps 0-3 read their TMEM lanes (row r = TMEM lane r), add bias * sum_s w_s, store.
// The A operand is only RQ rows per 64-wide K block: consecutive K blocks are RQ * 128 bytes apart, so the MMA's
// rows RQ..127 read the next block (or zeroed slack after the last one) and only produce accumulator rows that
// are never read. Rounding m to 16 bits before the MMA adds about one half-ulp relative error per channel.
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
    int B, Q, C, H, D, L, P;
    int RQ;       // queries per CTA, multiple of 8, <= 128
    int q_tiles;  // ceil(Q / RQ)
};

constexpr int kFtcWarps = 8;
constexpr int kFtcThreads = kFtcWarps * 32;
constexpr int kFtcBatch = 16;  // corner rows in flight per lane

struct FusedTcLayout {
    uint32_t w_off, a_off, tok_off, wt_off, wsum_off, bar_off, slot_off, bytes;
    __host__ __device__ FusedTcLayout(int RQ, int C, int D, int S) {
        const uint32_t kb = uint32_t(C / 64);
        w_off = 0;
        a_off = w_off + kb * uint32_t(D) * 128u;
        tok_off = a_off + kb * uint32_t(RQ) * 128u + uint32_t(128 - RQ) * 128u;
        wt_off = tok_off + uint32_t(RQ * S) * 4u;
        wsum_off = wt_off + uint32_t(RQ * S) * 4u;
        bar_off = (wsum_off + uint32_t(RQ) * 4u + 7u) & ~7u;
        slot_off = bar_off + 16u;
        bytes = slot_off + 16u + 1024u;  // + slack to align the base to 1024 bytes
    }
};

__host__ __device__ inline uint32_t tmem_cols_for(int n) {
    uint32_t c = 32;
    while (c < uint32_t(n)) c <<= 1;
    return c;
}

template <typename T>
__global__ void __launch_bounds__(kFtcThreads)
    fused_tc_kernel(const __grid_constant__ CUtensorMap map_w, const FusedTcArgs<T> a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ Level lv[kMaxLevels];
    unsigned char* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);

    const int LP = a.L * a.P, S = 4 * LP, C = a.C, D = a.D, RQ = a.RQ;
    const FusedTcLayout lay(RQ, C, D, S);
    unsigned char* w_tile = smem + lay.w_off;
    unsigned char* a_tile = smem + lay.a_off;
    int* tok = reinterpret_cast<int*>(smem + lay.tok_off);
    float* wt = reinterpret_cast<float*>(smem + lay.wt_off);
    float* wsum = reinterpret_cast<float*>(smem + lay.wsum_off);
    uint64_t* wbar = reinterpret_cast<uint64_t*>(smem + lay.bar_off);
    uint64_t* mbar = wbar + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + lay.slot_off);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = int(blockIdx.x % a.H);
    const long long bq = blockIdx.x / a.H;
    const int qt = int(bq % a.q_tiles), b = int(bq / a.q_tiles);
    const int q0 = qt * RQ, rows = min(RQ, a.Q - q0);
    const int kblocks = C / 64;
    const uint32_t tmem_cols = tmem_cols_for(D);

    if (threadIdx.x == 0) {
        mbar_init(wbar, 1);
        mbar_init(mbar, 1);
        mbar_fence_init();
        tma_prefetch_desc(&map_w);
        mbar_arrive_expect_tx(wbar, uint32_t(kblocks) * uint32_t(D) * 128u);
        for (int kb = 0; kb < kblocks; ++kb)
            tma_load_2d(w_tile + kb * D * 128, &map_w, wbar, kb * 64, h * D);
    }
    __syncwarp();
    if (warp == 0) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    // zero the slack after the last K block, so the rows the MMA reads past the A tile are finite
    for (int i = threadIdx.x; i < (128 - RQ) * 8; i += kFtcThreads)
        reinterpret_cast<uint4*>(a_tile + kblocks * RQ * 128)[i] = make_uint4(0, 0, 0, 0);
    load_levels(a.shapes, a.starts, a.L, lv);
    __syncthreads();

    // 1. corners of the tile's RQ x LP sampling points
    for (int i = threadIdx.x; i < RQ * LP; i += kFtcThreads) {
        const int r = i / LP, j = i - r * LP;
        if (r < rows) {
            const long long bqh = ((long long)b * a.Q + q0 + r) * a.H + h;
            row_corners(a.loc, a.attn, lv, LP, a.P, a.n_tok, bqh, j, tok + r * S + 4 * j, wt + r * S + 4 * j);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) { tok[r * S + 4 * j + k] = -1; wt[r * S + 4 * j + k] = 0.f; }
        }
    }
    __syncthreads();

    // 2. gather m into the A operand (rounded to T), and the weight sums
    const T* mb = a.memory + (long long)b * a.n_tok * C;
    for (int r = warp; r < RQ; r += kFtcWarps) {
        const int* tk = tok + r * S;
        const float* w = wt + r * S;
        float ws = 0.f;
        for (int i = lane; i < S; i += 32) ws += w[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
        if (lane == 0) wsum[r] = ws;
        for (int c0 = 0; c0 < C; c0 += 256) {
            const int cv = (c0 >> 3) + lane;          // 16-byte vector index within the row
            const bool active = cv * 8 < C;
            float acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.f;
            for (int s0 = 0; s0 < S; s0 += kFtcBatch) {
                uint4 raw[kFtcBatch];
                float wv[kFtcBatch];
#pragma unroll
                for (int u = 0; u < kFtcBatch; ++u) {
                    const int s = s0 + u;
                    const int t = s < S ? tk[s] : -1;
                    wv[u] = s < S ? w[s] : 0.f;
                    raw[u] = (t >= 0 && active)
                                 ? __ldg(reinterpret_cast<const uint4*>(mb + (long long)t * C) + cv)
                                 : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int u = 0; u < kFtcBatch; ++u) {
                    const uint32_t q[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float2 f;
                        if constexpr (std::is_same<T, __half>::value)
                            f = __half22float2(*reinterpret_cast<const __half2*>(&q[i]));
                        else
                            f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q[i]));
                        acc[2 * i] = fmaf(wv[u], f.x, acc[2 * i]);
                        acc[2 * i + 1] = fmaf(wv[u], f.y, acc[2 * i + 1]);
                    }
                }
            }
            if (active) {
                const int kb = cv >> 3, j = cv & 7;
                store16<T>(reinterpret_cast<T*>(a_tile + kb * RQ * 128 + r * 128 + ((j ^ (r & 7)) << 4)), acc);
            }
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // 3. projection on the tensor cores
    if (threadIdx.x == 0) {
        if (mbar_wait(wbar, 0, kErrTmaWait)) {
            const uint32_t idesc = idesc_f16(std::is_same<T, __nv_bfloat16>::value, 128, D);
            const uint32_t sa = smem_addr(a_tile), sw = smem_addr(w_tile);
            for (int kb = 0; kb < kblocks; ++kb) {
                const uint64_t da = sdesc_sw128(sa + kb * RQ * 128), dw = sdesc_sw128(sw + kb * D * 128);
#pragma unroll
                for (int k = 0; k < 4; ++k) mma_f16(tmem, da + uint64_t(2 * k), dw + uint64_t(2 * k), idesc,
                                                    (kb | k) != 0);
            }
        }
        mma_commit(mbar);
    }
    __syncwarp();

    // 4. epilogue: warp w < 4 reads TMEM lanes 32 w .. 32 w + 31 = tile rows
    if (warp < 4 && warp * 32 < rows) {
        const bool ready = mbar_wait(mbar, 0, kErrMmaWait);
        tc_fence_after();
        const int r = warp * 32 + lane;
        const float ws = r < rows ? wsum[r] : 0.f;
        T* orow = a.out + (((long long)b * a.Q + q0 + r) * a.H + h) * D;
        for (int d0 = 0; d0 < D; d0 += 16) {
            uint32_t v[16];
            tmem_ld_32x32b_x16(tmem + (uint32_t(warp * 32) << 16) + uint32_t(d0), v);
            tmem_ld_wait();
            if (ready && r < rows) {
                float o[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    o[i] = __uint_as_float(v[i]);
                    if (a.bias != nullptr) o[i] = fmaf(to_acc(a.bias[h * D + d0 + i]), ws, o[i]);
                }
                store16<T>(orow + d0, o);
                store16<T>(orow + d0 + 8, o + 8);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols);
    }
}

}  // namespace td
