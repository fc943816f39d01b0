// td_gemm_tc.cuh -- value projection on tcgen05 tensor cores (float16 / bfloat16): value = memory @ W^T + b.
//
// Replaces the cuBLAS F.linear of upstream's project order (marearts_tinydeform/__init__.py:77).
// One CTA computes a 128 x BN tile of value (M = B*N tokens, N = H*D output channels, K = C):
//   * warp 0, one thread: TMA producer -- 128 x 64 tiles of memory and BN x 64 tiles of W (128-byte swizzle,
//     K-major) into a kStages-deep ring of shared-memory slots, each slot completed on its own mbarrier;
//   * warp 1, one thread: MMA issuer -- four tcgen05.mma (M=128, N=BN, K=16) per 64-wide K block into a
//     128 x BN float32 accumulator in tensor memory; a tcgen05.commit per block hands the slot back;
//   * all four warps: epilogue -- tcgen05.ld of the thread's accumulator row (TMEM lane = tile row), + bias,
//     narrowed to 16 bits and stored 16 bytes at a time, either as [B*N, HD] or head-major [B, H, N, D]
//     (every 8-column group of a row lands in one head's D-row, so the stores stay 16-byte vectors).
// Memory is read once per N tile (BN = 256 covers H*D = 256 in one tile when there are enough M tiles).
#pragma once

#include <type_traits>

#include "td_common.cuh"
#include "td_gemm_simt.cuh"
#include "td_ptx.cuh"

namespace td {

template <typename T>
struct ProjTcArgs {
    const T* bias;  // [HD] or null
    T* value;
    long long M, n_tok;
    int C, HD, H, D;
    int head_major;
    int k_blocks;   // ceil(C / 64)
};

constexpr int kTcBM = 128, kTcBK = 64, kTcStages = 4;

template <int BN>
struct ProjTcLayout {
    static constexpr uint32_t kABytes = kTcBM * kTcBK * 2;  // 16 KB
    static constexpr uint32_t kBBytes = BN * kTcBK * 2;
    static constexpr uint32_t kStageBytes = kABytes + kBBytes;
    static constexpr uint32_t kTileBytes = kTcStages * kStageBytes;
    static constexpr uint32_t kBarOffset = kTileBytes;                 // full[S], empty[S], accum
    static constexpr uint32_t kSlotOffset = kBarOffset + (2 * kTcStages + 1) * 8;
    static constexpr uint32_t kBiasOffset = kSlotOffset + 16;           // BN floats
    static constexpr uint32_t kSmemBytes = kBiasOffset + BN * 4 + 1024;  // + slack to align the base to 1024
    static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
};

template <typename T, int BN>
__global__ void __launch_bounds__(128, 1)
    proj_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const ProjTcArgs<T> a) {
    using Lay = ProjTcLayout<BN>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    // 1024-byte aligned base (the 128-byte swizzle pattern is anchored at 1024-byte boundaries)
    unsigned char* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lay::kBarOffset);
    uint64_t* empty = full + kTcStages;
    uint64_t* accum = empty + kTcStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::kSlotOffset);
    float* sbias = reinterpret_cast<float*>(smem + Lay::kBiasOffset);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long m0 = (long long)blockIdx.x * kTcBM;
    const int n0 = blockIdx.y * BN;

    const int KB = a.k_blocks;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        mbar_fence_init();
        tma_prefetch_desc(&map_a);
        tma_prefetch_desc(&map_b);
    }
    __syncwarp();
    if (warp == 0) {
        tmem_alloc(tmem_slot, Lay::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Everything above touches only shared memory and TMEM, so under programmatic dependent launch it overlaps the
    // previous kernel in the stream; every global read and write comes after this wait.
    grid_dependency_wait();
    // the sampler that follows in the project order may start its prologue now (it waits for this grid before
    // reading value)
    launch_dependents();

    if (threadIdx.x == 0) {
        // the first kTcStages K blocks need no free slot
        for (int kb = 0; kb < KB && kb < kTcStages; ++kb) {
            unsigned char* st = smem + kb * Lay::kStageBytes;
            mbar_arrive_expect_tx(&full[kb], Lay::kStageBytes);
            tma_load_2d(st, &map_a, &full[kb], kb * kTcBK, int(m0));
            tma_load_2d(st + Lay::kABytes, &map_b, &full[kb], kb * kTcBK, n0);
        }
    }
    if (warp == 0 && lane == 0) {
        // TMA producer for the K blocks beyond the first kTcStages
        for (int kb = kTcStages; kb < KB; ++kb) {
            const int s = kb % kTcStages, round = kb / kTcStages;
            if (!mbar_wait(&empty[s], (round & 1) ^ 1, kErrSlotWait)) break;
            unsigned char* st = smem + s * Lay::kStageBytes;
            mbar_arrive_expect_tx(&full[s], Lay::kStageBytes);
            tma_load_2d(st, &map_a, &full[s], kb * kTcBK, int(m0));
            tma_load_2d(st + Lay::kABytes, &map_b, &full[s], kb * kTcBK, n0);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer
        constexpr uint32_t idesc = idesc_f16(std::is_same<T, __nv_bfloat16>::value, kTcBM, BN);
        for (int kb = 0; kb < KB; ++kb) {
            const int s = kb % kTcStages, round = kb / kTcStages;
            if (!mbar_wait(&full[s], round & 1, kErrTmaWait)) break;
            tc_fence_after();
            const uint32_t sa = smem_addr(smem + s * Lay::kStageBytes);
            const uint64_t da = sdesc_sw128(sa), db = sdesc_sw128(sa + Lay::kABytes);
#pragma unroll
            for (int k = 0; k < kTcBK / 16; ++k)  // K = 16 per MMA = 32 bytes along the swizzled row
                mma_f16(tmem, da + uint64_t(2 * k), db + uint64_t(2 * k), idesc, (kb | k) != 0);
            mma_commit(&empty[s]);
        }
        mma_commit(accum);
    }
    __syncwarp();
    // the tile's bias columns, staged while the loads and MMAs run
    for (int i = threadIdx.x; i < BN; i += 128)
        sbias[i] = (a.bias != nullptr && n0 + i < a.HD) ? to_acc(a.bias[n0 + i]) : 0.f;

    // epilogue: thread (warp w, lane i) owns tile row 32 w + i = TMEM lane 32 w + i
    const bool ready = mbar_wait(accum, 0, kErrMmaWait);
    __syncthreads();  // the staged bias is visible
    tc_fence_after();
    if (ready) {
        const long long row = m0 + warp * 32 + lane;
        // where an 8-column group of this row goes: value + base + (column's head) * head_step + column's d
        long long base = row * a.HD, head_step = a.D;
        if (a.head_major) {
            const long long bimg = row / a.n_tok, n = row - bimg * a.n_tok;
            base = bimg * a.H * a.n_tok * a.D + n * a.D;
            head_step = a.n_tok * a.D;
        }
#pragma unroll 1
        for (int j = 0; j < BN / 32; ++j) {
            const int col0 = n0 + 32 * j;
            if (col0 >= a.HD) break;  // uniform across the warp
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem + (uint32_t(warp * 32) << 16) + uint32_t(32 * j), r);
            tmem_ld_wait();
            if (row < a.M) {
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const int col = col0 + 8 * g;
                    if (col >= a.HD) break;
                    const int h = col / a.D, d = col - h * a.D;
                    float v[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[8 * g + i]) + sbias[32 * j + 8 * g + i];
                    store16<T>(a.value + base + h * head_step + d, v);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, Lay::kTmemCols);
    }
}

}  // namespace td
