// td_gemm_grad.cuh -- the GEMMs of nn.Linear's backward, for the parameter and input gradients of the training path.
//
// For y = x @ W^T + b (x [M, K], W [Nout, K]) and the gradient g of y:
//   grad_x [M, K]    = g @ W            "input gradient"   A = g [M, Nout] (K-major: the sum runs along g's rows),
//                                                          B = W [Nout, K] (MN-major: the sum runs down W's columns)
//   grad_W [Nout, K] = g^T @ x          "weight gradient"  A = g [M, Nout], B = x [M, K], both MN-major: the sum runs
//                                                          over the M rows (all tokens of all images)
// In the operator's backward, x is memory, W value_weight and g grad_value; for output_proj, x is the attention
// result, W output_weight and g the gradient of the layer output.
//
// 16-bit types run grad_gemm_tc_kernel on tcgen05 tensor cores, one CTA per (output tile of 128 rows x BN columns,
// K slice):
//   * warp 0, one lane per box: TMA producers into a ring of slots, each slot one 64-deep K block of A and of B with the
//     128-byte swizzle: a K-major A is one 64 x 128 box; an MN-major operand is a box of 64 rows of K by 64 columns
//     of M (or N) per 64 columns -- the canonical MN-major layout, whose atom is 64 elements by 8 K rows (1 KB):
//     stride byte offset 1024 (the next 8 K rows), leading byte offset 8192 (the next 64 columns, the next box);
//   * warp 1, one lane: MMA issuer (tcgen05.mma kind::f16, M = 128, N = BN, four K steps of 16 a block; a K step
//     advances a K-major descriptor by 32 bytes and an MN-major one by 2048 bytes), float32 accumulator in TMEM;
//   * warps 4-7: epilogue, TMEM lane = tile row. Input gradient: narrowed to the input type and stored. Weight
//     gradient (K split over CTAs so that the grid fills the SMs): each CTA stores its float32 partial tile into its
//     split's slice of a workspace, and grad_split_reduce_kernel then sums the slices in split order and converts
//     (deterministic; it replaced float32 vector reductions into one accumulator with a last-arriving CTA
//     converting, whose 33-way contention per address at c1h made the GEMM 24.8 us). No CTA waits for another.
// float32 and float64 run grad_gemm_simt_kernel: 64 x 64 tiles on CUDA cores, K split the same way, float32 /
// float64 atomic adds straight into the (zeroed) output for the weight gradient.
// Every mbarrier wait is bounded (td_ptx.cuh).
#pragma once

#include <type_traits>

#include "td_common.cuh"
#include "td_ptx.cuh"

namespace td {

template <typename T>
struct GradGemmArgs {
    T* out;               // [rows, cols] row-major
    float* acc;           // weight gradient of 16-bit types: float32 partial sums [splits, rows, cols]
    int rows, cols;       // output size (M x N of the GEMM)
    int m_tiles, n_tiles, splits;
    int k_blocks;         // 64-deep K blocks in all
    int kb_per_split;     // K blocks per split (the last split takes what is left)
    // Test of the bounded waits (td_test_starve_next_grad_gemm): starve = 1 makes the TMA producer issue nothing,
    // so that every wait runs out after spin_limit cycles with nothing in flight; 0 in every ordinary launch.
    int starve;
    long long spin_limit;  // cycles a wait gives up after (kSpinLimitCycles in ordinary launches)
};

template <int BN>
struct GradTcLayout {
    static constexpr uint32_t kABytes = 128 * 128;  // 128 rows x 64 16-bit elements
    static constexpr uint32_t kBBytes = BN * 128;
    static constexpr uint32_t kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = BN == 256 ? 4 : 6;
    static constexpr uint32_t kBarOffset = kStages * kStageBytes;  // full[S], empty[S], tfull, drained
    static constexpr uint32_t kSlotOffset = kBarOffset + (2 * kStages + 2) * 8;  // TMEM base, last-arrival flag
    static constexpr uint32_t kSmemBytes = kSlotOffset + 16 + 1024;  // + slack to align the base to 1024
    static constexpr int kThreads = 256;
    static_assert(BN == 128 || BN == 256, "tile width");
};

// Shared-memory descriptor of an MN-major operand in the 128-byte-swizzle canonical layout (see the file comment).
__device__ __forceinline__ uint64_t sdesc_sw128_mn(uint32_t saddr) {
    uint64_t d = 0;
    d |= uint64_t((saddr & 0x3FFFFu) >> 4);
    d |= uint64_t(8192 >> 4) << 16;  // leading byte offset: the next 64 M / N elements
    d |= uint64_t(1024 >> 4) << 32;  // stride byte offset: the next 8 K rows
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// A_MN: A is MN-major (weight gradient); otherwise K-major (input gradient). SPLIT: each CTA stores its float32
// partial tile into its split's slice of `acc` (weight gradient; grad_split_reduce_kernel sums the slices in split
// order and converts); otherwise direct stores.
template <typename T, bool A_MN, int BN, bool SPLIT>
__global__ void __launch_bounds__(256) grad_gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a,
                                                           const __grid_constant__ CUtensorMap map_b,
                                                           const GradGemmArgs<T> a) {
    using Lay = GradTcLayout<BN>;
    constexpr int S = Lay::kStages;
    constexpr int kABoxes = A_MN ? 2 : 1;  // MN-major: two 64-column boxes of 64 K rows; K-major: one 64 x 128 box
    constexpr int kBoxes = kABoxes + BN / 64;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lay::kBarOffset);
    uint64_t* empty = full + S;
    uint64_t* tfull = empty + S;
    uint64_t* drained = tfull + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::kSlotOffset);
    auto slot_a = [&](int s) { return smem + s * Lay::kStageBytes; };
    auto slot_b = [&](int s) { return smem + s * Lay::kStageBytes + Lay::kABytes; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int t = blockIdx.x;
    const int split = t % a.splits;
    t /= a.splits;
    const int nt = t % a.n_tiles, mt = t / a.n_tiles;
    const int m0 = mt * 128, n0 = nt * BN;
    const int kb0 = split * a.kb_per_split;
    const int kb1 = min(kb0 + a.kb_per_split, a.k_blocks);
    const int nkb = kb1 - kb0;  // >= 1: the host sizes the splits so that none is empty

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], kBoxes);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tfull, 1);
        mbar_init(drained, 1);
        mbar_fence_init();
        tma_prefetch_desc(&map_a);
        tma_prefetch_desc(&map_b);
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dependency_wait();  // the operands were written by the kernels before this one
    launch_dependents();

    const long long limit = a.spin_limit;
    if (warp == 0) {
        // one issuing lane per box of a slot (kBoxes of them: the TMA copies of one thread are served one after
        // another, those of different threads overlap); each arms the slot's full barrier for its own bytes
        if (lane < kBoxes) {
            const uint64_t pol = l2_evict_first();
            const int issue = a.starve ? 0 : nkb;  // the blocks this producer loads
            int issued = 0;
            for (int i = 0; i < issue; ++i, ++issued) {
                const int s = i % S;
                if (!mbar_wait_limit(&empty[s], uint32_t((i / S) & 1) ^ 1u, kErrSlotWait, limit)) break;
                const int k0 = (kb0 + i) * 64;
                if (lane < kABoxes) {
                    mbar_arrive_expect_tx(&full[s], Lay::kABytes / kABoxes);
                    if constexpr (A_MN)
                        tma_load_2d(slot_a(s) + lane * 8192, &map_a, &full[s], m0 + 64 * lane, k0, pol);
                    else
                        tma_load_2d(slot_a(s), &map_a, &full[s], k0, m0, pol);
                } else {
                    const int j = lane - kABoxes;
                    mbar_arrive_expect_tx(&full[s], 8192u);
                    tma_load_2d(slot_b(s) + j * 8192, &map_b, &full[s], n0 + 64 * j, k0, pol);
                }
            }
            // the MMA commit of each slot's last use arrives before the CTA exits
            if (lane == 0)
                for (int i = issued > S ? issued - S : 0; i < issued; ++i)
                    if (!mbar_wait_limit(&empty[i % S], uint32_t((i / S) & 1), kErrSlotWait, limit)) break;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
            constexpr uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(A_MN) << 15) | (1u << 16) |
                                       (uint32_t(BN >> 3) << 17) | (uint32_t(128 >> 4) << 24);
            bool ok = true;
            for (int i = 0; i < nkb; ++i) {
                const int s = i % S;
                if (!mbar_wait_limit(&full[s], uint32_t((i / S) & 1), kErrTmaWait, limit)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t da = A_MN ? sdesc_sw128_mn(smem_addr(slot_a(s))) : sdesc_sw128(smem_addr(slot_a(s)));
                const uint64_t db = sdesc_sw128_mn(smem_addr(slot_b(s)));
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    mma_f16(tmem, da + uint64_t(A_MN ? 128 * k : 2 * k), db + uint64_t(128 * k), idesc,
                            (i | k) != 0);
                mma_commit(&empty[s]);
            }
            if (ok) {
                mma_commit(tfull);
            } else {
                // a load never landed: no accumulator for the epilogue, and before the CTA frees TMEM and exits,
                // every MMA this thread issued has completed
                mma_commit(drained);
                mbar_wait_limit(drained, 0u, kErrMmaWait, limit);
            }
        }
    } else if (warp >= 4) {
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;  // tile row = TMEM lane
        const int row = m0 + r;
        const bool ready = __all_sync(0xffffffffu, mbar_wait_limit(tfull, 0u, kErrMmaWait, limit));
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < BN / 32 && ready; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + (uint32_t(quarter * 32) << 16) + uint32_t(32 * c), v);
            tmem_ld_wait();
            if (row >= a.rows) continue;
            const int col0 = n0 + 32 * c;
#pragma unroll
            for (int g = 0; g < 8; ++g) {  // 4 columns at a time (cols is a multiple of 8)
                const int col = col0 + 4 * g;
                if (col >= a.cols) break;
                const float f0 = __uint_as_float(v[4 * g]), f1 = __uint_as_float(v[4 * g + 1]);
                const float f2 = __uint_as_float(v[4 * g + 2]), f3 = __uint_as_float(v[4 * g + 3]);
                if constexpr (SPLIT) {
                    *reinterpret_cast<float4*>(a.acc + ((long long)split * a.rows + row) * a.cols + col) =
                        make_float4(f0, f1, f2, f3);
                } else {
                    const T q[4] = {from_acc<T>(f0), from_acc<T>(f1), from_acc<T>(f2), from_acc<T>(f3)};
                    *reinterpret_cast<uint2*>(a.out + (long long)row * a.cols + col) =
                        *reinterpret_cast<const uint2*>(q);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, BN);
    }
}

// The weight gradient's second stage: out[i] = sum over s < splits, in order, of partial[s][i] (float32), converted
// to T; four elements a thread (elems is a multiple of 4: cols is a multiple of 8), the partials read eight splits
// at a time so that eight L2 round trips are in flight (the sum is still taken in split order).
constexpr int kReduceThreads = 128;
template <typename T>
__global__ void __launch_bounds__(kReduceThreads) grad_split_reduce_kernel(const float* __restrict__ partial,
                                                                           T* __restrict__ out, int splits,
                                                                           long long elems) {
    grid_dependency_wait();
    launch_dependents();
    const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i >= elems) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < splits; s0 += 8) {
        float4 x[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            x[u] = s0 + u < splits ? __ldcg(reinterpret_cast<const float4*>(partial + (long long)(s0 + u) * elems + i))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            acc.x += x[u].x; acc.y += x[u].y; acc.z += x[u].z; acc.w += x[u].w;
        }
    }
    const T q[4] = {from_acc<T>(acc.x), from_acc<T>(acc.y), from_acc<T>(acc.z), from_acc<T>(acc.w)};
    *reinterpret_cast<uint2*>(out + i) = *reinterpret_cast<const uint2*>(q);
}

// CUDA-core form (float32, float64, and 16-bit shapes the tensor-core kernel does not take): out[m, n] =
// sum over k of A(m, k) B(k, n), A(m, k) = a[m * sam + k * sak], B(k, n) = b[k * sbk + n * sbn]. 64 x 64 tiles,
// 16-deep K steps through shared memory, 4 x 4 outputs per thread. ATOMIC: the K range is split over blockIdx.z and
// the partial sums are added into `out` (float32 / float64 only; zero before the launch).
template <typename T>
struct GradSimtArgs {
    const T* a;
    const T* b;
    T* out;
    long long sam, sak, sbk, sbn;
    int rows, cols;
    long long K;
    long long k_per_split;  // a multiple of 16
};

template <typename T, bool ATOMIC>
__global__ void __launch_bounds__(256) grad_gemm_simt_kernel(const GradSimtArgs<T> p) {
    using A = typename Elem<T>::acc;
    __shared__ A sa[16][64 + 1];
    __shared__ A sb[16][64 + 1];
    grid_dependency_wait();
    launch_dependents();
    const int m0 = blockIdx.x * 64, n0 = blockIdx.y * 64;
    const long long k_begin = (long long)blockIdx.z * p.k_per_split;
    const long long k_end = min(k_begin + p.k_per_split, p.K);
    const int tid = threadIdx.x, tm = tid / 16, tn = tid % 16;
    A acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = A(0);
    for (long long k0 = k_begin; k0 < k_end; k0 += 16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e = tid + 256 * i;
            // A tile as [k][m]: consecutive threads walk m when A is MN-major (sam = 1), k otherwise
            const int kk = p.sam == 1 ? e / 64 : e % 16, mm = p.sam == 1 ? e % 64 : e / 16;
            const long long gk = k0 + kk;
            const int gm = m0 + mm;
            sa[kk][mm] = (gm < p.rows && gk < k_end) ? to_acc(p.a[gm * p.sam + gk * p.sak]) : A(0);
            const int kb = p.sbn == 1 ? e / 64 : e % 16, nn = p.sbn == 1 ? e % 64 : e / 16;
            const long long gkb = k0 + kb;
            const int gn = n0 + nn;
            sb[kb][nn] = (gn < p.cols && gkb < k_end) ? to_acc(p.b[gkb * p.sbk + gn * p.sbn]) : A(0);
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            A av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = sa[k][tm + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = sb[k][tn + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + tm + 16 * i;
        if (gm >= p.rows) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tn + 16 * j;
            if (gn >= p.cols) continue;
            T* dst = p.out + (long long)gm * p.cols + gn;
            if constexpr (ATOMIC) atomicAdd(dst, acc[i][j]);
            else *dst = from_acc<T>(acc[i][j]);
        }
    }
}

// Column sums of x [rows, cols] into float32 (float64 for float64) `sums` (zero before the launch): a thread owns
// one column of a block of rows and adds its partial sum with one atomic. With `out` set (16-bit types), the CTA
// whose arrival on its column block's counter (`arrivals`, zero before the launch) comes last converts that block's
// sums to the input type. The bias gradient of a linear layer.
template <typename T>
__global__ void __launch_bounds__(256) column_sum_kernel(const T* __restrict__ x, typename Elem<T>::acc* sums,
                                                         T* out, unsigned* arrivals, long long rows, int cols,
                                                         long long rows_per_cta) {
    using A = typename Elem<T>::acc;
    __shared__ unsigned last;
    grid_dependency_wait();
    launch_dependents();
    const long long r0 = (long long)blockIdx.y * rows_per_cta;
    const long long r1 = min(r0 + rows_per_cta, rows);
    const int c = blockIdx.x * 256 + threadIdx.x;
    if (c < cols) {
        A s0 = A(0), s1 = A(0), s2 = A(0), s3 = A(0);
        long long r = r0;
        for (; r + 4 <= r1; r += 4) {  // four rows' loads in flight
            s0 += to_acc(x[r * cols + c]);
            s1 += to_acc(x[(r + 1) * cols + c]);
            s2 += to_acc(x[(r + 2) * cols + c]);
            s3 += to_acc(x[(r + 3) * cols + c]);
        }
        for (; r < r1; ++r) s0 += to_acc(x[r * cols + c]);
        atomicAdd(sums + c, (s0 + s1) + (s2 + s3));
    }
    if (out == nullptr) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(arrivals + blockIdx.x, 1u) == gridDim.y - 1 ? 1u : 0u;
    __syncthreads();
    if (last != 0u && c < cols) {
        __threadfence();
        out[c] = from_acc<T>(__ldcg(sums + c));
    }
}

}  // namespace td
