// td_gemm_tc.cuh -- value projection on tcgen05 tensor cores: value = memory @ W^T + b.
//
// Replaces the cuBLAS F.linear of upstream's project order (marearts_tinydeform/__init__.py:77) for float16 and
// bfloat16 (kind::f16) and for float32 (kind::tf32, three products per K step -- below).
// Output tiles are 128 tokens of one image x BN channels (a tile never spans two images, so every tile is a box of
// the [B, N, ...] tensors). Persistent and warp-specialised: each CTA walks tiles t = blockIdx.x, + gridDim.x, ...
// (channel tiles fastest, so the CTAs that share a 128-token slice of memory run together and it is read from HBM
// once):
//   * warp 0, two lanes per slot: TMA producers -- per tile and per 128-byte-wide K block, the 128-token slice of
//     memory (lane 2s) and the BN-row slice of W (lane 2s + 1), K-major with 128-byte swizzle, into slot s of a ring
//     of kStages shared-memory slots (memory with an L2 evict_first hint, W evict_last). The TMA operations of one
//     issuing thread are served one after another (about 0.15-0.3 us each on B200, whatever their size) while those
//     of different threads overlap, so every box of a ring round has its own issuer; a lane walks its slot's rounds
//     in order (so a parity wait on the slot's barrier never runs two phases ahead) and polls without blocking, so a
//     slot that is not free yet holds up no other. RES (resident weights): lane s loads only memory boxes, and
//     lanes S .. S + KB - 1 load the CTA's weight slice once;
//   * EPI warps from warp 4 on (8, or 16 for 256-wide tiles): epilogue -- tcgen05.ld of the accumulator (TMEM lane =
//     tile row; warp w reads lanes 32 (w % 4) .. + 31, and the EPI / 4 warps of a quarter split its columns), + bias
//     (double-buffered in shared memory), narrowed to T, and either stored straight from registers as 32-byte
//     pieces (direct32: each piece one whole L2 sector, evict_last, so the sampler finds the value in L2) or, for
//     outputs whose pieces would straddle heads, written into a staging tile laid out as the output's boxes (TMA
//     swizzle) and stored with TMA tensor stores by each warp as soon as it has staged them. The accumulator is
//     handed back as soon as it is read. STG = false: no staging tile (every job stores directly);
//   * warp 3, one thread: MMA issuer -- four K steps per block (tcgen05.mma, M = 128, N = BN) into one of two TMEM
//     accumulators (2 x BN float32 columns), so the epilogue of one tile runs under the MMAs of the next;
//   * float32 only, four more warps: split -- every landed slot is rewritten as hi = x with its 13 low mantissa bits
//     cleared (exact in TF32) and lo = x - hi in a second slot; the MMA issuer then accumulates
//     hi*hi + hi*lo + lo*hi, which keeps about 21 bits of each product where one TF32 product keeps 11.
// Every mbarrier wait is bounded (td_ptx.cuh): a wait that gives up records the device error word and that role
// stops issuing work, so a broken launch ends with an error status instead of a hang.
#pragma once

#include <type_traits>

#include "td_common.cuh"
#include "td_ptx.cuh"

namespace td {

// One projection of a launch. A launch runs one or two (the decoder layer's value projection and query projection
// share K and ride in one persistent grid: the second one's tiles follow the first one's).
template <typename T>
struct ProjJob {
    const T* bias;  // [HD] or null
    T* value;
    int N;            // tokens per image
    int HD, H, D;
    int head_major;
    int n_tiles;      // ceil(HD / BN)
    int m_tiles;      // ceil(N / 128): token tiles per image
    int tiles;        // B * m_tiles * n_tiles (< 2^31); 0 for an absent second job
    // epilogue through TMA stores: boxes of `piece` columns (piece_bytes = piece * sizeof(T) in {16, 32, 64, 128})
    // x 32 tokens, 0 = direct stores
    int tma_store, piece, piece_bytes;
    // direct32: each thread stores its row's 32-byte pieces straight from registers (value 32-byte aligned, every
    // 32-byte piece inside one head: D a power of two, D * sizeof(T) a multiple of 32); d_shift = log2(D)
    int direct32, d_shift;
};

template <typename T>
struct ProjTcArgs {
    ProjJob<T> job[2];
    int C;
    int k_blocks;     // ceil(C / kBK), the same for both jobs
    int tiles;        // job[0].tiles + job[1].tiles (< 2^31)
};

constexpr int kTcBM = 128;
// opt-in maximum, less the alignment slack, the barriers and 12 KB left for sampler CTAs on the same SM
constexpr int kTcSmemBudget = 232448 - 1024 - 512 - 12288;

template <typename T> struct GemmKind;
template <> struct GemmKind<__half> {
    static constexpr int kBK = 64;  // elements of one 128-byte swizzled row
    static constexpr bool kSplit = false;
    static constexpr uint32_t kFormat = 0;  // A / B format field: f16
};
template <> struct GemmKind<__nv_bfloat16> {
    static constexpr int kBK = 64;
    static constexpr bool kSplit = false;
    static constexpr uint32_t kFormat = 1;  // bf16
};
template <> struct GemmKind<float> {
    static constexpr int kBK = 32;
    static constexpr bool kSplit = true;
    static constexpr uint32_t kFormat = 2;  // tf32
};

// Resident-weight tiles (RES): every tile of a CTA has the same BN-row slice of W (the grid is a multiple of the
// channel-tile count and channel tiles run fastest), so the CTA loads that slice once, for all of its tiles, and the
// slot ring carries only memory boxes. A 128 x 256 tile that reloads its 128 KB of W reads 192 KB into the SM; a
// resident-weight 128 x 128 tile reads 64 KB. At most kResKBlocks K blocks (C <= 256 for 16-bit types).
constexpr int kResKBlocks = 4;

// STG: the layout holds a staging tile for TMA stores (jobs whose output the direct 32-byte stores cannot write);
// without it the slot ring gets the space.
template <typename T, int BN, int EPI, bool RES = false, bool STG = true>
struct ProjTcLayout {
    static constexpr bool kSplit = GemmKind<T>::kSplit;
    static constexpr bool kRes = RES;
    static constexpr int kBK = GemmKind<T>::kBK;
    static constexpr uint32_t kABytes = kTcBM * 128;  // 16 KB
    static constexpr uint32_t kBBytes = BN * 128;
    // a slot: the memory box and (unless the weights are resident) the weight box; float32: + the lo copies
    static constexpr uint32_t kStageBytes = RES ? kABytes : (kABytes + kBBytes) * (kSplit ? 2 : 1);
    static constexpr uint32_t kWBytes = RES ? kResKBlocks * kBBytes : 0;  // the resident weight slice
    static constexpr uint32_t kStgBytes = STG ? kTcBM * BN * sizeof(T) : 0;
    static constexpr uint32_t kBiasBytes = 2 * BN * 4;  // double-buffered: tile tc uses half tc & 1
    static constexpr int kFit = int((kTcSmemBudget - kStgBytes - kBiasBytes - kWBytes) / kStageBytes);
    static constexpr int kStages = kFit < 8 ? kFit : 8;  // two producer lanes a slot: at most 16
    static constexpr uint32_t kWOffset = kStages * kStageBytes;  // 1024-aligned: stage sizes are multiples of 1 KB
    static constexpr uint32_t kStgOffset = kWOffset + kWBytes;
    static constexpr uint32_t kBiasOffset = kStgOffset + kStgBytes;
    // barriers: full[S] (two arrivals: the memory and the weight box; one with resident weights), split[S],
    // empty[S], tfull[2], tempty[2], wfull (the resident weight slice: one arrival per K block)
    static constexpr uint32_t kBarOffset = kBiasOffset + kBiasBytes;
    static constexpr uint32_t kSlotOffset = kBarOffset + (3 * kStages + 5) * 8;
    static constexpr uint32_t kSmemBytes = kSlotOffset + 16 + 1024;  // + slack to align the base to 1024
    static constexpr uint32_t kTmemCols = 2 * BN;
    // warp 0 loads, warp 3 issues the MMAs, warps 4 .. 4+EPI-1 run the epilogue (a multiple of 4 apart, as epilogue
    // warp w reads TMEM lanes 32 (w % 4) ..), then the float32 split warps: whole groups of four warps, so that every
    // SM sub-partition holds the same share of the CTA's registers
    static constexpr int kMmaWarp = 3;
    static constexpr int kEpiWarp0 = 4;
    static constexpr int kSplitWarp0 = kEpiWarp0 + EPI;
    static constexpr int kThreads = 32 * (kSplitWarp0 + (kSplit ? 4 : 0));
    static_assert(BN == 64 || BN == 128 || BN == 256, "tile width");
    static_assert(EPI == 4 || EPI == 8 || EPI == 16, "epilogue warps");
    static_assert(BN * 4 / EPI >= 32, "every epilogue warp converts whole 32-column chunks");
    static_assert(kStages >= 2, "pipeline depth");
    static_assert(!RES || !kSplit, "resident weights: 16-bit types only");
    static_assert(!RES || !STG, "resident weights: direct stores only");
    static_assert(kSlotOffset + 16 <= uint32_t(kTcSmemBudget) + 512, "shared memory");
};

template <typename T>
__device__ __forceinline__ void mma_issue(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    if constexpr (GemmKind<T>::kSplit) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc)
            : "memory");
    } else {
        mma_f16(d, a, b, idesc, acc);
    }
}

// hi = x with the 13 low mantissa bits cleared, lo = x - hi (exact)
__device__ __forceinline__ void split_tf32(float4& x, float4& lo) {
    float4 h;
    h.x = __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
    h.y = __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
    h.z = __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
    h.w = __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
    lo = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
    x = h;
}

// 8 accumulator columns -> T, as 16-byte words (one for 16-bit types, two for float32)
template <typename T>
__device__ __forceinline__ void pack8(const float* f, uint4* w) {
    if constexpr (std::is_same<T, float>::value) {
        w[0] = make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
        w[1] = make_uint4(__float_as_uint(f[4]), __float_as_uint(f[5]), __float_as_uint(f[6]), __float_as_uint(f[7]));
    } else {
        uint32_t u[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (std::is_same<T, __half>::value) {
                const __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
                u[i] = *reinterpret_cast<const uint32_t*>(&h);
            } else {
                const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
                u[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
        }
        w[0] = make_uint4(u[0], u[1], u[2], u[3]);
    }
}

// The projection tiles of this CTA, from barrier setup to TMEM release (ends with a CTA-wide barrier; every value
// store of the CTA has completed by then). smem is the 1024-byte aligned dynamic shared memory.
template <typename T, int BN, int EPI, bool RES, bool STG>
__device__ __forceinline__ void proj_tc_tiles(const CUtensorMap& map_a0, const CUtensorMap& map_b0,
                                              const CUtensorMap& map_out0, const CUtensorMap& map_a1,
                                              const CUtensorMap& map_b1, const CUtensorMap& map_out1,
                                              const ProjTcArgs<T>& a, unsigned char* smem) {
    using Lay = ProjTcLayout<T, BN, EPI, RES, STG>;
    constexpr int S = Lay::kStages;
    constexpr int kBK = Lay::kBK;
    constexpr bool kSplit = Lay::kSplit;
    constexpr int kWords = sizeof(T) == 4 ? 2 : 1;  // 16-byte words per 8 columns
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lay::kBarOffset);
    uint64_t* split = full + S;
    uint64_t* empty = split + S;
    uint64_t* tfull = empty + S;
    uint64_t* tempty = tfull + 2;
    uint64_t* wfull = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::kSlotOffset);
    unsigned char* stg = smem + Lay::kStgOffset;
    float* sbias = reinterpret_cast<float*>(smem + Lay::kBiasOffset);
    // slot s: A (16 KB), B (BN x 128 B), and for float32 their lo halves after them
    auto slot_a = [&](int s) { return smem + s * Lay::kStageBytes; };
    auto slot_b = [&](int s) { return smem + s * Lay::kStageBytes + Lay::kABytes; };
    auto slot_alo = [&](int s) { return smem + s * Lay::kStageBytes + Lay::kABytes + Lay::kBBytes; };
    auto slot_blo = [&](int s) { return smem + s * Lay::kStageBytes + 2 * Lay::kABytes + Lay::kBBytes; };
    // the weight box of K block kb: from slot s, or from the resident slice
    auto b_tile = [&](int s, int kb) {
        return RES ? smem + Lay::kWOffset + kb * Lay::kBBytes : slot_b(s);
    };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = a.k_blocks;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], RES ? 1 : 2);
            mbar_init(&split[s], 4);  // one arrival per split warp
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], EPI);  // one arrival per epilogue warp
        }
        mbar_init(wfull, RES ? KB : 1);
        mbar_fence_init();
        tma_prefetch_desc(&map_a0);
        tma_prefetch_desc(&map_b0);
        if (a.job[0].tma_store) tma_prefetch_desc(&map_out0);
        if (a.job[1].tiles > 0) {
            tma_prefetch_desc(&map_a1);
            tma_prefetch_desc(&map_b1);
            if (a.job[1].tma_store) tma_prefetch_desc(&map_out1);
        }
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
    // tile t -> job j, image b, first token n0, first channel c0 (32-bit: the host keeps the tile count below 2^31)
    const int tiles0 = a.job[0].tiles;
    auto tile_at = [&](int t, int& j, int& b, int& n0, int& c0) {
        j = t >= tiles0;
        if (j) t -= tiles0;
        const int n_tiles = j ? a.job[1].n_tiles : a.job[0].n_tiles;
        const int per_img = (j ? a.job[1].m_tiles : a.job[0].m_tiles) * n_tiles;
        b = t / per_img;
        const int r = t - b * per_img;
        const int mt = r / n_tiles;
        n0 = mt * kTcBM;
        c0 = (r - mt * n_tiles) * BN;
    };
    const int my_tiles = a.tiles > int(blockIdx.x) ? (a.tiles - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
    // Under programmatic dependent launch everything up to a thread's first global access overlaps the previous
    // kernel in the stream: each role waits for it (grid_dependency_wait) right before its first global read or
    // write, after the set-up work and the first pass through its code. The MMA and split warps touch only shared
    // memory and TMEM, behind the producers. Dependents are released only after that wait (by the producer lanes):
    // the sampler that follows in the project order reads this call's locations and weights before its own wait,
    // so the kernels that wrote them must have completed.

    if (warp < Lay::kMmaWarp) {
        if (RES && warp == 0 && lane >= S && lane < S + KB) {
            // resident weights: lane S + kb loads K block kb of the CTA's weight slice, once
            if (my_tiles > 0) {
                int j, b, n0, c0;
                tile_at(int(blockIdx.x), j, b, n0, c0);
                const int kb = lane - S;
                grid_dependency_wait();
                launch_dependents();
                mbar_arrive_expect_tx(wfull, Lay::kBBytes);
                tma_load_2d(b_tile(0, kb), &map_b0, wfull, kb * kBK, c0, l2_evict_last());
            }
        } else if (warp == 0 && lane < (RES ? S : 2 * S)) {
            // TMA producer lane: slot s, the memory box (even lane; every lane s with resident weights) or the weight
            // box (odd lane) of the K blocks it = s, s + S, ... of this CTA's sequence (tile-major); then one more
            // round that only waits, so that no MMA commit is still to arrive on the slot when the CTA exits
            const int s = RES ? lane : lane >> 1;
            const bool box_a = RES || (lane & 1) == 0;
            const int total = my_tiles * KB;
            const uint64_t pol_a = l2_evict_first(), pol_w = l2_evict_last();
            long long t0 = clock64();
            bool waited = false;
            for (int it = s; it < total + S;) {
                if (mbar_test(&empty[s], uint32_t((it / S) & 1) ^ 1u)) {
                    if (it < total) {
                        const int tl = it / KB, kb = it - tl * KB;
                        int j, b, n0, c0;
                        tile_at(int(blockIdx.x) + tl * int(gridDim.x), j, b, n0, c0);
                        if (!waited) {
                            grid_dependency_wait();
                            launch_dependents();
                            waited = true;
                        }
                        if (box_a) {
                            mbar_arrive_expect_tx(&full[s], Lay::kABytes);
                            tma_load_3d(slot_a(s), j ? &map_a1 : &map_a0, &full[s], kb * kBK, n0, b, pol_a);
                        } else {
                            mbar_arrive_expect_tx(&full[s], Lay::kBBytes);
                            tma_load_2d(slot_b(s), j ? &map_b1 : &map_b0, &full[s], kb * kBK, c0, pol_w);
                        }
                    }
                    it += S;
                    t0 = clock64();
                } else if (clock64() - t0 > kSpinLimitCycles) {
                    record_error(kErrSlotWait);
                    break;
                } else {
                    __nanosleep(32);  // leave the issue slots to the epilogue warps of this sub-partition
                }
            }
        }
    } else if (warp == Lay::kMmaWarp) {
        if (lane == 0) {
            // MMA issuer. Instruction descriptor: f32 accumulator [4,6), A / B format [7,10) / [10,13), both K-major,
            // N >> 3 at [17,23), M >> 4 at [24,29).
            constexpr uint32_t idesc = (1u << 4) | (GemmKind<T>::kFormat << 7) | (GemmKind<T>::kFormat << 10) |
                                       (uint32_t(BN >> 3) << 17) | (uint32_t(kTcBM >> 4) << 24);
            int it = 0;
            // resident weights: the slice has landed before the first MMA
            bool ok = !RES || my_tiles == 0 || mbar_wait(wfull, 0u, kErrTmaWait);
            for (int tc = 0; ok && tc < my_tiles; ++tc) {
                const int acc = tc & 1;
                if (!mbar_wait(&tempty[acc], uint32_t((tc >> 1) & 1) ^ 1u, kErrSlotWait)) break;
                tc_fence_after();
                const uint32_t d = tmem + uint32_t(acc * BN);
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const int s = it % S;
                    if (!mbar_wait(kSplit ? &split[s] : &full[s], uint32_t((it / S) & 1), kErrTmaWait)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t da = sdesc_sw128(smem_addr(slot_a(s)));
                    const uint64_t db = sdesc_sw128(smem_addr(b_tile(s, kb)));
#pragma unroll
                    for (int k = 0; k < 4; ++k) {  // 4 K steps of 32 bytes per 128-byte row
                        const uint64_t kofs = uint64_t(2 * k);
                        mma_issue<T>(d, da + kofs, db + kofs, idesc, (kb | k) != 0);
                        if constexpr (kSplit) {
                            const uint64_t dal = sdesc_sw128(smem_addr(slot_alo(s)));
                            const uint64_t dbl = sdesc_sw128(smem_addr(slot_blo(s)));
                            mma_issue<T>(d, da + kofs, dbl + kofs, idesc, 1u);
                            mma_issue<T>(d, dal + kofs, db + kofs, idesc, 1u);
                        }
                    }
                    mma_commit(&empty[s]);
                }
                if (ok) mma_commit(&tfull[acc]);
            }
        }
    } else if (warp >= Lay::kEpiWarp0 && warp < Lay::kSplitWarp0) {
        // epilogue
        constexpr int kEpiThreads = EPI * 32;
        const int etid = threadIdx.x - 32 * Lay::kEpiWarp0;
        const int ew = warp - Lay::kEpiWarp0;
        const int quarter = warp & 3;
        constexpr int kCols = BN * 4 / EPI;  // columns this warp converts (EPI / 4 warps share each 32-row quarter)
        const int c_lo = (ew >> 2) * kCols;
        const int r = quarter * 32 + lane;  // tile row = TMEM lane
        const bool any_tma_store = STG && (a.job[0].tma_store || (a.job[1].tiles > 0 && a.job[1].tma_store));
        const uint64_t pol_out = l2_evict_last();  // the sampler reads the projected value right after
        // After a wait that gave up, a warp still walks its tiles and takes part in every named barrier (so no
        // other epilogue warp waits on it), but reads no TMEM and stores nothing.
        bool dead = false;
        // tc = -1 is a dry pass: the code below runs once on zeros into the staging tile, storing nothing, while the
        // first tile's loads are in flight -- so that its instructions are already cached when the tile is ready
        // (a first pass through cold code costs about as much as the loads).
        for (int tc = -1; tc < my_tiles; ++tc) {
            const bool dry = tc < 0;
            const int acc = tc & 1;
            int j, b, n0, c0;
            tile_at(int(blockIdx.x) + (dry ? 0 : tc) * int(gridDim.x), j, b, n0, c0);
            const ProjJob<T> J = j ? a.job[1] : a.job[0];
            const CUtensorMap* map_out = j ? &map_out1 : &map_out0;
            const int pb = J.piece_bytes;
            const int pshift = 31 - __clz(J.piece);  // piece is a power of two
            const int swz = pb / 16 - 1;             // 16-byte chunk index ^= (row * pb / 128) & swz
            if (tc == 0) grid_dependency_wait();  // the dry pass reads and writes no global memory
            // this tile's bias, in the half of the double buffer that tile tc - 2 used: every warp is past that
            // tile, as no warp has passed this tile's barrier below before all of them finished tile tc - 1
            float* const tbias = sbias + (tc & 1) * BN;
            for (int i = etid; i < BN; i += kEpiThreads)
                tbias[i] = (!dry && J.bias != nullptr && c0 + i < J.HD) ? to_acc(J.bias[c0 + i]) : 0.f;
            // the staging tile is free once the previous tile's stores have read it
            if (any_tma_store) bulk_wait_read();
            named_barrier(1, kEpiThreads);
            bool ready = dry || (!dead && mbar_wait(&tfull[acc], uint32_t((tc >> 1) & 1), kErrMmaWait));
            ready = __all_sync(0xffffffffu, ready);
            dead = !ready;
            tc_fence_after();
            const int n = n0 + r;
            const long long m = (long long)b * J.N + n;
            // first element of this thread's row at output column col (direct stores)
            auto out_at = [&](int col) -> T* {
                if (J.head_major) {
                    const int h = col >> J.d_shift;
                    return J.value + (((long long)b * J.H + h) * J.N + n) * J.D + (col - (h << J.d_shift));
                }
                return J.value + m * J.HD + col;
            };
#pragma unroll 1
            for (int j = 0; j < kCols / 32; ++j) {
                const int cl = c_lo + 32 * j;  // tile column of this chunk
                const bool live = ready && c0 + cl < J.HD;  // uniform across the warp
                uint32_t v[32];
                if (live && !dry) {
                    tmem_ld_32x32b_x32(tmem + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN + cl), v);
                    tmem_ld_wait();
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = 0u;
                }
                if (j == kCols / 32 - 1 && !dry) {
                    // every column of this warp is in registers: hand the accumulator back
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[acc]);
                }
                if (!live) continue;
                uint4 held = make_uint4(0u, 0u, 0u, 0u);  // direct32, 16-bit types: the first half of a piece
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const int c = cl + 8 * g;  // tile column
                    // the 8 bias values as two 16-byte shared-memory reads (sbias is 16-byte aligned, c a multiple
                    // of 8; every lane reads the same words: broadcast)
                    const float4 b0 = reinterpret_cast<const float4*>(tbias + c)[0];
                    const float4 b1 = reinterpret_cast<const float4*>(tbias + c)[1];
                    const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
                    float f[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(v[8 * g + i]) + bb[i];
                    uint4 w[kWords];
                    pack8<T>(f, w);
                    if (STG && J.tma_store) {
                        // piece p = c / piece, 16-byte chunk q within the piece's row r
                        const int p = c >> pshift, q = ((c - (p << pshift)) * int(sizeof(T))) >> 4;
                        unsigned char* row = stg + p * (kTcBM * pb) + r * pb;
                        const int x = (r * pb >> 7) & swz;
#pragma unroll
                        for (int k = 0; k < kWords; ++k) *reinterpret_cast<uint4*>(row + (((q + k) ^ x) << 4)) = w[k];
                    } else if (J.direct32) {
                        // whole 32-byte pieces: 16 columns of a 16-bit type (two groups), 8 of float32 (one group)
                        if constexpr (kWords == 1) {
                            if ((g & 1) == 0)
                                held = w[0];
                            else if (!dry && n < J.N && c0 + c - 8 < J.HD)
                                st_global_32b(out_at(c0 + c - 8), held, w[0], pol_out);
                        } else {
                            if (!dry && n < J.N && c0 + c < J.HD) st_global_32b(out_at(c0 + c), w[0], w[1], pol_out);
                        }
                    } else if (!dry && n < J.N && c0 + c < J.HD) {
                        const int col = c0 + c, h = col / J.D;
                        T* dst = J.head_major
                                     ? J.value + (((long long)b * J.H + h) * J.N + n) * J.D + (col - h * J.D)
                                     : J.value + m * J.HD + col;
#pragma unroll
                        for (int k = 0; k < kWords; ++k) reinterpret_cast<uint4*>(dst)[k] = w[k];
                    }
                }
            }
            if (STG && J.tma_store) {
                // this warp's boxes -- its columns [c_lo, c_lo + kCols) by its 32 rows -- as soon as it has staged
                // them, without waiting for the other epilogue warps
                fence_proxy_async_smem();  // the TMA stores (async proxy) read what these threads wrote
                __syncwarp();
                // one box per lane: the TMA operations of one thread are served one after another
                const int p = (c_lo >> pshift) + lane;
                const int col = c0 + (p << pshift);
                if (ready && !dry && p < ((c_lo + kCols) >> pshift) && col < J.HD) {
                    const unsigned char* src = stg + p * (kTcBM * pb) + quarter * 32 * pb;
                    if (J.head_major) {
                        const int h = col / J.D;
                        tma_store_3d(map_out, src, col - h * J.D, n0 + quarter * 32, b * J.H + h, l2_evict_last());
                    } else {
                        tma_store_3d(map_out, src, col, n0 + quarter * 32, b, l2_evict_last());
                    }
                    bulk_commit();
                }
            }
        }
        // the CTA may exit once its stores have read the staging tile; the grid completes only when they are written
        if (any_tma_store) bulk_wait_read();
    } else if (kSplit && warp >= Lay::kSplitWarp0) {
        // float32: split every landed slot into hi (in place) and lo
        const int tid = (warp - Lay::kSplitWarp0) * 32 + lane;  // 128 threads
        const int total = my_tiles * KB;
        for (int it = 0; it < total; ++it) {
            const int s = it % S;
            const bool landed = mbar_wait(&full[s], uint32_t((it / S) & 1), kErrTmaWait);
            if (!__all_sync(0xffffffffu, landed)) break;  // warp-uniform, for the __syncwarp below
            float4* x = reinterpret_cast<float4*>(slot_a(s));
            float4* xl = reinterpret_cast<float4*>(slot_alo(s));
#pragma unroll 4
            for (int i = tid; i < int(Lay::kABytes / 16); i += 128) {
                float4 v = x[i], lo;
                split_tf32(v, lo);
                x[i] = v;
                xl[i] = lo;
            }
            x = reinterpret_cast<float4*>(slot_b(s));
            xl = reinterpret_cast<float4*>(slot_blo(s));
#pragma unroll 4
            for (int i = tid; i < int(Lay::kBBytes / 16); i += 128) {
                float4 v = x[i], lo;
                split_tf32(v, lo);
                x[i] = v;
                xl[i] = lo;
            }
            fence_proxy_async_smem();  // the MMAs (async proxy) read what these threads wrote
            __syncwarp();
            if (lane == 0) mbar_arrive(&split[s]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();  // the producer lanes took different paths: converge for the .sync.aligned dealloc
        tc_fence_after();
        tmem_dealloc(tmem, Lay::kTmemCols);
    }
}

__device__ __forceinline__ unsigned char* align1024(unsigned char* p) {
    return p + ((1024 - (smem_addr(p) & 1023)) & 1023);
}

// 72 registers a thread (no spills): 12 warps, 3 per SM sub-partition (27 K registers), leave room on the SM for two
// CTAs of the sampler that follows in the project order (launched early, under programmatic dependent launch).
// Tensor maps of job 0 (memory, weight, output) and job 1 (the same; copies of job 0's when there is no job 1).
template <typename T, int BN, int EPI, bool RES, bool STG>
__global__ void __maxnreg__(72)
    proj_tc_kernel(const __grid_constant__ CUtensorMap map_a0, const __grid_constant__ CUtensorMap map_b0,
                   const __grid_constant__ CUtensorMap map_out0, const __grid_constant__ CUtensorMap map_a1,
                   const __grid_constant__ CUtensorMap map_b1, const __grid_constant__ CUtensorMap map_out1,
                   const ProjTcArgs<T> a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    proj_tc_tiles<T, BN, EPI, RES, STG>(map_a0, map_b0, map_out0, map_a1, map_b1, map_out1, a, align1024(smem_raw));
}

}  // namespace td
