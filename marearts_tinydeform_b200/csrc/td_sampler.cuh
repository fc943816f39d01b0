// td_sampler.cuh -- project order, sampling half: out[b,q,h,:] = sum_s w_s * value[b, tok_s, h, :].
//
// Same result as upstream sample_kernel (csrc/ma_deform_fused.cu:212-233), laid out for B200:
//   * one warp per (batch, query, head) row; the row's levels x points x 4 corners are computed once, by lanes in
//     parallel, into shared memory;
//   * the head slice of a corner row (D * e bytes) is read as G 16-byte vectors by G lanes (rows of 128 bytes and
//     more: 32-byte vectors, sm_100's 256-bit loads), so one warp keeps 32/G corner rows in flight at a time, and the
//     corner groups are summed with xor shuffles at the end; when the value is large against L2 the loads skip L1;
//   * value is addressed through (image, token, head) strides, so the same kernel reads the nn.Linear layout
//     [B, N, H*D] and the head-major [B, H, N, D] layout the projection kernel writes (x-adjacent corners are then
//     adjacent D-rows in memory).
// The generic kernel (any D, alignment or dtype, float64 included) keeps upstream's lanes-over-D mapping.
#pragma once

#include "td_common.cuh"
#include "td_producer.cuh"
#include "td_ptx.cuh"

namespace td {

template <typename T>
struct SampleArgs {
    const T* value;
    const T* loc;
    const T* attn;
    T* out;
    const int64_t* shapes;
    const int64_t* starts;
    long long rows;                 // B * Q * H
    long long s_img, s_tok, s_head; // value strides in elements
    long long n_tok;                // N
    const uint8_t* mask;            // value padding mask [B, N] (nonzero = padded) or null
    ProducerIn<T> prod;             // prod.proj set: locations and weights come from the query projection
    int Q, H, D, L, P;
    int G;                          // lanes per corner row = D * sizeof(T) / 16 (vector kernel only)
    int S_pad = 0;                  // two rows a warp: corner slots a row's lists hold, 4 L P rounded up to whole
                                    // batches (kBatch x 16 / G); the tail slots sample nothing
};

constexpr int kSampleWarps = 8;

// what a corner outside the map reads (16 or 32 bytes of zeros)
__device__ __align__(16) const uint4 g_zero16 = {0u, 0u, 0u, 0u};
__device__ __align__(32) const uint4 g_zero32[2] = {{0u, 0u, 0u, 0u}, {0u, 0u, 0u, 0u}};

// Read-only loads of corner rows. kNoAlloc: without L1 allocation -- on the DINO shape (91 MB of value, most of the
// 126 MB L2) the gather measured 5 % faster that way, while on the RT-DETR shapes (4-34 MB) it was 0.2-0.3 us
// slower, so the host picks it by the size of the value.
template <bool kNoAlloc>
__device__ __forceinline__ void ld_corner(const void* p, uint4 (&r)[1]) {
    if constexpr (kNoAlloc) {
        asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(r[0].x), "=r"(r[0].y), "=r"(r[0].z), "=r"(r[0].w)
                     : "l"(p));
    } else {
        r[0] = __ldg(static_cast<const uint4*>(p));
    }
}
// 32 bytes (sm_100 256-bit load), never allocating in L1; p is 32-byte aligned
template <bool kNoAlloc>
__device__ __forceinline__ void ld_corner(const void* p, uint4 (&r)[2]) {
    asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0].x), "=r"(r[0].y), "=r"(r[0].z), "=r"(r[0].w), "=r"(r[1].x), "=r"(r[1].y), "=r"(r[1].z),
                   "=r"(r[1].w)
                 : "l"(p));
}

// Dynamic shared memory of the vector kernel: per warp, S = 4 L P corner tokens and weights.
template <typename T>
__host__ __device__ inline size_t sample_vec_smem(int L, int P) {
    return size_t(kSampleWarps) * 4 * L * P * (sizeof(int) + sizeof(typename Coord<T>::type));
}

// The corners of one (batch, query, head) row into the warp's s_tok / s_wt (lanes over the L x P points).
template <typename T>
__device__ __forceinline__ void sample_row_corners(const SampleArgs<T>& a, long long row, int lane, int* s_tok,
                                                   typename Coord<T>::type* s_wt) {
    using CT = typename Coord<T>::type;
    const int LP = a.L * a.P;
    const uint8_t* mask_b = a.mask != nullptr ? a.mask + row / ((long long)a.Q * a.H) * a.n_tok : nullptr;
    if (a.prod.proj != nullptr) {  // the producer's softmax and locations, straight from the query projection
        using A = typename Elem<T>::acc;
        // the level geometry first: with prod.wait_first it is read before the dependency wait, with the reference
        // points, and the corners then follow proj by one round trip
        Level lv[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int j = lane + 32 * k;
            lv[k] = level_at(a.shapes, a.starts, j < LP ? level_of(j, a.P) : 0);
        }
        A lx[2], ly[2], w[2];
        produce_row<T, A>(a.prod, a.shapes, row, a.H, a.L, a.P, lane, lx, ly, w);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int j = lane + 32 * k;
            if (j < LP)
                corners4<CT>(CT(lx[k]), CT(ly[k]), CT(w[k]), lv[k], a.n_tok, &s_tok[4 * j], &s_wt[4 * j], mask_b);
        }
        return;
    }
    for (int j = lane; j < LP; j += 32) {
        const Level lv = level_at(a.shapes, a.starts, level_of(j, a.P));
        const long long i = row * LP + j;
        corners4<CT>(CT(to_acc(a.loc[2 * i])), CT(to_acc(a.loc[2 * i + 1])), CT(to_acc(a.attn[i])), lv, a.n_tok,
                     &s_tok[4 * j], &s_wt[4 * j], mask_b);
    }
}

// Corner rows in flight per lane (kBatch): a row's S = 4 L P corners are split over lanes / G lane groups (lanes =
// 32, or 16 for two rows a warp), each lane loading kBatch of its group's corners at once, in
// ceil(S / (kBatch * groups)) passes. In one wave of CTAs (every
// row resident at once, latency-bound) the fewest passes win: 48 corners over 8 groups in one pass of 6 (c1h 8.40 ->
// 7.99 us per call, against 8 slots of which a quarter fetched a zero row); 64 corners in two passes of 4 (as fast as
// one pass of 8 at DINO batch 1, 14.3 us). Over several waves (throughput-bound) the fewest empty slots at the
// smallest depth win, as smaller batches need fewer registers and so more resident CTAs: 48 corners in two passes of
// 3 (c3 31.5 -> 30.5 us), 64 in two of 4 (c4 93.4 -> 84.2 us, against one pass of 8 at 64 registers). The 32-byte
// forms (rows of 128 bytes and more) take 3 or 4, whichever leaves fewer empty slots. Two rows a warp (four groups
// of 64-byte rows) follow the same rule, which measured best there too: c1h 48 corners in two passes of 6; c3 in
// three of 4 and c4 in four of 4 (2, 6 and 8 slower at both).
inline int sample_batch_depth(int S, int G, bool wide, long long rows, int sm_count, int lanes = 32) {
    const int groups = lanes / G;
    auto passes = [&](int b) { return (S + b * groups - 1) / (b * groups); };
    auto slots = [&](int b) { return passes(b) * b * groups; };
    if (wide) return slots(3) < slots(4) ? 3 : 4;
    const long long wave_rows = (long long)sm_count * 5 * 8;  // five CTAs of eight rows on every SM
    if (rows <= wave_rows) {
        int best = 6;
        for (int b : {4, 3})
            if (passes(b) < passes(best) || (passes(b) == passes(best) && slots(b) < slots(best))) best = b;
        return best;
    }
    return slots(3) < slots(4) ? 3 : 4;
}

// The sum over the row's corners of weight * value[token] (head slice): G lanes per corner row, each loading
// 16 bytes of it (kWide: 32 bytes, for rows of 128 bytes and more -- half the load instructions, which measured 16 %
// faster on the stress shape's 128-byte rows and made no difference on 64-byte rows), kBatch corner rows in flight
// per lane, the lanes' groups summed with an xor butterfly. The row takes kLanes lanes (32, or 16 when a warp holds
// two rows; lane is then the index within the row's half). kPadded: the row's lists hold a.S_pad slots, whole
// batches, so no slot needs a bounds test. On return every lane holds the finished sum of its slice: head channels
// [(v * kWords + k) * V, + V) in acc[k * V ..], v = lane % G.
template <typename T, bool kWide, bool kNoAlloc, int kBatch, int kLanes = 32, bool kPadded = false>
__device__ __forceinline__ void sample_row_sum(const SampleArgs<T>& a, long long row, int lane, const int* s_tok_l,
                                               const typename Coord<T>::type* s_wt,
                                               typename Elem<T>::acc (&acc)[(kWide ? 2 : 1) * Elem<T>::kVec]) {
    using A = typename Elem<T>::acc;
    constexpr int V = Elem<T>::kVec;         // elements per 16-byte word
    constexpr int kWords = kWide ? 2 : 1;    // 16-byte words per lane and corner row
    const int S = 4 * a.L * a.P;
    int h;
    long long b;
    if (a.rows < (1LL << 31)) {  // 32-bit divisions where the row index allows
        const unsigned r = unsigned(row);
        h = int(r % unsigned(a.H));
        b = r / (unsigned(a.Q) * unsigned(a.H));
    } else {
        h = int(row % a.H);
        b = row / ((long long)a.Q * a.H);
    }
    const T* vb = a.value + b * a.s_img + (long long)h * a.s_head;
    const int G = a.G, CG = kLanes / G, cg = lane / G, v = lane - cg * G;
#pragma unroll
    for (int i = 0; i < kWords * V; ++i) acc[i] = A(0);
    const int s_end = kPadded ? a.S_pad : S;
    // the value stride of a token fits 32 bits (the host takes the vector kernels only then): a 32 x 32 -> 64-bit
    // product per corner
    const int s_tok = int(a.s_tok);
    for (int s0 = cg; s0 < s_end; s0 += kBatch * CG) {
        uint4 raw[kBatch][kWords];
        A w[kBatch];
        // every load of the batch is issued unconditionally (no branch between them, so they are all in flight
        // together): a corner outside the map, or past the row's last, reads a word of zeros
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int s = s0 + u * CG;
            int t = kPadded || s < S ? s_tok_l[s] : -1;
            TD_BOUNDS_TOKEN(t, a.n_tok);
            w[u] = kPadded || s < S ? A(s_wt[s]) : A(0);  // a corner outside the map already carries weight 0
            const void* src = t < 0 ? static_cast<const void*>(g_zero32)
                                    : static_cast<const void*>(vb + (long long)t * s_tok + v * kWords * V);
            ld_corner<kNoAlloc>(src, raw[u]);
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
#pragma unroll
            for (int k = 0; k < kWords; ++k) {
                A x[V];
                unpack16<T>(raw[u][k], x);
#pragma unroll
                for (int i = 0; i < V; ++i) acc[k * V + i] = fma(w[u], x[i], acc[k * V + i]);
            }
        }
    }
    for (int o = G; o < kLanes; o <<= 1) {
#pragma unroll
        for (int i = 0; i < kWords * V; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
    }
}

// out[row] = sample_row_sum, stored by the first corner group's lanes.
template <typename T, bool kWide, bool kNoAlloc, int kBatch>
__device__ __forceinline__ void sample_row_gather(const SampleArgs<T>& a, long long row, int lane, const int* s_tok,
                                                  const typename Coord<T>::type* s_wt) {
    using A = typename Elem<T>::acc;
    constexpr int V = Elem<T>::kVec;
    constexpr int kWords = kWide ? 2 : 1;
    A acc[kWords * V];
    sample_row_sum<T, kWide, kNoAlloc, kBatch>(a, row, lane, s_tok, s_wt, acc);
    if (lane < a.G) {
#pragma unroll
        for (int k = 0; k < kWords; ++k) store16<T>(a.out + row * a.D + (lane * kWords + k) * V, acc + k * V);
    }
}

// With prod.proj set, the corners come from the query projection (produce_row). Either that projection ran in the
// same launch as the value projection right before this kernel (prod.wait_first: the corner prologue waits for
// that launch between its reads of the reference points and of proj), or two launches earlier (query projection ->
// value projection -> this kernel): the value projection, launched with programmatic serialization, lets this
// kernel start only after its own grid dependency wait has seen the query projection complete, so the corner
// prologue may read proj before this kernel's own wait.
// Vector kernel: needs D * sizeof(T) % 16 == 0, D * sizeof(T) <= 512, 16-byte aligned value/out and strides (kWide:
// D * sizeof(T) a multiple of 32, 32-byte aligned value and strides).
// The dependent-latency chain is kept to two memory round trips: (level geometry + locations + attention weights,
// all issued together) -> corners -> (every corner row of the lane's group issued together) -> butterfly -> store.
// When launched with programmatic serialization right after the projection kernel, everything before
// grid_dependency_wait() overlaps that kernel; value is only read after it.
// Registers: the 16-byte forms of the 16- and 32-bit types are held to 48 (five CTAs an SM; no spills at any
// depth), the 32-byte forms to 64 (four CTAs; held to 48 they spill), float64 to 85 (three CTAs, no spills).
// The corners of a warp's two rows in one pass (kRW = 2): 16 lanes a row, a lane per sampling point (L * P <= 16;
// locations and weights read from the tensors, or produced from the query projection with a softmax over the row's
// 16 lanes), into lists of a.S_pad slots a row; a row past the last one and the tail slots sample nothing. The
// corner prologue is most of a row's instructions (level geometry, locations, clamps, four tokens and their bounds
// tests): a pass per row keeps only 12 of 32 lanes busy at the RT-DETR shapes' 12 points, this one 24.
template <typename T>
__device__ __forceinline__ void sample_pair_corners(const SampleArgs<T>& a, long long row0, int lane, int* s_tok,
                                                    typename Coord<T>::type* s_wt) {
    using CT = typename Coord<T>::type;
    const int LP = a.L * a.P, Sp = a.S_pad;
    const int r = lane >> 4, j = lane & 15;
    const long long row = row0 + r;
    for (int i = 4 * LP + j; i < Sp; i += 16) {  // the tail slots of the last batch
        s_tok[r * Sp + i] = -1;
        s_wt[r * Sp + i] = CT(0);
    }
    if (a.prod.proj != nullptr) {  // the producer's softmax and locations, straight from the query projection
        using A = typename Elem<T>::acc;
        const Level lv = level_at(a.shapes, a.starts, j < LP ? level_of(j, a.P) : 0);
        A lx[2], ly[2], w[2];
        // every lane takes part in its row's softmax; a row past the last one computes the last row's, unused
        const long long prow = row < a.rows ? row : a.rows - 1;
        produce_row<T, A, 16>(a.prod, a.shapes, prow, a.H, a.L, a.P, j, lx, ly, w);
        if (j >= LP) return;
        int* tk = s_tok + r * Sp + 4 * j;
        CT* wt = s_wt + r * Sp + 4 * j;
        if (row < a.rows) {
            const uint8_t* mask_b = a.mask != nullptr ? a.mask + row / ((long long)a.Q * a.H) * a.n_tok : nullptr;
            corners4<CT>(CT(lx[0]), CT(ly[0]), CT(w[0]), lv, a.n_tok, tk, wt, mask_b);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                tk[k] = -1;
                wt[k] = CT(0);
            }
        }
        return;
    }
    if (j >= LP) return;
    int* tk = s_tok + r * Sp + 4 * j;
    CT* wt = s_wt + r * Sp + 4 * j;
    if (row < a.rows) {
        const Level lv = level_at(a.shapes, a.starts, level_of(j, a.P));
        const uint8_t* mask_b = a.mask != nullptr ? a.mask + row / ((long long)a.Q * a.H) * a.n_tok : nullptr;
        const long long i = row * LP + j;
        corners4<CT>(CT(to_acc(a.loc[2 * i])), CT(to_acc(a.loc[2 * i + 1])), CT(to_acc(a.attn[i])), lv, a.n_tok, tk,
                     wt, mask_b);
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            tk[k] = -1;
            wt[k] = CT(0);
        }
    }
}

// Two rows a warp: corner slots a row's lists hold (whole batches of kBatch x 16 / G) and the dynamic shared memory.
inline int sample_pair_slots(int L, int P, int G, int batch) {
    const int step = batch * (16 / G);
    return (4 * L * P + step - 1) / step * step;
}
template <typename T>
inline size_t sample_pair_smem(int S_pad) {
    return size_t(kSampleWarps) * 2 * S_pad * (sizeof(int) + sizeof(typename Coord<T>::type));
}

// Whether a grid of `rows` sampler rows takes two rows a warp: the halved grid still gives every SM a CTA (2 x
// kSampleWarps rows a CTA), value rows of at most 16 load lanes, and points that fit 16 lanes. Measured on B200: c3
// 30.6 -> 27.1 us per call and c4 83.4 -> 72.7 (several waves, issue-bound), c1h 7.80 -> 7.66 (one wave); the layer
// with the producer in the prologue, c1h 10.14 -> 8.91 and c3 41.0 -> 29.9. With fewer rows (800 at batch 1 with 100
// queries: 50 CTAs) it measured slower, 7.25 -> 7.66 us.
inline bool sample_pair_form(long long rows, int G, long long L, long long P, int sm_count) {
    return rows >= 2LL * kSampleWarps * sm_count && G <= 16 && L * P <= 16;
}

// kRW rows per warp: 1, or 2 when the halved grid still fills the SMs and the rows' points fit 16 lanes -- the
// corner prologue in one pass for both rows, and each row's corner groups in one half
// of the warp (c3 30.6 -> 27.1 us per call, c4 83.4 -> 72.7 us on B200).
template <typename T, bool kWide, bool kNoAlloc, int kBatch, int kRW = 1>
__global__ void __launch_bounds__(kSampleWarps * 32, (!kWide && sizeof(T) < 8) ? 5 : (sizeof(T) == 8 ? 3 : 4))
    sample_vec_kernel(const SampleArgs<T> a) {
    using A = typename Elem<T>::acc;
    using CT = typename Coord<T>::type;
    constexpr int V = Elem<T>::kVec;
    constexpr int kWords = kWide ? 2 : 1;
    // per warp: kRW lists of corner tokens, then kRW lists of corner weights (dynamic: sample_vec_smem bytes, or
    // sample_pair_smem for two rows a warp, so that the CTAs stay small enough to become resident beside a running
    // projection kernel)
    extern __shared__ __align__(16) unsigned char smem_raw[];

    // the next call's projection may be scheduled now; it waits for this grid before touching memory
    launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = kRW == 1 ? 4 * a.L * a.P : a.S_pad;  // list slots a row
    int* s_tok = reinterpret_cast<int*>(smem_raw) + warp * kRW * S;
    CT* s_wt = reinterpret_cast<CT*>(smem_raw + kSampleWarps * kRW * S * sizeof(int)) + warp * kRW * S;
    if constexpr (kRW == 1) {
        const long long row = (long long)blockIdx.x * kSampleWarps + warp;
        const bool live = row < a.rows;  // dead warps still reach grid_dependency_wait
        if (live) sample_row_corners<T>(a, row, lane, s_tok, s_wt);
        __syncwarp();
        grid_dependency_wait();
        if (!live) return;
        sample_row_gather<T, kWide, kNoAlloc, kBatch>(a, row, lane, s_tok, s_wt);
    } else {
        static_assert(kRW == 2, "one or two rows a warp");
        const long long row0 = ((long long)blockIdx.x * kSampleWarps + warp) * 2;
        sample_pair_corners<T>(a, row0, lane, s_tok, s_wt);
        __syncwarp();
        grid_dependency_wait();
        if (row0 >= a.rows) return;
        const int r = lane >> 4, hl = lane & 15;
        A acc[kWords * V];
        sample_row_sum<T, kWide, kNoAlloc, kBatch, 16, true>(a, row0 + r, hl, s_tok + r * S, s_wt + r * S, acc);
        if (row0 + r < a.rows && hl < a.G) {
#pragma unroll
            for (int k = 0; k < kWords; ++k) store16<T>(a.out + (row0 + r) * a.D + (hl * kWords + k) * V, acc + k * V);
        }
    }
}

// Generic kernel: lanes over the head's D channels, scalar loads.
template <typename T>
__global__ void __launch_bounds__(kSampleWarps * 32) sample_generic_kernel(const SampleArgs<T> a) {
    using A = typename Elem<T>::acc;
    using CT = typename Coord<T>::type;
    __shared__ Level lv[kMaxLevels];
    __shared__ int s_tok[kSampleWarps][kMaxCorners];
    __shared__ CT s_wt[kSampleWarps][kMaxCorners];
    grid_dependency_wait();
    launch_dependents();
    load_levels(a.shapes, a.starts, a.L, lv);
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long row = (long long)blockIdx.x * kSampleWarps + warp;
    if (row >= a.rows) return;
    const int LP = a.L * a.P, S = 4 * LP;
    const uint8_t* mask_b = a.mask != nullptr ? a.mask + row / ((long long)a.Q * a.H) * a.n_tok : nullptr;
    if (a.prod.proj != nullptr) {
        A lx[2], ly[2], w[2];
        produce_row<T, A>(a.prod, a.shapes, row, a.H, a.L, a.P, lane, lx, ly, w);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int j = lane + 32 * k;
            if (j < LP)
                corners4<CT>(CT(lx[k]), CT(ly[k]), CT(w[k]), lv[level_of(j, a.P)], a.n_tok, &s_tok[warp][4 * j],
                             &s_wt[warp][4 * j], mask_b);
        }
    } else {
        for (int j = lane; j < LP; j += 32)
            row_corners(a.loc, a.attn, lv, LP, a.P, a.n_tok, row, j, &s_tok[warp][4 * j], &s_wt[warp][4 * j],
                        mask_b);
    }
    __syncwarp();

    const int h = int(row % a.H);
    const long long b = row / ((long long)a.Q * a.H);
    const T* vb = a.value + b * a.s_img + (long long)h * a.s_head;
    for (int d = lane; d < a.D; d += 32) {
        A acc = A(0);
        for (int s = 0; s < S; ++s) {
            int t = s_tok[warp][s];
            TD_BOUNDS_TOKEN(t, a.n_tok);
            if (t >= 0) acc = fma(A(s_wt[warp][s]), to_acc(vb[(long long)t * a.s_tok + d]), acc);
        }
        a.out[row * a.D + d] = from_acc<T>(acc);
    }
}

}  // namespace td
