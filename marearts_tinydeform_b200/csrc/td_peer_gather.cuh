// td_peer_gather.cuh -- the batch-sharded project order with the output all-gather fused into the sampler: every
// rank computes its own images' rows and stores each finished row into every rank's copy of the gathered output
// [B_global, Q, H * D] over NVLink (peer stores through CUDA IPC mappings), so the all-gather's bytes cross NVLink
// while the gather of the next rows is still in flight, and no separate collective runs afterwards. Completion: a
// one-warp kernel queued behind the sampler with programmatic dependent launch (resident early, released when the
// sampler's grid has completed and its stores are visible to it) makes those stores visible system-wide, writes the
// new epoch into this rank's slot of every peer's flag array, waits (bounded) until every peer's slot in its own
// array holds that epoch, and advances the rank's epoch. Epochs live in device memory, so the sequence can be
// captured in a CUDA graph and replayed; flags never need clearing.
//
// Per rank, one control block of kPeerCtrlWords 32-bit words (zeroed once at allocation): flags[kMaxPeers] (slot s =
// the last epoch rank s signalled to this rank), then the epoch.
#pragma once

#include "td_sampler.cuh"

namespace td {

constexpr int kMaxPeers = 8;
constexpr int kPeerCtrlWords = 16;
constexpr int kPeerEpochWord = kMaxPeers;

template <typename T>
struct PeerOut {
    T* out[kMaxPeers];          // every rank's gathered output (rank order), this rank's own included
    long long row0;             // this rank's first (batch, query, head) row in the gathered output
    int world, rank;
};

// Every rank's control block, as mapped in this process (passed by value).
struct PeerCtrl {
    unsigned* p[kMaxPeers];
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// sample_vec_kernel's rows (one or two a warp, the same form and sums), each stored into all `world` copies of the
// gathered output.
template <typename T, bool kWide, bool kNoAlloc, int kBatch, int kRW = 1>
__global__ void __launch_bounds__(kSampleWarps * 32) sample_peer_kernel(const SampleArgs<T> a, const PeerOut<T> p) {
    using A = typename Elem<T>::acc;
    using CT = typename Coord<T>::type;
    constexpr int V = Elem<T>::kVec;
    constexpr int kWords = kWide ? 2 : 1;
    extern __shared__ __align__(16) unsigned char smem_raw[];

    // the completion kernel may be scheduled now: it waits for this grid before it signals
    launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = kRW == 1 ? 4 * a.L * a.P : a.S_pad;  // list slots a row
    int* s_tok = reinterpret_cast<int*>(smem_raw) + warp * kRW * S;
    CT* s_wt = reinterpret_cast<CT*>(smem_raw + kSampleWarps * kRW * S * sizeof(int)) + warp * kRW * S;
    A acc[kWords * V];
    long long row;
    int hl;
    if constexpr (kRW == 1) {
        row = (long long)blockIdx.x * kSampleWarps + warp;
        const bool live = row < a.rows;
        if (live) sample_row_corners<T>(a, row, lane, s_tok, s_wt);
        __syncwarp();
        grid_dependency_wait();
        if (!live) return;
        hl = lane;
        sample_row_sum<T, kWide, kNoAlloc, kBatch>(a, row, lane, s_tok, s_wt, acc);
    } else {
        static_assert(kRW == 2, "one or two rows a warp");
        const long long row0 = ((long long)blockIdx.x * kSampleWarps + warp) * 2;
        sample_pair_corners<T>(a, row0, lane, s_tok, s_wt);
        __syncwarp();
        grid_dependency_wait();
        if (row0 >= a.rows) return;
        const int r = lane >> 4;
        hl = lane & 15;
        row = row0 + r;
        sample_row_sum<T, kWide, kNoAlloc, kBatch, 16, true>(a, row, hl, s_tok + r * S, s_wt + r * S, acc);
        if (row >= a.rows) return;
    }
    if (hl < a.G) {
        const long long at = (p.row0 + row) * a.D + (hl * kWords) * V;
        for (int r = 0; r < p.world; ++r) {
#pragma unroll
            for (int k = 0; k < kWords; ++k) store16<T>(p.out[r] + at + k * V, acc + k * V);
        }
    }
}

// One warp, behind the sampler (programmatic dependent launch): once the sampler's grid has completed, make its
// stores visible system-wide, signal the new epoch to every peer, then lane r waits until peer r has signalled it
// (at most `limit` clock cycles; a wait that runs out records kErrPeerWait in the library's error word), and lane 0
// advances this rank's epoch. signal = 0: wait only (tests).
__global__ void __launch_bounds__(32) peer_signal_wait_kernel(const PeerCtrl ctrl, int world, int rank, int signal,
                                                              long long limit) {
    const int lane = threadIdx.x;
    unsigned* mine = ctrl.p[rank];
    grid_dependency_wait();
    const unsigned e = *reinterpret_cast<volatile unsigned*>(mine + kPeerEpochWord) + 1u;
    if (signal) {
        __threadfence_system();  // cumulative: the sampler's stores, seen by this grid, before the flags
        __syncwarp();
        if (lane < world && lane != rank) st_release_sys(ctrl.p[lane] + rank, e);
    }
    if (lane < world && lane != rank) {
        const long long t0 = clock64();
        while (int(ld_acquire_sys(mine + lane) - e) < 0) {
            if (clock64() - t0 > limit) {
                record_error(kErrPeerWait);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncwarp();
    if (lane == 0) *reinterpret_cast<volatile unsigned*>(mine + kPeerEpochWord) = e;
}

}  // namespace td
