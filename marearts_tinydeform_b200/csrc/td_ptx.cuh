// td_ptx.cuh -- thin inline-PTX wrappers for the sm_100a features the tensor-core kernels use: mbarriers with
// bounded waits, TMA tile loads and stores (each CTA moves its own tiles), tcgen05 TMEM allocation, MMA, commit and
// loads, and the shared-memory / instruction descriptors of tcgen05.mma.
//
// Every wait here is bounded: after kSpinLimitCycles (about a second) it gives up, records the place in the
// library's device error word and returns false, so a wrong descriptor or byte count ends the kernel with an error
// status the host can read (td_device_error) instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace td {

// device error word: 0 = fine, otherwise the code of the first wait that timed out (see td_device_error)
__device__ unsigned int g_device_error = 0;

enum DeviceError : unsigned int {
    kErrNone = 0,
    kErrTmaWait = 1,      // a TMA load never completed its mbarrier
    kErrMmaWait = 2,      // an MMA commit never arrived
    kErrSlotWait = 3,     // a pipeline slot was never released
    kErrBounds = 4,       // TD_DEBUG_BOUNDS builds: a corner token outside [0, N) reached a gather or scatter
    kErrPeerWait = 5,     // the peer-gather wait: a peer rank never signalled its rows within the limit
};

constexpr long long kSpinLimitCycles = 2000000000LL;  // ~1 s at 1.9 GHz

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_error(unsigned int code) { atomicCAS(&g_device_error, 0u, code); }

// Checked builds (-DTD_DEBUG_BOUNDS, the library _tinydeform_debug.so): every corner token is tested against [0, n)
// where a kernel is about to read or write the token's row; a token outside it is recorded (kErrBounds) and turned
// into an outside corner (-1), so the access is skipped. The corner rule already keeps tokens inside [0, n); this
// re-checks that promise at every use. Ordinary builds compile the test away.
#ifdef TD_DEBUG_BOUNDS
#define TD_BOUNDS_TOKEN(t, n)                                                       \
    do {                                                                            \
        if ((t) >= 0 && (long long)(t) >= (long long)(n)) {                         \
            record_error(kErrBounds);                                               \
            (t) = -1;                                                               \
        }                                                                           \
    } while (0)
#else
#define TD_BOUNDS_TOKEN(t, n) \
    do {                      \
    } while (0)
#endif

// ---- mbarrier -----------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Non-blocking test: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait for the phase with the given parity to complete; false (and the error word set) after `limit` cycles.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, unsigned int err_code,
                                                long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) {
            record_error(err_code);
            return false;
        }
    }
    return true;
}

// Wait for the phase with the given parity to complete; false (and the error word set) after ~1 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int err_code) {
    return mbar_wait_limit(bar, parity, err_code, kSpinLimitCycles);
}

// ---- L2 eviction priority ---------------------------------------------------------------------------------
// Cache policies (createpolicy) for the .L2::cache_hint forms of the TMA copies below. evict_first marks data read
// once (the projection's input rows, which would otherwise push out what comes next); evict_last marks data read
// again soon (weights, read by every tile; the projected value, which the sampler gathers right after the
// projection). On the DINO shape (B = 8, 91 MB of value against a 126 MB L2) this took the project order from 114 to
// 109 us.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---- TMA ----------------------------------------------------------------------------------------------------
// 2-D tiled load of box (x = innermost, y) into shared memory, completing `bytes` on the mbarrier, with L2 cache
// policy `pol`. x * element size must be a multiple of 16 bytes (callers pass multiples of 64 elements).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "l"(pol)
        : "memory");
}

// 3-D tiled load of box (x, y, z), completing its bytes on the mbarrier. Same alignment rule on x.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5}], [%2], %6;"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z),
          "l"(pol)
        : "memory");
}

// 3-D tiled store of the box at (x, y, z) from shared memory, tracked by the issuing thread's bulk async-group.
// Elements of the box outside the tensor are not written. x * element size must be a multiple of 16 bytes and no
// coordinate may be negative.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z,
                                             uint64_t pol) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3, %4}], [%1], %5;"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(src)), "r"(x), "r"(y), "r"(z), "l"(pol)
                 : "memory");
}

// 32-byte store from registers (sm_100 256-bit vector store): one whole L2 sector per thread. dst is 32-byte aligned.
__device__ __forceinline__ void st_global_32b(void* dst, const uint4& lo, const uint4& hi, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8}, %9;"
                 ::"l"(dst), "r"(lo.x), "r"(lo.y), "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w),
                   "l"(pol)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk store of this thread has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Barrier among `count` threads (a multiple of 32) on hardware barrier `id` (1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Writes made with ordinary st.shared become visible to tcgen05.mma and TMA (the async proxy) after this fence.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- programmatic dependent launch ----------------------------------------------------------------------------
// In a kernel launched with programmatic stream serialization, wait until the preceding grid has completed and
// its memory is visible; a no-op when the kernel was launched normally.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream, if launched with programmatic serialization, to start its prologue now.
__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- thread-block clusters and distributed shared memory -----------------------------------------------------
// Rank of this CTA in its cluster (0 .. cluster size - 1).
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of the variable at shared::cta address `saddr` in the CTA of cluster rank `rank`.
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
// 16 bytes from the shared memory of a CTA of the cluster (16-byte aligned shared::cluster address).
__device__ __forceinline__ uint4 ld_cluster_v4(uint32_t caddr) {
    uint4 v;
    asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(caddr)
                 : "memory");
    return v;
}
// Cluster-wide barrier in two halves (every thread of every CTA of the cluster executes both, in order): arrive
// releases this thread's earlier shared-memory writes to the cluster, wait returns once every thread has arrived
// and acquires theirs. A hardware barrier, not a spin: the cluster's CTAs are co-scheduled by construction.
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Arrive without ordering this thread's earlier memory accesses (for a barrier that only marks that they are done).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

// ---- tcgen05: tensor memory ---------------------------------------------------------------------------------
// Executed by one whole warp. Writes the TMEM base address to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- tcgen05: MMA -------------------------------------------------------------------------------------------
// D[tmem] (+)= A[smem desc] x B[smem desc]^T, kind::f16 (f16 or bf16 inputs, f32 accumulator). One thread issues.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on the mbarrier when every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// Instruction descriptor for kind::f16: f32 accumulator, A and B K-major, M x N tile.
// Bits: [4,6) D format (1 = f32), [7,10) A format, [10,13) B format (0 = f16, 1 = bf16), [15] A MN-major,
// [16] B MN-major, [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N) {
    return (1u << 4) | (uint32_t(bf16) << 7) | (uint32_t(bf16) << 10) | (uint32_t(N >> 3) << 17) |
           (uint32_t(M >> 4) << 24);
}

// Shared-memory matrix descriptor of a K-major operand in the 128-byte-swizzle canonical layout: rows of 128 bytes
// (64 16-bit elements of K), 8-row atoms of 1024 bytes stacked along M/N (stride byte offset 1024), tile base
// 1024-byte aligned. Bits: [0,14) start >> 4, [16,30) leading byte offset >> 4 (unused here), [32,46) stride byte
// offset >> 4, [46,48) version = 1, [49,52) base offset = 0, [61,64) layout = 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= uint64_t((saddr & 0x3FFFFu) >> 4);
    d |= uint64_t(1024 >> 4) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// ---- tcgen05: TMEM -> registers -----------------------------------------------------------------------------
// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets row (lane base + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace td
