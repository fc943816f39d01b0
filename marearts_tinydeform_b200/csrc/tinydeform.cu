// tinydeform.cu -- the C ABI (include/tinydeform.h): argument contract, kernel choice and launches.
//
// The argument contract mirrors upstream's check_geometry and weight/bias checks (csrc/ma_deform_fused.cu:235-266,
// :298-308, :333): levels x points <= 64, C <= 8192, N and B*Q*H within int32, HD a multiple of H. Tensor-level
// checks (ranks, dtypes, devices) live in the Python mirror, which only ever passes dense device pointers here.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <initializer_list>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "../../include/tinydeform.h"
#include "td_common.cuh"
#include "td_fused_simt.cuh"
#include "td_fused_tc.cuh"
#include "td_fused_warp.cuh"
#include "td_gemm_simt.cuh"
#include "td_gemm_tc.cuh"
#include "td_gemm_grad.cuh"
#include "td_producer.cuh"
#include "td_backward.cuh"
#include "td_sampler.cuh"
#include "td_sample_outproj.cuh"
#include "td_peer_gather.cuh"
#include "td_probe.cuh"

namespace td {
namespace {

std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_policy{TD_POLICY_BEST};
std::atomic<int> g_outproj_plan{TD_OUTPROJ_AUTO};

int fail(char* err, size_t err_len, int code, const char* fmt, ...) {
    if (err != nullptr && err_len > 0) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err, err_len, fmt, ap);
        va_end(ap);
    }
    return code;
}

int check_launch(char* err, size_t err_len, const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return TD_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

size_t dtype_size(int dtype) {
    switch (dtype) {
        case TD_F32: return 4;
        case TD_F16: return 2;
        case TD_BF16: return 2;
        case TD_F64: return 8;
        default: return 0;
    }
}

// Per-device facts, read once per device (the first call on a device should come before any graph capture,
// although every call made here is also legal during capture).
struct DeviceFacts {
    int sm_count = 0, major = 0, minor = 0, smem_optin = 0;
};

constexpr int kMaxDevices = 64;
std::atomic<bool> g_dev_known[kMaxDevices];
DeviceFacts g_dev[kMaxDevices];
std::mutex g_dev_mutex;

int device_facts(DeviceFacts* out, char* err, size_t err_len) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(err, err_len, TD_ERR_CUDA, "device index %d out of range", dev);
    if (!g_dev_known[dev].load(std::memory_order_acquire)) {
        // stored only once every query has succeeded; a failed query is retried by the next call
        std::lock_guard<std::mutex> lock(g_dev_mutex);
        if (!g_dev_known[dev].load(std::memory_order_relaxed)) {
            DeviceFacts f;
            e = cudaDeviceGetAttribute(&f.sm_count, cudaDevAttrMultiProcessorCount, dev);
            if (e == cudaSuccess) e = cudaDeviceGetAttribute(&f.major, cudaDevAttrComputeCapabilityMajor, dev);
            if (e == cudaSuccess) e = cudaDeviceGetAttribute(&f.minor, cudaDevAttrComputeCapabilityMinor, dev);
            if (e == cudaSuccess)
                e = cudaDeviceGetAttribute(&f.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
            if (e != cudaSuccess || f.sm_count <= 0) {
                cudaGetLastError();
                return fail(err, err_len, TD_ERR_CUDA, "could not query device %d: %s", dev, cudaGetErrorString(e));
            }
            g_dev[dev] = f;
            g_dev_known[dev].store(true, std::memory_order_release);
        }
    }
    *out = g_dev[dev];
    return TD_OK;
}

// Shared geometry checks (upstream check_geometry, csrc/ma_deform_fused.cu:236-266).
int check_geometry(int64_t B, int64_t Q, int64_t N, int64_t H, int64_t L, int64_t P, char* err, size_t err_len) {
    if (B < 0 || Q < 0 || N < 0 || L < 0 || P < 0)
        return fail(err, err_len, TD_ERR_ARG, "sizes must be non-negative");
    if (N > INT32_MAX) return fail(err, err_len, TD_ERR_ARG, "too many memory tokens");
    if (H <= 0) return fail(err, err_len, TD_ERR_ARG, "need at least one head");
    if (L > kMaxLevels || L * P > TD_MAX_LEVEL_POINTS)
        return fail(err, err_len, TD_ERR_ARG, "levels x points must be <= %d", TD_MAX_LEVEL_POINTS);
    if (double(B) * double(Q) * double(H) > double(INT32_MAX))
        return fail(err, err_len, TD_ERR_ARG, "too many (batch, query, head) rows");
    return TD_OK;
}

// Launch `kernel` on `stream`; with `pdl`, as a programmatic dependent launch: its CTAs may be scheduled while the
// previous kernel in the stream is still running, and the kernel's griddepcontrol.wait (which every kernel here
// executes before its first global memory access that could depend on earlier work) restores stream order.
template <typename K, typename... Args>
cudaError_t launch_kernel(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                          Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <typename T>
int launch_sampler(const T* value, long long s_img, long long s_tok, long long s_head, const int64_t* shapes,
                   const int64_t* starts, const T* loc, const T* attn, T* out, int64_t B, int64_t Q, int64_t N,
                   int64_t H, int64_t D, int64_t L, int64_t P, cudaStream_t stream, char* err, size_t err_len,
                   bool after_producer = false, const uint8_t* mask = nullptr, ProducerIn<T> prod = {}) {
    SampleArgs<T> a;
    a.value = value; a.loc = loc; a.attn = attn; a.out = out; a.shapes = shapes; a.starts = starts; a.prod = prod;
    a.rows = B * Q * H; a.s_img = s_img; a.s_tok = s_tok; a.s_head = s_head; a.n_tok = N; a.mask = mask;
    a.Q = int(Q); a.H = int(H); a.D = int(D); a.L = int(L); a.P = int(P);
    const long long row_bytes = D * (long long)sizeof(T);
    a.G = int(row_bytes / 16);
    // the corner groups of a warp are summed with an xor butterfly, so G must be a power of two dividing 32
    // (a token stride below 2^31 elements: the vector kernels form corner addresses with a 32 x 32-bit product)
    const bool vec = row_bytes % 16 == 0 && row_bytes <= 512 && (a.G & (a.G - 1)) == 0 && aligned16(value) &&
                     aligned16(out) && s_tok < (1LL << 31) &&
                     (s_img * (long long)sizeof(T)) % 16 == 0 && (s_tok * (long long)sizeof(T)) % 16 == 0 &&
                     (s_head * (long long)sizeof(T)) % 16 == 0;
    // 32-byte loads for rows of 128 bytes and more (G = row_bytes / 32 lanes a row, still a power of two)
    const bool wide = vec && row_bytes % 32 == 0 && row_bytes >= 128 && aligned32(value) &&
                      (s_img * (long long)sizeof(T)) % 32 == 0 && (s_tok * (long long)sizeof(T)) % 32 == 0 &&
                      (s_head * (long long)sizeof(T)) % 32 == 0;
    if (wide) a.G = int(row_bytes / 32);
    const unsigned grid = unsigned((a.rows + kSampleWarps - 1) / kSampleWarps);
    // Right after td_project_forward's projection kernel, launch with programmatic stream serialization: the
    // sampler's corner prologue then overlaps the projection, and it waits for it before reading value.
    const size_t smem = sample_vec_smem<T>(int(L), int(P));
    // corner loads without L1 allocation when the value is large against L2 (more than 64 MB)
    const bool no_alloc = vec && B * H * N * D * (long long)sizeof(T) > (64LL << 20);
    // corner rows in flight per lane (sample_batch_depth)
    int depth = 4;
    bool pair = false;
    if (vec) {
        DeviceFacts f;
        if (int rc = device_facts(&f, err, err_len)) return rc;
        // Two rows a warp (sample_vec_kernel's kRW = 2) when the halved grid still gives every SM a CTA and the
        // rows' points fit 16 lanes (sample_pair_form): the corner prologue then runs once for both rows.
        pair = sample_pair_form(a.rows, a.G, L, P, f.sm_count);
        depth = sample_batch_depth(int(4 * L * P), a.G, wide, a.rows, f.sm_count, pair ? 16 : 32);
    }
    auto vec_launch = [&](auto k_wide, auto k_noalloc) -> cudaError_t {
        constexpr bool W = decltype(k_wide)::value, NA = decltype(k_noalloc)::value;
        const dim3 blk(kSampleWarps * 32);
        if (pair) {
            const dim3 g2(unsigned((a.rows + 2 * kSampleWarps - 1) / (2 * kSampleWarps)));
            a.S_pad = sample_pair_slots(int(L), int(P), a.G, depth);
            const size_t ps = sample_pair_smem<T>(a.S_pad);
            if (depth == 3)
                return launch_kernel(sample_vec_kernel<T, W, NA, 3, 2>, g2, blk, ps, stream, after_producer, a);
            if (depth == 4)
                return launch_kernel(sample_vec_kernel<T, W, NA, 4, 2>, g2, blk, ps, stream, after_producer, a);
            if constexpr (!W)
                if (depth == 6)
                    return launch_kernel(sample_vec_kernel<T, W, NA, 6, 2>, g2, blk, ps, stream, after_producer, a);
            return cudaErrorInvalidValue;
        }
        const dim3 g(grid);
        if (depth == 3) return launch_kernel(sample_vec_kernel<T, W, NA, 3>, g, blk, smem, stream, after_producer, a);
        if (depth == 4) return launch_kernel(sample_vec_kernel<T, W, NA, 4>, g, blk, smem, stream, after_producer, a);
        if constexpr (!W) return launch_kernel(sample_vec_kernel<T, W, NA, 6>, g, blk, smem, stream, after_producer, a);
        return cudaErrorInvalidValue;
    };
    cudaError_t e = wide       ? vec_launch(std::true_type{}, std::true_type{})
                    : no_alloc ? vec_launch(std::false_type{}, std::true_type{})
                    : vec      ? vec_launch(std::false_type{}, std::false_type{})
                          : launch_kernel(sample_generic_kernel<T>, dim3(grid), dim3(kSampleWarps * 32), 0, stream,
                                          after_producer, a);
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "sampler launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, vec ? "sample_vec_kernel" : "sample_generic_kernel");
}

// The sampler with output_proj in the same kernel (sample_outproj_kernel, clusters of 4 or 8 CTAs): y [B * Q,
// C_out] = Wo . attention + bo, the attention never written to global memory. Returns TD_OK having launched it, or
// kNotApplicable (nothing launched) when the shapes, the alignment or the plan rule it out -- the caller then chains
// the sampler and the output GEMM. Under TD_OUTPROJ_AUTO it is taken while the kernel's grid is at most
// kOpAutoCtasPerSm CTAs per SM (one wave). There the chained GEMM is a second grid of a few CTAs behind a kernel
// boundary, which the cluster epilogue saves; in several waves each CTA's longer life (weight loads, cluster
// barriers, the product) is paid once per wave and the chained GEMM wins. Measured on B200, float16, RT-DETR levels,
// C_out = 256, graphs of 100 calls: B x Q = 1 x 50: 8.3 against 10.7 us chained; 1 x 100: 8.7 / 10.9;
// 1 x 300: 11.0 / 12.2; 2 x 300: 17.6 / 15.9; 8 x 300 (bfloat16): 46.6 / 38.1.
constexpr int kNotApplicable = -1000;
constexpr long long kOpAutoCtasPerSm = 3;

template <typename T>
int launch_sample_outproj(const T* value, long long s_img, long long s_tok, long long s_head, const int64_t* shapes,
                          const int64_t* starts, const T* loc, const T* attn, const T* out_w, const T* out_b, T* y,
                          int64_t C_out, int64_t B, int64_t Q, int64_t N, int64_t H, int64_t D, int64_t L, int64_t P,
                          cudaStream_t stream, char* err, size_t err_len, bool after_producer,
                          const uint8_t* mask = nullptr, ProducerIn<T> prod = {}) {
    const int plan = g_outproj_plan.load(std::memory_order_relaxed);
    if (plan == TD_OUTPROJ_CHAINED) return kNotApplicable;
    if (plan == TD_OUTPROJ_AUTO) {
        DeviceFacts f;
        if (int rc = device_facts(&f, err, err_len)) return rc;
        if ((B * Q * H + kSampleWarps - 1) / kSampleWarps > kOpAutoCtasPerSm * f.sm_count) return kNotApplicable;
    }
    const long long HD = H * D;
    const long long row_bytes = D * (long long)sizeof(T);
    const long long G = row_bytes / 16;
    const bool ok = kSampleWarps % H == 0 && HD * (long long)sizeof(T) == 512 &&
                    C_out <= 256 && row_bytes % 16 == 0 && row_bytes <= 512 &&
                    (G & (G - 1)) == 0 && aligned16(value) && aligned16(out_w) &&
                    (s_img * (long long)sizeof(T)) % 16 == 0 && (s_tok * (long long)sizeof(T)) % 16 == 0 &&
                    (s_head * (long long)sizeof(T)) % 16 == 0 && B * Q > 0;
    if (!ok) return kNotApplicable;
    SampleArgs<T> a;
    a.value = value; a.loc = loc; a.attn = attn; a.out = nullptr; a.shapes = shapes; a.starts = starts; a.prod = prod;
    a.rows = B * Q * H; a.s_img = s_img; a.s_tok = s_tok; a.s_head = s_head; a.n_tok = N; a.mask = mask;
    a.Q = int(Q); a.H = int(H); a.D = int(D); a.L = int(L); a.P = int(P); a.G = int(G);
    const bool wide = row_bytes % 32 == 0 && row_bytes >= 128 && aligned32(value) &&
                      (s_img * (long long)sizeof(T)) % 32 == 0 && (s_tok * (long long)sizeof(T)) % 32 == 0 &&
                      (s_head * (long long)sizeof(T)) % 32 == 0;
    if (wide) a.G = int(row_bytes / 32);
    const bool no_alloc = B * H * N * D * (long long)sizeof(T) > (64LL << 20);
    OutProjArgs<T> o;
    o.weight = out_w; o.bias = out_b; o.out = y; o.queries = B * Q; o.C_out = int(C_out); o.HD = int(HD);
    // clusters of 8 CTAs, each computing C_out / 8 output columns (clusters of 4 measured slower: twice the weight
    // loads per CTA; of 16, slower from two images on)
    constexpr int CS = kOpCluster;
    o.cols = int((C_out + CS - 1) / CS);
    DeviceFacts f;
    if (int rc = device_facts(&f, err, err_len)) return rc;
    // two rows a warp under the sampler's rule (sample_pair_form): a CTA then holds 16 rows, 16 / H whole queries
    const bool pair = sample_pair_form(a.rows, a.G, L, P, f.sm_count) && (2 * kSampleWarps) % H == 0;
    const int depth = sample_batch_depth(int(4 * L * P), a.G, wide, a.rows, f.sm_count, pair ? 16 : 32);
    if (pair) a.S_pad = sample_pair_slots(int(L), int(P), a.G, depth);
    const long long rows_per_cta = (pair ? 2 : 1) * kSampleWarps;
    const long long ctas = (B * Q * H + rows_per_cta - 1) / rows_per_cta;
    const unsigned grid = unsigned((ctas + CS - 1) / CS * CS);
    const size_t smem = sample_outproj_smem<T>(int(L), int(P), int(H), int(HD), CS, pair ? a.S_pad : 0);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kSampleWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = after_producer ? 2 : 1;
    auto op_launch = [&](auto k_wide, auto k_noalloc) -> cudaError_t {
        constexpr bool W = decltype(k_wide)::value, NA = decltype(k_noalloc)::value;
        if (pair) {
            if (depth == 3) return cudaLaunchKernelEx(&cfg, sample_outproj_kernel<T, W, NA, CS, 3, 2>, a, o);
            if (depth == 4) return cudaLaunchKernelEx(&cfg, sample_outproj_kernel<T, W, NA, CS, 4, 2>, a, o);
            if constexpr (!W) return cudaLaunchKernelEx(&cfg, sample_outproj_kernel<T, W, NA, CS, 6, 2>, a, o);
            return cudaErrorInvalidValue;
        }
        if (depth == 3) return cudaLaunchKernelEx(&cfg, sample_outproj_kernel<T, W, NA, CS, 3>, a, o);
        if (depth == 4) return cudaLaunchKernelEx(&cfg, sample_outproj_kernel<T, W, NA, CS, 4>, a, o);
        if constexpr (!W) return cudaLaunchKernelEx(&cfg, sample_outproj_kernel<T, W, NA, CS, 6>, a, o);
        return cudaErrorInvalidValue;
    };
    const cudaError_t e = wide       ? op_launch(std::true_type{}, std::true_type{})
                          : no_alloc ? op_launch(std::false_type{}, std::true_type{})
                                     : op_launch(std::false_type{}, std::false_type{});
    if (e != cudaSuccess)
        return fail(err, err_len, TD_ERR_CUDA, "sample_outproj_kernel launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "sample_outproj_kernel");
}

int tensor_map_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows, char* err,
                  size_t err_len, uint32_t elem_bytes = 2);
template <typename K>
int allow_smem(K kernel, size_t bytes, std::atomic<uint64_t>& done, char* err, size_t err_len);

// CTAs of `kernel` one SM holds at once, from its register count, its shared memory (dynamic + static + the
// per-block reservation) and the thread limit. At least 1.
template <typename K>
int resident_ctas(K kernel, int threads, size_t dyn_smem) {
    int dev = 0, regs_sm = 65536, smem_sm = 233472, reserved = 1024, threads_sm = 2048;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    cudaDeviceGetAttribute(&threads_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
    cudaFuncAttributes attr;
    if (cudaFuncGetAttributes(&attr, kernel) != cudaSuccess) return 1;
    const int regs_cta = ((attr.numRegs * 32 + 255) / 256 * 256) * (threads / 32);  // per-warp allocation unit
    const size_t smem_cta = dyn_smem + attr.sharedSizeBytes + size_t(reserved);
    int n = threads_sm / threads;
    if (regs_cta > 0) n = n < regs_sm / regs_cta ? n : regs_sm / regs_cta;
    const int by_smem = int(size_t(smem_sm) / smem_cta);
    n = n < by_smem ? n : by_smem;
    return n < 1 ? 1 : n;
}

template <typename T, int CV>
int launch_fused_tc_cfg(const CUtensorMap& map_w, const FusedTcArgs<T>& a, int sm_count, size_t smem,
                        cudaStream_t stream, char* err, size_t err_len) {
    static std::atomic<uint64_t> smem_done{0};
    auto kernel = fused_tc_kernel<T, CV>;
    if (int rc = allow_smem(kernel, smem, smem_done, err, err_len)) return rc;
    // one persistent CTA per SM, each with an equal share of the rows
    const int grid = int(a.rows < sm_count ? a.rows : sm_count);
    const cudaError_t e = launch_kernel(kernel, dim3(unsigned(grid)), dim3(kFtcThreads), smem, stream, true, map_w, a);
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "fused_tc_kernel launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "fused_tc_kernel");
}

// Fused order on the tensor cores; *launched stays false when the shapes do not fit it (the caller then uses the
// CUDA-core kernel).
template <typename T>
int launch_fused_tc(const T* memory, const T* weight, const T* bias, const int64_t* shapes, const int64_t* starts,
                    const T* loc, const T* attn, T* out, int64_t B, int64_t Q, int64_t N, int64_t C, int64_t H,
                    int64_t D, int64_t L, int64_t P, const uint8_t* mask, const DeviceFacts& f, cudaStream_t stream,
                    char* err, size_t err_len, bool* launched) {
    *launched = false;
    if (C > 1024 || 2 * D > 512) return TD_OK;
    const int S = int(4 * L * P);
    const int CV = C <= 256 ? 1 : (C <= 512 ? 2 : 4);
    const int pieces = fused_tc_pieces(S);
    const size_t smem = FusedTcLayout(int(C), int(D), S, pieces).bytes;
    if (smem > size_t(f.smem_optin) - 1024) return TD_OK;
    CUtensorMap map_w;
    if (int rc = tensor_map_2d(&map_w, weight, uint64_t(C), uint64_t(H * D), uint32_t(D), err, err_len)) return rc;
    FusedTcArgs<T> a;
    a.memory = memory; a.bias = bias; a.loc = loc; a.attn = attn; a.out = out; a.shapes = shapes; a.starts = starts;
    a.n_tok = N; a.mask = mask; a.rows = B * H * Q; a.B = int(B); a.Q = int(Q); a.C = int(C); a.H = int(H);
    a.D = int(D); a.L = int(L); a.P = int(P); a.pieces = pieces;
    *launched = true;
    if (CV == 1) return launch_fused_tc_cfg<T, 1>(map_w, a, f.sm_count, smem, stream, err, err_len);
    if (CV == 2) return launch_fused_tc_cfg<T, 2>(map_w, a, f.sm_count, smem, stream, err, err_len);
    return launch_fused_tc_cfg<T, 4>(map_w, a, f.sm_count, smem, stream, err, err_len);
}

// Fused order, one warp per row (td_fused_warp.cuh); *launched stays false when the shapes do not fit it: rows of
// C * e = 512, 1024 or 2048 bytes (2048-byte rows keep two rows in flight per lane, to fit 96 registers a thread at
// 20 warps per SM), D = 32 or 64, 16-byte aligned memory, weights and output.
template <typename T>
int launch_fused_warp(const FusedWarpArgs<T>& a, int64_t C, int64_t D, cudaStream_t stream, char* err, size_t err_len,
                      bool* launched) {
    *launched = false;
    const int64_t row_bytes = C * int64_t(sizeof(T));
    if ((row_bytes != 512 && row_bytes != 1024 && row_bytes != 2048) || (D != 32 && D != 64) || !aligned16(a.memory) ||
        !aligned16(a.weight) || !aligned16(a.out))
        return TD_OK;
    const int CV = int(row_bytes / 512);
    const dim3 grid(unsigned((a.rows + kFwWarps - 1) / kFwWarps));
    auto go = [&](auto kernel) {
        *launched = true;
        const cudaError_t e = launch_kernel(kernel, grid, dim3(kFwWarps * 32), 0, stream, true, a);
        if (e != cudaSuccess)
            return fail(err, err_len, TD_ERR_CUDA, "fused_warp_kernel launch: %s", cudaGetErrorString(e));
        g_launches.fetch_add(1, std::memory_order_relaxed);
        return check_launch(err, err_len, "fused_warp_kernel");
    };
    // 512-byte rows in a grid of at most 8 rows per SM take the deeper corner batch (fused_warp_kernel's kDeep)
    DeviceFacts f;
    if (int rc = device_facts(&f, err, err_len)) return rc;
    const bool deep = CV == 1 && a.rows <= 8LL * f.sm_count;
    if (D == 32) {
        if (CV == 1) return deep ? go(fused_warp_kernel<T, 1, 1, true>) : go(fused_warp_kernel<T, 1, 1>);
        return CV == 2 ? go(fused_warp_kernel<T, 2, 1>) : go(fused_warp_kernel<T, 4, 1>);
    }
    if (CV == 1) return deep ? go(fused_warp_kernel<T, 1, 2, true>) : go(fused_warp_kernel<T, 1, 2>);
    return CV == 2 ? go(fused_warp_kernel<T, 2, 2>) : go(fused_warp_kernel<T, 4, 2>);
}

template <typename T>
int launch_fused(const T* memory, const T* weight, const T* bias, const int64_t* shapes, const int64_t* starts,
                 const T* loc, const T* attn, T* out, int64_t B, int64_t Q, int64_t N, int64_t C, int64_t H,
                 int64_t D, int64_t L, int64_t P, cudaStream_t stream, char* err, size_t err_len,
                 const uint8_t* mask = nullptr) {
    using A = typename Elem<T>::acc;
    DeviceFacts f;
    if (int rc = device_facts(&f, err, err_len)) return rc;
    if constexpr (!std::is_same<T, double>::value) {
        if (g_policy.load(std::memory_order_relaxed) == TD_POLICY_BEST) {
            FusedWarpArgs<T> w;
            w.memory = memory; w.weight = weight; w.bias = bias; w.loc = loc; w.attn = attn; w.out = out;
            w.shapes = shapes; w.starts = starts; w.mask = mask; w.n_tok = N; w.rows = B * H * Q;
            w.Q = int(Q); w.C = int(C); w.H = int(H); w.L = int(L); w.P = int(P);
            bool launched = false;
            const int rc = launch_fused_warp<T>(w, C, D, stream, err, err_len, &launched);
            if (rc != TD_OK || launched) return rc;
        }
    }
    if constexpr (std::is_same<T, __half>::value || std::is_same<T, __nv_bfloat16>::value) {
        // tcgen05 path: N = D a multiple of 16, whole 64-wide K blocks, 16-byte aligned rows and outputs
        if (g_policy.load(std::memory_order_relaxed) == TD_POLICY_BEST && D % 16 == 0 && D <= 256 && C % 64 == 0 &&
            aligned16(memory) && aligned16(weight) && aligned16(out)) {
            bool launched = false;
            const int rc = launch_fused_tc<T>(memory, weight, bias, shapes, starts, loc, attn, out, B, Q, N, C, H, D,
                                              L, P, mask, f, stream, err, err_len, &launched);
            if (rc != TD_OK || launched) return rc;
        }
    }
    const int S = int(4 * L * P);
    // rows per CTA: up to 16 queries of one (batch, head), fewer when that leaves SMs idle or m does not fit
    int R = kFusedMaxRows;
    while (R > 1 && B * H * ((Q + R - 1) / R) < 2LL * f.sm_count) R >>= 1;
    const size_t smem_cap = size_t(f.smem_optin) - 2048;
    while (R > 1 && fused_simt_smem<T>(R, int(C), S) > smem_cap) R >>= 1;
    const size_t smem = fused_simt_smem<T>(R, int(C), S);
    if (smem > smem_cap) return fail(err, err_len, TD_ERR_ARG, "channels too large for shared memory");
    FusedArgs<T> a;
    a.memory = memory; a.weight = weight; a.bias = bias; a.loc = loc; a.attn = attn; a.out = out;
    a.shapes = shapes; a.starts = starts; a.n_tok = N; a.mask = mask;
    a.B = int(B); a.Q = int(Q); a.C = int(C); a.H = int(H); a.D = int(D); a.L = int(L); a.P = int(P);
    a.R = R; a.q_tiles = int((Q + R - 1) / R);
    a.vec = (C % Elem<T>::kVec == 0) && aligned16(memory);
    (void)sizeof(A);
    static std::atomic<uint64_t> smem_done{0};
    if (int rc = allow_smem(fused_simt_kernel<T>, smem, smem_done, err, err_len)) return rc;
    const long long grid = B * H * (long long)a.q_tiles;
    const cudaError_t e = launch_kernel(fused_simt_kernel<T>, dim3(unsigned(grid)), dim3(kFusedThreads), smem, stream,
                                        true, a);
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "fused_simt_kernel launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "fused_simt_kernel");
}

// cuTensorMapEncodeTiled, reached through the runtime so the library does not link libcuda directly.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// cuTensorMapEncodeTiled on the calling thread. A thread on which the CUDA runtime has not yet made a context
// current (autograd's worker thread, for one, when its device is the runtime's default) gets
// CUDA_ERROR_INVALID_CONTEXT from the driver; the thread's current device's primary context is then made current
// (cudaSetDevice, no stream work, legal during capture) and the encoding tried once more.
CUresult encode_tiled(CUtensorMap* map, CUtensorMapDataType type, cuuint32_t rank, void* base,
                      const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                      const cuuint32_t* estr, CUtensorMapSwizzle swizzle) {
    auto encode = tensor_map_encoder();
    if (encode == nullptr) return CUDA_ERROR_NOT_FOUND;
    CUresult r = encode(map, type, rank, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_ERROR_INVALID_CONTEXT) {
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess)
            r = encode(map, type, rank, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        cudaGetLastError();
    }
    return r;
}

// 2-D row-major tensor [rows, cols] of 16-bit (or 32-bit) elements, 128-byte-swizzled boxes of box_rows rows x
// 128 bytes (64 or 32 elements).
int tensor_map_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows, char* err,
                  size_t err_len, uint32_t elem_bytes) {
    if (tensor_map_encoder() == nullptr)
        return fail(err, err_len, TD_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * elem_bytes};
    const cuuint32_t box[2] = {128u / elem_bytes, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType type = elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    const CUresult r = encode_tiled(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
                                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (r != CUDA_SUCCESS) return fail(err, err_len, TD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
    return TD_OK;
}

// 3-D tensor (x innermost) of 16- or 32-bit elements with byte strides for y and z, boxes of box[0..2] elements and
// the given shared-memory swizzle.
int tensor_map_3d(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides[2],
                  const uint32_t box[3], uint32_t elem_bytes, CUtensorMapSwizzle swizzle, char* err, size_t err_len) {
    if (tensor_map_encoder() == nullptr)
        return fail(err, err_len, TD_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
    const cuuint64_t st[2] = {strides[0], strides[1]};
    const cuuint32_t bx[3] = {box[0], box[1], box[2]};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType type = elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    const CUresult r = encode_tiled(map, type, 3, const_cast<void*>(base), d, st, bx, estr, swizzle);
    if (r != CUDA_SUCCESS) return fail(err, err_len, TD_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", int(r));
    return TD_OK;
}

// Raise a kernel's dynamic shared memory limit once per device.
template <typename K>
int allow_smem(K kernel, size_t bytes, std::atomic<uint64_t>& done, char* err, size_t err_len) {
    // the limit is raised to the device's opt-in maximum (less the kernel's static shared memory) once, so later
    // calls may ask for any size up to it
    DeviceFacts f;
    if (int rc = device_facts(&f, err, err_len)) return rc;
    cudaFuncAttributes attr;
    cudaError_t e = cudaFuncGetAttributes(&attr, kernel);
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
    const int dyn_max = f.smem_optin - int(attr.sharedSizeBytes);
    if (bytes > size_t(dyn_max))
        return fail(err, err_len, TD_ERR_ARG, "%zu bytes of shared memory needed, %d available", bytes, dyn_max);
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = uint64_t(1) << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return TD_OK;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn_max);
    // the whole unified L1 / shared array as shared memory, so several CTAs of a kernel fit on one SM
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    done.fetch_or(bit, std::memory_order_acq_rel);
    return TD_OK;
}

#ifndef TD_EPI_DIRECT
#define TD_EPI_DIRECT 1  // 0: the projection epilogue always stages tiles for TMA stores (for comparison builds)
#endif

// Whether the projection epilogue can write value with direct 32-byte stores (ProjJob::direct32): a 32-byte aligned
// value whose rows split into 32-byte pieces that each lie inside one head (D a power of two, D * e a multiple of 32)
// when head-major.
inline bool proj_direct32(const void* value, int64_t HD, int64_t D, int head_major, int64_t e) {
    if (!TD_EPI_DIRECT || reinterpret_cast<uintptr_t>(value) % 32 != 0 || (HD * e) % 32 != 0) return false;
    return !head_major || ((D & (D - 1)) == 0 && (D * e) % 32 == 0);
}

// One projection of the tcgen05 kernel: value[B, N, HD] (or head-major [B, H, N, D]) = memory[B, N, C] @ W^T + b.
struct ProjShape {
    const void* memory;
    const void* weight;
    const void* bias;
    void* value;
    int64_t B, N, C, H, HD;
    int head_major;
};

// Tensor maps and arguments of one job of the tcgen05 projection kernel.
template <typename T, int BN, int EPI>
int prepare_proj_tc(const ProjShape& ps, CUtensorMap* map_a, CUtensorMap* map_b, CUtensorMap* map_out,
                    ProjJob<T>* job, char* err, size_t err_len) {
    constexpr uint32_t e = sizeof(T);
    const T* memory = static_cast<const T*>(ps.memory);
    const T* weight = static_cast<const T*>(ps.weight);
    const int64_t B = ps.B, N = ps.N, C = ps.C, H = ps.H, HD = ps.HD;
    const int head_major = ps.head_major;
    T* value = static_cast<T*>(ps.value);
    const int64_t D = HD / H;
    {
        // memory as [B][N][C]: 128-token boxes never cross into the next image (rows past N read as zeros)
        const uint64_t dims[3] = {uint64_t(C), uint64_t(N), uint64_t(B)};
        const uint64_t strides[2] = {uint64_t(C) * e, uint64_t(N * C) * e};
        const uint32_t box[3] = {128u / e, uint32_t(kTcBM), 1u};
        if (int rc = tensor_map_3d(map_a, memory, dims, strides, box, e, CU_TENSOR_MAP_SWIZZLE_128B, err, err_len))
            return rc;
    }
    if (int rc = tensor_map_2d(map_b, weight, uint64_t(C), uint64_t(HD), BN, err, err_len, e)) return rc;
    // Epilogue boxes: `piece` columns x 32 tokens. Head-major value [B, H, N, D]: a piece is a head, or a 128-byte
    // part of one; [B, N, HD]: 128-byte column groups. The row of a box must be 16, 32, 64 or 128 bytes (the TMA
    // swizzle widths that keep the staging writes free of bank conflicts).
    // Direct 32-byte stores from the epilogue's registers when every 32-byte piece of a row lies inside one head (and
    // the value is 32-byte aligned): cheaper than staging the tile in shared memory for TMA stores, which cost about
    // as much per tile as the MMAs.
    const int direct32 = proj_direct32(value, HD, D, head_major, e) ? 1 : 0;
    int d_shift = 0;
    if (direct32 && head_major)
        while ((int64_t(1) << d_shift) < D) ++d_shift;
    int piece = 0;
    if (direct32) {
        piece = 0;
    } else if (head_major) {
        const int64_t db = D * e;
        if (db == 16 || db == 32 || db == 64 || db == 128) piece = int(D);
        else if (db % 128 == 0) piece = int(128 / e);
    } else {
        piece = int(128 / e);
    }
    const int piece_bytes = piece * int(e);
    *map_out = *map_b;  // unused when the epilogue stores directly
    if (piece) {
        const CUtensorMapSwizzle sw = piece_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                      : piece_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                      : piece_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                          : CU_TENSOR_MAP_SWIZZLE_NONE;
        const uint32_t box[3] = {uint32_t(piece), 32u, 1u};  // one epilogue warp's rows
        if (head_major) {
            const uint64_t dims[3] = {uint64_t(D), uint64_t(N), uint64_t(B * H)};
            const uint64_t strides[2] = {uint64_t(D) * e, uint64_t(N * D) * e};
            if (int rc = tensor_map_3d(map_out, value, dims, strides, box, e, sw, err, err_len)) return rc;
        } else {
            const uint64_t dims[3] = {uint64_t(HD), uint64_t(N), uint64_t(B)};
            const uint64_t strides[2] = {uint64_t(HD) * e, uint64_t(N * HD) * e};
            if (int rc = tensor_map_3d(map_out, value, dims, strides, box, e, sw, err, err_len)) return rc;
        }
    }
    ProjJob<T>& a = *job;
    a.bias = static_cast<const T*>(ps.bias); a.value = value; a.N = int(N); a.HD = int(HD); a.H = int(H);
    a.D = int(D); a.head_major = head_major;
    a.direct32 = direct32;
    a.d_shift = d_shift;
    a.n_tiles = int((HD + BN - 1) / BN);
    a.m_tiles = int((N + kTcBM - 1) / kTcBM);
    a.tiles = int(B * a.m_tiles * a.n_tiles);
    a.tma_store = piece != 0; a.piece = piece ? piece : 8; a.piece_bytes = piece ? piece_bytes : 16;
    return TD_OK;
}

// One launch of the tcgen05 projection kernel for job0 and, when job1 is not null, job1 (same C): job1's tiles
// follow job0's in the persistent grid. RES: resident weight slices (job0 alone, at most kResKBlocks K blocks).
// STG = false: no staging tile (every job stores directly).
template <typename T, int BN, int EPI, bool RES = false, bool STG = true>
int launch_proj_tc(const ProjShape& job0, const ProjShape* job1, cudaStream_t stream, bool pdl, char* err,
                   size_t err_len) {
    using Lay = ProjTcLayout<T, BN, EPI, RES, STG>;
    static std::atomic<uint64_t> smem_done{0};
    DeviceFacts f;
    if (int rc = device_facts(&f, err, err_len)) return rc;
    CUtensorMap map_a0, map_b0, map_out0, map_a1, map_b1, map_out1;
    ProjTcArgs<T> a;
    if (int rc = prepare_proj_tc<T, BN, EPI>(job0, &map_a0, &map_b0, &map_out0, &a.job[0], err, err_len)) return rc;
    if (job1 != nullptr) {
        if (int rc = prepare_proj_tc<T, BN, EPI>(*job1, &map_a1, &map_b1, &map_out1, &a.job[1], err, err_len))
            return rc;
    } else {
        map_a1 = map_a0; map_b1 = map_b0; map_out1 = map_out0;
        a.job[1] = a.job[0];
        a.job[1].tiles = 0;
    }
    a.C = int(job0.C);
    a.k_blocks = int((job0.C + Lay::kBK - 1) / Lay::kBK);
    a.tiles = a.job[0].tiles + a.job[1].tiles;
    if (RES && (job1 != nullptr || a.k_blocks > kResKBlocks))
        return fail(err, err_len, TD_ERR_ARG, "resident-weight projection: one job of at most %d K blocks",
                    kResKBlocks);
    if (!STG && (!a.job[0].direct32 || (job1 != nullptr && !a.job[1].direct32)))
        return fail(err, err_len, TD_ERR_ARG, "projection without a staging tile: every job must store directly");
    if (int rc = allow_smem(proj_tc_kernel<T, BN, EPI, RES, STG>, Lay::kSmemBytes, smem_done, err, err_len))
        return rc;
    // persistent: at most one CTA per SM (the slot ring takes most of the shared memory). With resident weights the
    // grid is a multiple of the channel-tile count, so that every tile of a CTA has the same channel tile (the tile
    // count itself is one, when it is the smaller).
    const int cap = RES ? f.sm_count - f.sm_count % a.job[0].n_tiles : f.sm_count;
    if (cap <= 0)
        return fail(err, err_len, TD_ERR_ARG, "resident-weight projection: %d channel tiles do not fit %d SMs",
                    a.job[0].n_tiles, f.sm_count);
    const int grid = a.tiles < cap ? a.tiles : cap;
    const cudaError_t err_launch = launch_kernel(proj_tc_kernel<T, BN, EPI, RES, STG>, dim3(unsigned(grid)),
                                                 dim3(Lay::kThreads),
                                                 Lay::kSmemBytes, stream, pdl, map_a0, map_b0, map_out0, map_a1,
                                                 map_b1, map_out1, a);
    if (err_launch != cudaSuccess)
        return fail(err, err_len, TD_ERR_CUDA, "proj_tc_kernel launch: %s", cudaGetErrorString(err_launch));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "proj_tc_kernel");
}

#ifndef TD_PROJ_TILE
#define TD_PROJ_TILE 0  // 0: pick the tile width from the shape; 64 / 128 / 256 force one (for tuning builds)
#endif

template <typename T>
constexpr bool kTcType = std::is_same<T, __half>::value || std::is_same<T, __nv_bfloat16>::value ||
                         std::is_same<T, float>::value;

// tcgen05 projection: 16-byte aligned rows for TMA, K at least one 128-byte block, 8-column groups per head, and
// every count of 128 x 64 tiles and K blocks below 2^31 (the kernel indexes them in 32 bits)
template <typename T>
bool proj_tc_eligible(const T* memory, const T* weight, const T* value, int64_t B, int64_t N, int64_t C, int64_t H,
                      int64_t HD) {
    if constexpr (!kTcType<T>) {
        return false;
    } else {
        constexpr int kBK = GemmKind<T>::kBK;
        const int64_t D = HD / H;
        return g_policy.load(std::memory_order_relaxed) == TD_POLICY_BEST && C >= kBK &&
               (C * int64_t(sizeof(T))) % 16 == 0 && HD % 16 == 0 && D % 8 == 0 && N < (int64_t(1) << 31) &&
               B < (int64_t(1) << 31) / H &&
               B * ((N + kTcBM - 1) / kTcBM) * ((HD + 63) / 64) * ((C + kBK - 1) / kBK) < (int64_t(1) << 31) &&
               aligned16(memory) && aligned16(weight) && aligned16(value);
    }
}

// Tile plan of the tcgen05 projection. Tile width: the busiest CTA runs ceil(tiles / SMs) tiles, each costing about
// the load of its 128 memory rows (like 128 more output columns) plus the BN weight rows it loads with them; the
// width that makes that smallest, the widest of equals (float32 tiles are at most 128 wide: their slots hold hi and
// lo halves). 256-wide tiles get 16 epilogue warps (four per 32-row quarter of the accumulator): the conversion of a
// 128 x 256 tile is latency-bound, and with 8 warps it paced the tiles (B200, graphs of 50 calls: c3 39.6 -> 35.4 us
// a call, c4 110.7 -> 103.1, B=2 12.8 -> 12.4). Without a staging tile (every job stores directly) the slot ring
// takes its space. Resident weights (16-bit types, one job, C within kResKBlocks K blocks, direct stores, 256 wide):
// when CTAs run at least three tiles, loading the weight slice once beats reloading it with every tile (c3 35.4 ->
// 35.0 us, c4 103.1 -> 100.1). (B2, N2, HD2): a second job in the same launch (B2 = 0: none). direct: every job can
// take direct stores.
struct TilePlan {
    int bn;
    bool res;
    int epi;
    bool stg;
};

#ifndef TD_PROJ_PLAN_BN
#define TD_PROJ_PLAN_BN 0  // tuning builds: force single-job 16-bit plans to {BN, RES} where the job can take them
#define TD_PROJ_PLAN_RES 0
#endif

template <typename T>
TilePlan proj_tile_plan(int64_t B, int64_t N, int64_t C, int64_t HD, int sm_count, bool direct, int64_t B2 = 0,
                        int64_t N2 = 0, int64_t HD2 = 0) {
    constexpr bool f32 = std::is_same<T, float>::value;
    const bool res_fits = !f32 && B2 == 0 && direct && (C + GemmKind<T>::kBK - 1) / GemmKind<T>::kBK <= kResKBlocks;
    auto finish = [&](int bn, bool res) {
        return TilePlan{bn, res, bn == 256 ? 16 : (bn == 128 && !f32 ? 8 : 4), !direct || f32};
    };
    if (TD_PROJ_TILE != 0) return finish(TD_PROJ_TILE, false);
    if (TD_PROJ_PLAN_BN != 0 && B2 == 0 && !f32 && (res_fits || !TD_PROJ_PLAN_RES))
        return finish(TD_PROJ_PLAN_BN, TD_PROJ_PLAN_RES != 0);
    const int64_t m_tiles = B * ((N + kTcBM - 1) / kTcBM);
    const int64_t m_tiles2 = B2 * ((N2 + kTcBM - 1) / kTcBM);
    int bn = 64;
    long long best = -1;
    for (int w : {256, 128, 64}) {
        if (f32 && w > 128) continue;
        const long long tiles = m_tiles * ((HD + w - 1) / w) + m_tiles2 * ((HD2 + w - 1) / w);
        const long long cost = (tiles + sm_count - 1) / sm_count * (w + 128);
        if (best < 0 || cost < best) { best = cost; bn = w; }
    }
    // (the grid of a resident-weight launch is a multiple of the channel-tile count, so that count must fit the SMs)
    const bool res = res_fits && bn == 256 && (HD + 255) / 256 <= sm_count &&
                     m_tiles * ((HD + 255) / 256) >= 3LL * sm_count;
    return finish(bn, res);
}

// Calls f(std::integral_constant<int, BN>, std::integral_constant<int, EPI>, std::integral_constant<bool, RES>,
// std::integral_constant<bool, STG>) for the instantiated kernel of the plan.
template <typename T, typename F>
int with_tile(TilePlan plan, F&& f) {
    using no = std::integral_constant<bool, false>;
    using yes = std::integral_constant<bool, true>;
    using n64 = std::integral_constant<int, 64>;
    using n128 = std::integral_constant<int, 128>;
    using n256 = std::integral_constant<int, 256>;
    using e4 = std::integral_constant<int, 4>;
    using e8 = std::integral_constant<int, 8>;
    using e16 = std::integral_constant<int, 16>;
    if constexpr (std::is_same<T, float>::value) {
        if (plan.bn >= 128) return f(n128{}, e4{}, no{}, yes{});
        return f(n64{}, e4{}, no{}, yes{});
    } else {
        if (plan.bn == 256) {
            if (plan.res) return f(n256{}, e16{}, yes{}, no{});
            return plan.stg ? f(n256{}, e16{}, no{}, yes{}) : f(n256{}, e16{}, no{}, no{});
        }
        if (plan.bn == 128) return plan.stg ? f(n128{}, e8{}, no{}, yes{}) : f(n128{}, e8{}, no{}, no{});
        return f(n64{}, e4{}, no{}, yes{});
    }
}

template <typename T>
int launch_proj(const T* memory, const T* weight, const T* bias, T* value, int64_t B, int64_t N, int64_t C,
                int64_t H, int64_t HD, int head_major, cudaStream_t stream, char* err, size_t err_len,
                bool pdl = false) {
    if constexpr (kTcType<T>) {
        if (proj_tc_eligible<T>(memory, weight, value, B, N, C, H, HD)) {
            DeviceFacts f;
            if (int rc = device_facts(&f, err, err_len)) return rc;
            const ProjShape job{memory, weight, bias, value, B, N, C, H, HD, head_major};
            const bool direct = proj_direct32(value, HD, HD / H, head_major, int64_t(sizeof(T)));
            return with_tile<T>(proj_tile_plan<T>(B, N, C, HD, f.sm_count, direct),
                                [&](auto bn, auto epi, auto res, auto stg) {
                                    return launch_proj_tc<T, decltype(bn)::value, decltype(epi)::value,
                                                          decltype(res)::value, decltype(stg)::value>(
                                        job, nullptr, stream, pdl, err, err_len);
                                });
        }
    }
    ProjArgs<T> a;
    a.memory = memory; a.weight = weight; a.bias = bias; a.value = value;
    a.M = B * N; a.n_tok = N; a.C = int(C); a.HD = int(HD); a.H = int(H); a.D = int(HD / H);
    a.head_major = head_major;
    const dim3 grid(unsigned((a.M + kGemmBM - 1) / kGemmBM), unsigned((HD + kGemmBN - 1) / kGemmBN));
    const cudaError_t e = launch_kernel(proj_simt_kernel<T>, grid, dim3(kGemmThreads), 0, stream, pdl, a);
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "proj_simt_kernel launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "proj_simt_kernel");
}

// Two projections with the same K in one tcgen05 launch when both fit it (*paired = true); otherwise nothing is
// launched (*paired = false) and the caller launches them one by one.
template <typename T>
int launch_proj_pair(const ProjShape& j0, const ProjShape& j1, cudaStream_t stream, bool pdl, bool* paired,
                     char* err, size_t err_len) {
    *paired = false;
    if constexpr (kTcType<T>) {
        const auto* m0 = static_cast<const T*>(j0.memory);
        const auto* m1 = static_cast<const T*>(j1.memory);
        if (j0.C != j1.C || j0.B * j0.N == 0 || j1.B * j1.N == 0 ||
            !proj_tc_eligible<T>(m0, static_cast<const T*>(j0.weight), static_cast<const T*>(j0.value), j0.B, j0.N,
                                 j0.C, j0.H, j0.HD) ||
            !proj_tc_eligible<T>(m1, static_cast<const T*>(j1.weight), static_cast<const T*>(j1.value), j1.B, j1.N,
                                 j1.C, j1.H, j1.HD))
            return TD_OK;
        const int64_t t64 = j0.B * ((j0.N + kTcBM - 1) / kTcBM) * ((j0.HD + 63) / 64) +
                            j1.B * ((j1.N + kTcBM - 1) / kTcBM) * ((j1.HD + 63) / 64);
        if (t64 * ((j0.C + GemmKind<T>::kBK - 1) / GemmKind<T>::kBK) >= (int64_t(1) << 31)) return TD_OK;
        DeviceFacts f;
        if (int rc = device_facts(&f, err, err_len)) return rc;
        *paired = true;
        const bool direct =
            proj_direct32(j0.value, j0.HD, j0.HD / j0.H, j0.head_major, int64_t(sizeof(T))) &&
            proj_direct32(j1.value, j1.HD, j1.HD / j1.H, j1.head_major, int64_t(sizeof(T)));
        return with_tile<T>(proj_tile_plan<T>(j0.B, j0.N, j0.C, j0.HD, f.sm_count, direct, j1.B, j1.N, j1.HD),
                            [&](auto bn, auto epi, auto res, auto stg) {
                                // a paired launch never takes resident weights (the plan gives res = false)
                                return launch_proj_tc<T, decltype(bn)::value, decltype(epi)::value, false,
                                                      decltype(stg)::value || decltype(res)::value>(
                                    j0, &j1, stream, pdl, err, err_len);
                            });
    } else {
        (void)j0; (void)j1; (void)stream; (void)pdl; (void)err; (void)err_len;
        return TD_OK;
    }
}

// ---- the GEMMs of a linear layer's backward (td_linear_grad_input / td_linear_grad_weight) ----------------------

// Whether the tcgen05 gradient kernels take these operands: 16-bit types, every row 16-byte aligned (the TMA rule),
// sizes in int range.
template <typename T>
bool grad_tc_eligible(std::initializer_list<const void*> ptrs, int64_t M, int64_t Nout, int64_t K) {
    if constexpr (!std::is_same<T, __half>::value && !std::is_same<T, __nv_bfloat16>::value) {
        return false;
    } else {
        if (g_policy.load(std::memory_order_relaxed) != TD_POLICY_BEST) return false;
        if (Nout % 8 != 0 || K % 8 != 0 || M >= (int64_t(1) << 31) || Nout >= (int64_t(1) << 31) ||
            K >= (int64_t(1) << 31))
            return false;
        for (const void* p : ptrs)
            if (!aligned16(p)) return false;
        return true;
    }
}

// Test of the bounded waits: a positive value makes the next tensor-core gradient launch starve its own pipeline
// (its producers issue nothing) and give up every wait after that many cycles (td_test_starve_next_grad_gemm).
std::atomic<long long> g_starve_next{0};

template <typename T, bool A_MN, int BN, bool SPLIT>
int launch_grad_tc(const void* a_ptr, uint64_t a_cols, uint64_t a_rows, uint32_t a_box_rows, const void* b_ptr,
                   uint64_t b_cols, uint64_t b_rows, GradGemmArgs<T> args, cudaStream_t stream, char* err,
                   size_t err_len) {
    using Lay = GradTcLayout<BN>;
    const long long starve = g_starve_next.exchange(0);
    args.starve = starve > 0 ? 1 : 0;
    args.spin_limit = starve > 0 ? starve : kSpinLimitCycles;
    static std::atomic<uint64_t> smem_done{0};
    CUtensorMap map_a, map_b;
    if (int rc = tensor_map_2d(&map_a, a_ptr, a_cols, a_rows, a_box_rows, err, err_len, 2)) return rc;
    if (int rc = tensor_map_2d(&map_b, b_ptr, b_cols, b_rows, 64, err, err_len, 2)) return rc;
    if (int rc = allow_smem(grad_gemm_tc_kernel<T, A_MN, BN, SPLIT>, Lay::kSmemBytes, smem_done, err, err_len))
        return rc;
    const unsigned grid = unsigned(args.m_tiles * args.n_tiles * args.splits);
    const cudaError_t e = launch_kernel(grad_gemm_tc_kernel<T, A_MN, BN, SPLIT>, dim3(grid), dim3(Lay::kThreads),
                                        Lay::kSmemBytes, stream, true, map_a, map_b, args);
    if (e != cudaSuccess)
        return fail(err, err_len, TD_ERR_CUDA, "grad_gemm_tc_kernel launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "grad_gemm_tc_kernel");
}

template <typename T, bool ATOMIC>
int launch_grad_simt(const GradSimtArgs<T>& p, int splits, cudaStream_t stream, char* err, size_t err_len) {
    const dim3 grid(unsigned((p.rows + 63) / 64), unsigned((p.cols + 63) / 64), unsigned(splits));
    const cudaError_t e = launch_kernel(grad_gemm_simt_kernel<T, ATOMIC>, grid, dim3(256), 0, stream, true, p);
    if (e != cudaSuccess)
        return fail(err, err_len, TD_ERR_CUDA, "grad_gemm_simt_kernel launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "grad_gemm_simt_kernel");
}

// Splits of a K range of k_blocks blocks over CTAs: enough to give the SMs about one CTA each, none shorter than
// min_blocks blocks, none empty. Returns the splits and sets *per (blocks per split).
inline int grad_splits(int64_t tiles, int64_t k_blocks, int sm_count, int64_t min_blocks, int64_t* per) {
    int64_t splits = std::max<int64_t>(1, std::min<int64_t>(sm_count / std::max<int64_t>(tiles, 1),
                                                           k_blocks / std::max<int64_t>(min_blocks, 1)));
    *per = (k_blocks + splits - 1) / splits;
    splits = (k_blocks + *per - 1) / *per;
    return int(std::max<int64_t>(splits, 1));
}

// The weight gradient's K splits are capped so that tiles x splits <= kGradMaxCtas (at least the SM count of any
// part this runs on): its float32 partials then take at most kGradMaxCtas x 64 KB of workspace.
constexpr int64_t kGradMaxCtas = 256;
inline int64_t grad_split_cap(int64_t tiles) {
    return std::max<int64_t>(1, kGradMaxCtas / std::max<int64_t>(tiles, 1));
}

// Workspace of td_linear_grad_weight, laid out as: float32 partial sums [splits, Nout, K] | float32 bias sums [Nout] |
// bias arrival counters; every region 256-byte aligned (16-bit types only; float32 / float64 accumulate in the
// outputs themselves).
struct GradWeightWs {
    size_t acc = 0, bias = 0, bias_arrivals = 0, total = 0;
};
inline GradWeightWs grad_weight_ws(int dtype, int64_t Nout, int64_t K) {
    GradWeightWs w;
    if (dtype != TD_F16 && dtype != TD_BF16) return w;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    const int64_t tiles = ((Nout + 127) / 128) * ((K + 127) / 128);
    w.acc = 0;
    w.bias = up(size_t(grad_split_cap(tiles)) * size_t(Nout) * size_t(K) * 4);
    w.bias_arrivals = w.bias + up(size_t(Nout) * 4);
    w.total = w.bias_arrivals + up(size_t((Nout + 255) / 256) * 4) + 256;  // + 256: alignment of the base
    return w;
}

// Column sums of x [rows, cols] into out [cols] (the input type), through float32 (float64) `sums` and, for 16-bit
// types, a conversion by the last CTA of each column block (`arrivals`, one counter per column block). sums and
// arrivals are zeroed here.
template <typename T>
int launch_column_sum(const T* x, T* out, typename Elem<T>::acc* sums, unsigned* arrivals, int64_t rows, int64_t cols,
                      cudaStream_t stream, char* err, size_t err_len) {
    using A = typename Elem<T>::acc;
    DeviceFacts f;
    if (int rc = device_facts(&f, err, err_len)) return rc;
    cudaError_t e = cudaMemsetAsync(sums, 0, size_t(cols) * sizeof(A), stream);
    const int64_t col_blocks = (cols + 255) / 256;
    if (e == cudaSuccess && arrivals != nullptr) e = cudaMemsetAsync(arrivals, 0, size_t(col_blocks) * 4, stream);
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    const int64_t row_blocks = std::max<int64_t>(1, std::min<int64_t>((rows + 63) / 64, 2 * f.sm_count / col_blocks));
    const long long per = (long long)((rows + row_blocks - 1) / row_blocks);
    const dim3 grid(unsigned(col_blocks), unsigned((rows + per - 1) / per));
    e = launch_kernel(column_sum_kernel<T>, grid, dim3(256), 0, stream, true, x, sums,
                      std::is_same<A, T>::value ? static_cast<T*>(nullptr) : out, arrivals, (long long)rows,
                      int(cols), per);
    if (e != cudaSuccess)
        return fail(err, err_len, TD_ERR_CUDA, "column_sum_kernel launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "column_sum_kernel");
}

template <typename F>
int dispatch(int dtype, F&& f) {
    switch (dtype) {
        case TD_F32: return f(float{});
        case TD_F16: return f(__half{});
        case TD_BF16: return f(__nv_bfloat16{});
        case TD_F64: return f(double{});
        default: return -1;
    }
}

// The standalone sampling producer (td_producer.cuh), with programmatic dependent launch behind the query
// projection.
template <typename T>
int launch_producer(const T* proj, const T* ref, int ref_dim, const int64_t* shapes, T* loc, T* attn, int64_t B,
                    int64_t Q, int64_t H, int64_t L, int64_t P, cudaStream_t stream, char* err, size_t err_len) {
    ProducerArgs<T> a;
    a.in.proj = proj; a.in.ref = ref; a.in.ref_dim = ref_dim; a.shapes = shapes; a.loc = loc; a.attn = attn;
    a.rows = B * Q * H; a.H = int(H); a.L = int(L); a.P = int(P);
    const unsigned grid = unsigned((a.rows + kProducerWarps - 1) / kProducerWarps);
    const cudaError_t e = launch_kernel(sampling_producer_kernel<T>, dim3(grid), dim3(kProducerWarps * 32), 0, stream,
                                        true, a);
    if (e != cudaSuccess)
        return fail(err, err_len, TD_ERR_CUDA, "sampling_producer_kernel launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "sampling_producer_kernel");
}

template <typename T>
int launch_producer_backward(const ProducerBwdArgs<T>& a, cudaStream_t stream, char* err, size_t err_len) {
    const unsigned grid = unsigned(a.bq);  // one CTA per (batch, query)
    const cudaError_t e = launch_kernel(sampling_producer_backward_kernel<T>, dim3(grid), dim3(kProducerWarps * 32),
                                        0, stream, true, a);
    if (e != cudaSuccess)
        return fail(err, err_len, TD_ERR_CUDA, "sampling_producer_backward_kernel launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "sampling_producer_backward_kernel");
}

// Backward of the sampling half (td_backward.cuh): zeroes grad_value, then one warp per (b, q, h) row.
template <typename T>
int launch_sample_backward(const T* value, long long s_img, long long s_tok, long long s_head, const int64_t* shapes,
                           const int64_t* starts, const T* loc, const T* attn, const uint8_t* mask, const T* grad_out,
                           typename Coord<T>::type* grad_value, T* grad_loc, T* grad_attn, int64_t B, int64_t Q,
                           int64_t N, int64_t H, int64_t D, int64_t L, int64_t P, cudaStream_t stream, char* err,
                           size_t err_len) {
    using CT = typename Coord<T>::type;
    cudaError_t e = cudaMemsetAsync(grad_value, 0, size_t(B) * size_t(N) * size_t(H * D) * sizeof(CT), stream);
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    if (B * Q * L * P == 0) return TD_OK;
    BackArgs<T> a;
    a.value = value; a.s_img = s_img; a.s_tok = s_tok; a.s_head = s_head; a.loc = loc; a.attn = attn;
    a.grad_out = grad_out; a.grad_value = grad_value; a.grad_loc = grad_loc; a.grad_attn = grad_attn;
    a.shapes = shapes; a.starts = starts; a.mask = mask; a.rows = B * Q * H; a.n_tok = N;
    a.Q = int(Q); a.H = int(H); a.D = int(D); a.L = int(L); a.P = int(P);
    const long long row_bytes = D * (long long)sizeof(T);
    a.G = int(row_bytes / 16);
    const bool vec = row_bytes % 16 == 0 && row_bytes <= 512 && (a.G & (a.G - 1)) == 0 && aligned16(value) &&
                     aligned16(grad_out) && aligned16(grad_value) && (D * (long long)sizeof(CT)) % 16 == 0 &&
                     (s_img * (long long)sizeof(T)) % 16 == 0 && (s_tok * (long long)sizeof(T)) % 16 == 0 &&
                     (s_head * (long long)sizeof(T)) % 16 == 0;
    if (vec) {
        // 32 / G points per warp
        const long long points = a.rows * L * P, per_cta = (long long)kBackWarps * (32 / a.G);
        const long long grid = (points + per_cta - 1) / per_cta;
        if (grid > INT32_MAX) return fail(err, err_len, TD_ERR_ARG, "too many sampling points for one launch");
        e = launch_kernel(sample_backward_vec_kernel<T>, dim3(unsigned(grid)), dim3(kBackWarps * 32), 0, stream,
                          false, a);
    } else {
        const size_t smem = backward_smem<T>(int(L), int(P));  // up to 56 KB (float64, L * P = 64)
        static std::atomic<uint64_t> smem_generic{0};
        if (int rc = allow_smem(sample_backward_generic_kernel<T>, smem, smem_generic, err, err_len)) return rc;
        e = launch_kernel(sample_backward_generic_kernel<T>, dim3(unsigned((a.rows + kBackWarps - 1) / kBackWarps)),
                          dim3(kBackWarps * 32), smem, stream, false, a);
    }
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "backward launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, vec ? "sample_backward_vec_kernel" : "sample_backward_generic_kernel");
}

// Byte offsets of the decoder layer's intermediates in its workspace (each region 256-byte aligned, from the first
// 256-byte boundary of the workspace): the query projection, the projected value (project order), locations and
// weights (fused order), and the attention result when an output projection follows.
struct LayerWorkspace {
    size_t proj = 0, value = 0, loc = 0, attn = 0, mid = 0, bytes = 0;
};

LayerWorkspace layer_workspace(size_t e, int order, int64_t B, int64_t Q, int64_t N, int64_t H, int64_t HD,
                               int64_t L, int64_t P, bool output_proj) {
    LayerWorkspace w;
    size_t at = 0;
    auto take = [&](size_t n) {
        const size_t off = at;
        at += (n * e + 255) & ~size_t(255);
        return off;
    };
    const size_t rows = size_t(B) * size_t(Q);
    w.proj = take(rows * size_t(3 * H * L * P));
    if (order == TD_ORDER_PROJECT) {
        w.value = take(size_t(B) * size_t(N) * size_t(HD));
    } else {
        w.loc = take(rows * size_t(H * L * P * 2));
        w.attn = take(rows * size_t(H * L * P));
    }
    if (output_proj) w.mid = take(rows * size_t(HD));
    w.bytes = at + 256;
    return w;
}

}  // namespace
}  // namespace td

using namespace td;

extern "C" {

int td_fused_forward(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                     const int64_t* spatial_shapes, const int64_t* level_start_index,
                     const void* sampling_locations, const void* attention_weights, void* out,
                     int64_t B, int64_t Q, int64_t N, int64_t C, int64_t H, int64_t HD, int64_t L, int64_t P,
                     void* stream, char* err, size_t err_len) {
    return td_fused_forward_masked(dtype, memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                   sampling_locations, attention_weights, nullptr, out, B, Q, N, C, H, HD, L, P,
                                   stream, err, err_len);
}

int td_fused_forward_masked(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                            const int64_t* spatial_shapes, const int64_t* level_start_index,
                            const void* sampling_locations, const void* attention_weights,
                            const uint8_t* value_padding_mask, void* out, int64_t B, int64_t Q, int64_t N, int64_t C,
                            int64_t H, int64_t HD, int64_t L, int64_t P, void* stream, char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (int rc = check_geometry(B, Q, N, H, L, P, err, err_len)) return rc;
    if (C <= 0 || HD <= 0) return fail(err, err_len, TD_ERR_ARG, "channels and value_weight rows must be positive");
    if (HD % H != 0) return fail(err, err_len, TD_ERR_ARG, "value_weight rows must be a multiple of the head count");
    if (C > TD_MAX_CHANNELS) return fail(err, err_len, TD_ERR_ARG, "channels must be <= %d", TD_MAX_CHANNELS);
    if (B * Q == 0) return TD_OK;
    if (!memory || !value_weight || !sampling_locations || !attention_weights || !out ||
        (L * P > 0 && (!spatial_shapes || !level_start_index)))
        return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t D = HD / H;
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        return launch_fused<T>(static_cast<const T*>(memory), static_cast<const T*>(value_weight),
                               static_cast<const T*>(value_bias), spatial_shapes, level_start_index,
                               static_cast<const T*>(sampling_locations), static_cast<const T*>(attention_weights),
                               static_cast<T*>(out), B, Q, N, C, H, D, L, P, s, err, err_len, value_padding_mask);
    });
}

int td_sample_forward(int dtype, const void* value, int64_t heads, const int64_t* spatial_shapes,
                      const int64_t* level_start_index, const void* sampling_locations,
                      const void* attention_weights, void* out,
                      int64_t B, int64_t Q, int64_t N, int64_t HD, int64_t H, int64_t L, int64_t P,
                      void* stream, char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (int rc = check_geometry(B, Q, N, H, L, P, err, err_len)) return rc;
    if (heads != H || HD <= 0 || HD % H != 0)
        return fail(err, err_len, TD_ERR_ARG, "value must be [B, N, H * D] with H = sampling_locations.size(2)");
    if (B * Q == 0) return TD_OK;
    if (!value || !sampling_locations || !attention_weights || !out ||
        (L * P > 0 && (!spatial_shapes || !level_start_index)))
        return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t D = HD / H;
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        return launch_sampler<T>(static_cast<const T*>(value), N * HD, HD, D, spatial_shapes, level_start_index,
                                 static_cast<const T*>(sampling_locations), static_cast<const T*>(attention_weights),
                                 static_cast<T*>(out), B, Q, N, H, D, L, P, s, err, err_len);
    });
}

int td_value_proj(int dtype, const void* memory, const void* value_weight, const void* value_bias, void* value,
                  int64_t B, int64_t N, int64_t C, int64_t H, int64_t HD, int head_major,
                  void* stream, char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (B < 0 || N < 0 || C <= 0 || H <= 0 || HD <= 0 || HD % H != 0)
        return fail(err, err_len, TD_ERR_ARG, "value_proj needs B, N >= 0, C, H, HD > 0 and HD %% H == 0");
    if (N > INT32_MAX || C > INT32_MAX || HD > INT32_MAX) return fail(err, err_len, TD_ERR_ARG, "size too large");
    if (B * N == 0) return TD_OK;
    if (!memory || !value_weight || !value) return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        // with programmatic dependent launch, as td_linear: every role of the projection kernels waits for the
        // previous kernel before its first global access, so its set-up overlaps that kernel's tail
        return launch_proj<T>(static_cast<const T*>(memory), static_cast<const T*>(value_weight),
                              static_cast<const T*>(value_bias), static_cast<T*>(value), B, N, C, H, HD,
                              head_major ? 1 : 0, s, err, err_len, true);
    });
}

int td_linear(int dtype, const void* x, const void* weight, const void* bias, void* y, int64_t M, int64_t K,
              int64_t Nout, void* stream, char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (M < 0 || K <= 0 || Nout <= 0) return fail(err, err_len, TD_ERR_ARG, "linear needs M >= 0, K > 0, Nout > 0");
    if (M > INT32_MAX || K > INT32_MAX || Nout > INT32_MAX) return fail(err, err_len, TD_ERR_ARG, "size too large");
    if (M == 0) return TD_OK;
    if (!x || !weight || !y) return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        // one "image" of M tokens and one "head" of Nout channels: the projection kernel in its [B, N, HD] layout,
        // launched with programmatic dependent launch so it starts under the kernel before it
        return launch_proj<T>(static_cast<const T*>(x), static_cast<const T*>(weight), static_cast<const T*>(bias),
                              static_cast<T*>(y), 1, M, K, 1, Nout, 0, s, err, err_len, true);
    });
}

int td_sampling_producer(int dtype, const void* proj, const void* reference_points, int ref_dim,
                         const int64_t* spatial_shapes, void* sampling_locations, void* attention_weights, int64_t B,
                         int64_t Q, int64_t H, int64_t L, int64_t P, void* stream, char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (B < 0 || Q < 0 || H <= 0 || L <= 0 || P <= 0)
        return fail(err, err_len, TD_ERR_ARG, "producer needs B, Q >= 0 and H, L, P > 0");
    if (L * P > TD_MAX_LEVEL_POINTS)
        return fail(err, err_len, TD_ERR_ARG, "levels x points must be <= %d", TD_MAX_LEVEL_POINTS);
    if (ref_dim != 2 && ref_dim != 4)
        return fail(err, err_len, TD_ERR_ARG, "reference points must have 2 (x, y) or 4 (cx, cy, w, h) coordinates");
    if (B * Q * H > INT32_MAX) return fail(err, err_len, TD_ERR_ARG, "too many (batch, query, head) rows");
    if (B * Q == 0) return TD_OK;
    if (!proj || !reference_points || !spatial_shapes || !sampling_locations || !attention_weights)
        return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        return launch_producer<T>(static_cast<const T*>(proj), static_cast<const T*>(reference_points), ref_dim,
                                  spatial_shapes, static_cast<T*>(sampling_locations),
                                  static_cast<T*>(attention_weights), B, Q, H, L, P, s, err, err_len);
    });
}

int td_sampling_producer_backward(int dtype, const void* proj, const void* reference_points, int ref_dim,
                                  const int64_t* spatial_shapes, const void* grad_locations,
                                  const void* grad_weights, void* grad_proj, void* grad_reference_points, int64_t B,
                                  int64_t Q, int64_t H, int64_t L, int64_t P, void* stream, char* err,
                                  size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (B < 0 || Q < 0 || H <= 0 || L <= 0 || P <= 0)
        return fail(err, err_len, TD_ERR_ARG, "producer needs B, Q >= 0 and H, L, P > 0");
    if (L * P > TD_MAX_LEVEL_POINTS)
        return fail(err, err_len, TD_ERR_ARG, "levels x points must be <= %d", TD_MAX_LEVEL_POINTS);
    if (ref_dim != 2 && ref_dim != 4)
        return fail(err, err_len, TD_ERR_ARG, "reference points must have 2 (x, y) or 4 (cx, cy, w, h) coordinates");
    if (B * Q * H > INT32_MAX) return fail(err, err_len, TD_ERR_ARG, "too many (batch, query, head) rows");
    if (B * Q == 0) return TD_OK;
    if (!proj || !reference_points || !spatial_shapes || !grad_proj)
        return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        ProducerBwdArgs<T> a;
        a.proj = static_cast<const T*>(proj); a.ref = static_cast<const T*>(reference_points);
        a.shapes = spatial_shapes; a.g_loc = static_cast<const T*>(grad_locations);
        a.g_attn = static_cast<const T*>(grad_weights); a.g_proj = static_cast<T*>(grad_proj);
        a.g_ref = static_cast<T*>(grad_reference_points); a.bq = B * Q; a.ref_dim = ref_dim; a.H = int(H);
        a.L = int(L); a.P = int(P);
        return launch_producer_backward<T>(a, s, err, err_len);
    });
}

size_t td_linear_grad_workspace_bytes(int dtype, int64_t Nout, int64_t K) {
    if (dtype_size(dtype) == 0 || Nout <= 0 || K <= 0) return 0;
    return grad_weight_ws(dtype, Nout, K).total;
}

int td_linear_grad_input(int dtype, const void* grad_out, const void* weight, void* grad_input, int64_t M,
                         int64_t Nout, int64_t K, void* stream, char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (M < 0 || Nout <= 0 || K <= 0) return fail(err, err_len, TD_ERR_ARG, "linear grad needs M >= 0, Nout, K > 0");
    if (M > INT32_MAX || Nout > INT32_MAX || K > INT32_MAX) return fail(err, err_len, TD_ERR_ARG, "size too large");
    if (M == 0) return TD_OK;
    if (!grad_out || !weight || !grad_input) return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        if (grad_tc_eligible<T>({grad_out, weight, grad_input}, M, Nout, K)) {
            if constexpr (std::is_same<T, __half>::value || std::is_same<T, __nv_bfloat16>::value) {
                DeviceFacts f;
                if (int rc = device_facts(&f, err, err_len)) return rc;
                GradGemmArgs<T> g{};
                g.out = static_cast<T*>(grad_input);
                g.rows = int(M);
                g.cols = int(K);
                g.m_tiles = int((M + 127) / 128);
                g.splits = 1;
                g.k_blocks = int((Nout + 63) / 64);
                g.kb_per_split = g.k_blocks;
                // A = grad_out [M, Nout] (K-major, 128-row boxes), B = weight [Nout, K] (MN-major)
                if (int64_t(g.m_tiles) * ((K + 127) / 128) <= f.sm_count || K <= 128) {
                    g.n_tiles = int((K + 127) / 128);
                    return launch_grad_tc<T, false, 128, false>(grad_out, uint64_t(Nout), uint64_t(M), 128, weight,
                                                                uint64_t(K), uint64_t(Nout), g, s, err, err_len);
                }
                g.n_tiles = int((K + 255) / 256);
                return launch_grad_tc<T, false, 256, false>(grad_out, uint64_t(Nout), uint64_t(M), 128, weight,
                                                            uint64_t(K), uint64_t(Nout), g, s, err, err_len);
            }
        }
        GradSimtArgs<T> p{};
        p.a = static_cast<const T*>(grad_out);
        p.b = static_cast<const T*>(weight);
        p.out = static_cast<T*>(grad_input);
        p.sam = Nout; p.sak = 1; p.sbk = K; p.sbn = 1;
        p.rows = int(M); p.cols = int(K); p.K = Nout; p.k_per_split = (Nout + 15) / 16 * 16;
        return launch_grad_simt<T, false>(p, 1, s, err, err_len);
    });
}

int td_linear_grad_weight(int dtype, const void* grad_out, const void* input, void* grad_weight, void* grad_bias,
                          int64_t M, int64_t Nout, int64_t K, void* workspace, size_t workspace_bytes, void* stream,
                          char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (M < 0 || Nout <= 0 || K <= 0) return fail(err, err_len, TD_ERR_ARG, "linear grad needs M >= 0, Nout, K > 0");
    if (M > INT32_MAX || Nout > INT32_MAX || K > INT32_MAX || Nout * K > INT32_MAX)
        return fail(err, err_len, TD_ERR_ARG, "size too large");
    if (!grad_weight || (M > 0 && (!grad_out || !input))) return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    const GradWeightWs w = grad_weight_ws(dtype, Nout, K);
    if (w.total > 0 && (workspace == nullptr || workspace_bytes < w.total))
        return fail(err, err_len, TD_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", w.total,
                    workspace_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned char* ws =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        using A = typename Elem<T>::acc;
        constexpr bool k16 = std::is_same<T, __half>::value || std::is_same<T, __nv_bfloat16>::value;
        if (M == 0) {  // no rows: zero gradients
            cudaError_t e = cudaMemsetAsync(grad_weight, 0, size_t(Nout) * size_t(K) * sizeof(T), s);
            if (e == cudaSuccess && grad_bias) e = cudaMemsetAsync(grad_bias, 0, size_t(Nout) * sizeof(T), s);
            if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
            return int(TD_OK);
        }
        if (grad_bias) {
            A* sums = k16 ? reinterpret_cast<A*>(ws + w.bias) : static_cast<A*>(grad_bias);
            unsigned* arr = k16 ? reinterpret_cast<unsigned*>(ws + w.bias_arrivals) : nullptr;
            if (int rc = launch_column_sum<T>(static_cast<const T*>(grad_out), static_cast<T*>(grad_bias), sums, arr,
                                              M, Nout, s, err, err_len))
                return rc;
        }
        DeviceFacts f;
        if (int rc = device_facts(&f, err, err_len)) return rc;
        if constexpr (k16) {
            if (grad_tc_eligible<T>({grad_out, input, grad_weight}, M, Nout, K)) {
                GradGemmArgs<T> g{};
                g.out = static_cast<T*>(grad_weight);
                g.acc = reinterpret_cast<float*>(ws + w.acc);
                g.rows = int(Nout);
                g.cols = int(K);
                g.m_tiles = int((Nout + 127) / 128);
                g.n_tiles = int((K + 127) / 128);
                const int64_t tiles = int64_t(g.m_tiles) * g.n_tiles;
                int64_t per = 0;
                g.k_blocks = int((M + 63) / 64);
                g.splits = grad_splits(tiles, g.k_blocks, int(std::min<int64_t>(f.sm_count, kGradMaxCtas)), 4, &per);
                g.kb_per_split = int(per);
                // A = grad_out [M, Nout] and B = input [M, K], both MN-major (the sum runs over their M rows); every
                // CTA writes its whole partial tile, so the partials need no clearing
                if (int rc = launch_grad_tc<T, true, 128, true>(grad_out, uint64_t(Nout), uint64_t(M), 64, input,
                                                                uint64_t(K), uint64_t(M), g, s, err, err_len))
                    return rc;
                const long long elems = (long long)Nout * K;
                const unsigned grid = unsigned((elems / 4 + kReduceThreads - 1) / kReduceThreads);
                const cudaError_t e = launch_kernel(grad_split_reduce_kernel<T>, dim3(grid), dim3(kReduceThreads), 0,
                                                    s, true, static_cast<const float*>(g.acc),
                                                    static_cast<T*>(grad_weight), g.splits, elems);
                if (e != cudaSuccess)
                    return fail(err, err_len, TD_ERR_CUDA, "grad_split_reduce_kernel launch: %s",
                                cudaGetErrorString(e));
                g_launches.fetch_add(1, std::memory_order_relaxed);
                return check_launch(err, err_len, "grad_split_reduce_kernel");
            }
        }
        GradSimtArgs<T> p{};
        p.a = static_cast<const T*>(grad_out);
        p.b = static_cast<const T*>(input);
        p.out = static_cast<T*>(grad_weight);
        p.sam = 1; p.sak = Nout; p.sbk = K; p.sbn = 1;
        p.rows = int(Nout); p.cols = int(K); p.K = M;
        if constexpr (k16) {
            // 16-bit shapes the tensor cores do not take: one pass over all rows per tile, no atomics
            p.k_per_split = (M + 15) / 16 * 16;
            return launch_grad_simt<T, false>(p, 1, s, err, err_len);
        } else {
            const int64_t tiles = ((Nout + 63) / 64) * ((K + 63) / 64);
            int64_t per = 0;
            const int splits = grad_splits(tiles, (M + 15) / 16, 2 * f.sm_count, 16, &per);
            p.k_per_split = per * 16;
            const cudaError_t e = cudaMemsetAsync(grad_weight, 0, size_t(Nout) * size_t(K) * sizeof(T), s);
            if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
            return launch_grad_simt<T, true>(p, splits, s, err, err_len);
        }
    });
}

int td_sample_backward(int dtype, const void* value, int64_t s_img, int64_t s_tok, int64_t s_head,
                       const int64_t* spatial_shapes, const int64_t* level_start_index,
                       const void* sampling_locations, const void* attention_weights,
                       const uint8_t* value_padding_mask, const void* grad_out, void* grad_value,
                       void* grad_sampling_locations, void* grad_attention_weights, int64_t B, int64_t Q, int64_t N,
                       int64_t H, int64_t D, int64_t L, int64_t P, void* stream, char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (int rc = check_geometry(B, Q, N, H, L, P, err, err_len)) return rc;
    if (D <= 0 || s_img < 0 || s_tok < 0 || s_head < 0)
        return fail(err, err_len, TD_ERR_ARG, "head size must be positive and strides non-negative");
    if (!grad_value || (B * Q > 0 && (!value || !sampling_locations || !attention_weights || !grad_out ||
                                      !grad_sampling_locations || !grad_attention_weights ||
                                      (L * P > 0 && (!spatial_shapes || !level_start_index)))))
        return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    if (B * N == 0 && B * Q == 0) return TD_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        using CT = typename Coord<T>::type;
        return launch_sample_backward<T>(static_cast<const T*>(value), s_img, s_tok, s_head, spatial_shapes,
                                         level_start_index, static_cast<const T*>(sampling_locations),
                                         static_cast<const T*>(attention_weights), value_padding_mask,
                                         static_cast<const T*>(grad_out), static_cast<CT*>(grad_value),
                                         static_cast<T*>(grad_sampling_locations),
                                         static_cast<T*>(grad_attention_weights), B, Q, N, H, D, L, P, s, err,
                                         err_len);
    });
}

int td_grad_value_finish(int dtype, const float* grad_value, void* grad_value_dtype, float* grad_bias,
                         int64_t rows, int64_t HD, void* stream, char* err, size_t err_len) {
    if (dtype != TD_F32 && dtype != TD_F16 && dtype != TD_BF16)
        return fail(err, err_len, TD_ERR_ARG, "grad_value finish takes float32, float16 or bfloat16 (code %d)", dtype);
    if (rows < 0 || HD <= 0 || HD % 4 != 0 || HD > 4 * kFinishThreads)
        return fail(err, err_len, TD_ERR_ARG, "grad_value finish needs rows >= 0 and 0 < HD <= %d, HD %% 4 == 0",
                    4 * kFinishThreads);
    if (rows > 0 && (!grad_value || (dtype != TD_F32 && !grad_value_dtype)))
        return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    if ((rows > 0 && !aligned16(grad_value)) || (grad_bias && !aligned16(grad_bias)))
        return fail(err, err_len, TD_ERR_ARG, "grad_value and grad_bias must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (grad_bias) {
        const cudaError_t e = cudaMemsetAsync(grad_bias, 0, size_t(HD) * sizeof(float), s);
        if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    }
    if (rows == 0) return TD_OK;
    DeviceFacts f;
    if (int rc = device_facts(&f, err, err_len)) return rc;
    // about four CTAs per SM, each over a contiguous block of rows
    const long long ctas_wanted = 4LL * f.sm_count;
    const long long per_cta = std::max<long long>(1, (rows + ctas_wanted - 1) / ctas_wanted);
    const unsigned grid = unsigned((rows + per_cta - 1) / per_cta);
    auto go = [&](auto kernel, auto* out) {
        const cudaError_t e = launch_kernel(kernel, dim3(grid), dim3(kFinishThreads), 0, s, false, grad_value, out,
                                            grad_bias, (long long)rows, int(HD), per_cta);
        if (e != cudaSuccess)
            return fail(err, err_len, TD_ERR_CUDA, "grad_value_finish_kernel launch: %s", cudaGetErrorString(e));
        g_launches.fetch_add(1, std::memory_order_relaxed);
        return check_launch(err, err_len, "grad_value_finish_kernel");
    };
    if (dtype == TD_F16) return go(grad_value_finish_kernel<__half>, static_cast<__half*>(grad_value_dtype));
    if (dtype == TD_BF16)
        return go(grad_value_finish_kernel<__nv_bfloat16>, static_cast<__nv_bfloat16*>(grad_value_dtype));
    return go(grad_value_finish_kernel<float>, static_cast<float*>(nullptr));
}

int td_sample_strided(int dtype, const void* value, int64_t s_img, int64_t s_tok, int64_t s_head,
                      const int64_t* spatial_shapes, const int64_t* level_start_index,
                      const void* sampling_locations, const void* attention_weights, void* out,
                      int64_t B, int64_t Q, int64_t N, int64_t H, int64_t D, int64_t L, int64_t P,
                      void* stream, char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (int rc = check_geometry(B, Q, N, H, L, P, err, err_len)) return rc;
    if (D <= 0 || s_img < 0 || s_tok < 0 || s_head < 0)
        return fail(err, err_len, TD_ERR_ARG, "head size must be positive and strides non-negative");
    if (B * Q == 0) return TD_OK;
    if (!value || !sampling_locations || !attention_weights || !out ||
        (L * P > 0 && (!spatial_shapes || !level_start_index)))
        return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        return launch_sampler<T>(static_cast<const T*>(value), s_img, s_tok, s_head, spatial_shapes,
                                 level_start_index, static_cast<const T*>(sampling_locations),
                                 static_cast<const T*>(attention_weights), static_cast<T*>(out), B, Q, N, H, D, L,
                                 P, s, err, err_len);
    });
}

size_t td_project_workspace_bytes(int dtype, int64_t B, int64_t N, int64_t HD) {
    const size_t e = dtype_size(dtype);
    if (e == 0 || B < 0 || N < 0 || HD < 0) return 0;
    return size_t(B) * size_t(N) * size_t(HD) * e + 256;
}

int td_project_forward(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                       const int64_t* spatial_shapes, const int64_t* level_start_index,
                       const void* sampling_locations, const void* attention_weights, void* out,
                       int64_t B, int64_t Q, int64_t N, int64_t C, int64_t H, int64_t HD, int64_t L, int64_t P,
                       void* workspace, size_t workspace_bytes, void* stream, char* err, size_t err_len) {
    return td_project_forward_masked(dtype, memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                     sampling_locations, attention_weights, nullptr, out, B, Q, N, C, H, HD, L, P,
                                     workspace, workspace_bytes, stream, err, err_len);
}

int td_project_forward_masked(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                              const int64_t* spatial_shapes, const int64_t* level_start_index,
                              const void* sampling_locations, const void* attention_weights,
                              const uint8_t* value_padding_mask, void* out, int64_t B, int64_t Q, int64_t N,
                              int64_t C, int64_t H, int64_t HD, int64_t L, int64_t P, void* workspace,
                              size_t workspace_bytes, void* stream, char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (int rc = check_geometry(B, Q, N, H, L, P, err, err_len)) return rc;
    if (C <= 0 || HD <= 0) return fail(err, err_len, TD_ERR_ARG, "channels and value_weight rows must be positive");
    if (HD % H != 0) return fail(err, err_len, TD_ERR_ARG, "value_weight rows must be a multiple of the head count");
    if (B * Q == 0) return TD_OK;
    if (!memory || !value_weight || !sampling_locations || !attention_weights || !out ||
        (L * P > 0 && (!spatial_shapes || !level_start_index)))
        return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    const size_t need = td_project_workspace_bytes(dtype, B, N, HD);
    if (workspace == nullptr || workspace_bytes < need)
        return fail(err, err_len, TD_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need,
                    workspace_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t D = HD / H;
    // head-major value at the first 256-byte boundary of the workspace
    void* value = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        T* v = static_cast<T*>(value);
        if (int rc = launch_proj<T>(static_cast<const T*>(memory), static_cast<const T*>(value_weight),
                                    static_cast<const T*>(value_bias), v, B, N, C, H, HD, 1, s, err, err_len, true))
            return rc;
        return launch_sampler<T>(v, H * N * D, D, N * D, spatial_shapes, level_start_index,
                                 static_cast<const T*>(sampling_locations), static_cast<const T*>(attention_weights),
                                 static_cast<T*>(out), B, Q, N, H, D, L, P, s, err, err_len, true,
                                 value_padding_mask);
    });
}

static_assert(td::kErrPeerWait == TD_DEVERR_PEER_WAIT, "peer wait error code");
static_assert(td::kPeerCtrlWords * 4 == TD_PEER_CTRL_BYTES, "peer control block size");

int td_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle, char* err, size_t err_len) {
    if (ptr == nullptr || ipc_handle == nullptr || bytes == 0)
        return fail(err, err_len, TD_ERR_ARG, "peer buffer needs bytes > 0 and output pointers");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        if (p != nullptr) cudaFree(p);
        cudaGetLastError();
        return fail(err, err_len, TD_ERR_CUDA, "peer buffer of %zu bytes: %s", bytes, cudaGetErrorString(e));
    }
    static_assert(sizeof(h) == TD_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(ipc_handle, &h, sizeof(h));
    *ptr = p;
    return TD_OK;
}

int td_peer_buffer_open(const void* ipc_handle, void** ptr, char* err, size_t err_len) {
    if (ptr == nullptr || ipc_handle == nullptr) return fail(err, err_len, TD_ERR_ARG, "null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(err, err_len, TD_ERR_CUDA, "opening a peer's buffer: %s", cudaGetErrorString(e));
    }
    return TD_OK;
}

int td_peer_buffer_close(void* ptr, int opened, char* err, size_t err_len) {
    if (ptr == nullptr) return TD_OK;
    const cudaError_t e = opened ? cudaIpcCloseMemHandle(ptr) : cudaFree(ptr);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(err, err_len, TD_ERR_CUDA, "closing a peer buffer: %s", cudaGetErrorString(e));
    }
    return TD_OK;
}

int td_project_forward_peer(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                            const int64_t* spatial_shapes, const int64_t* level_start_index,
                            const void* sampling_locations, const void* attention_weights,
                            const uint8_t* value_padding_mask, int64_t B, int64_t Q, int64_t N, int64_t C,
                            int64_t H, int64_t HD, int64_t L, int64_t P, int64_t first_image, int world, int rank,
                            void* const* outputs, void* const* controls, void* workspace, size_t workspace_bytes,
                            void* stream, char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (int rc = check_geometry(B, Q, N, H, L, P, err, err_len)) return rc;
    if (C <= 0 || HD <= 0) return fail(err, err_len, TD_ERR_ARG, "channels and value_weight rows must be positive");
    if (HD % H != 0) return fail(err, err_len, TD_ERR_ARG, "value_weight rows must be a multiple of the head count");
    if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
        return fail(err, err_len, TD_ERR_ARG, "the peer gather takes 1 to %d ranks (rank %d of %d)", kMaxPeers, rank,
                    world);
    if (first_image < 0) return fail(err, err_len, TD_ERR_ARG, "first_image must be >= 0");
    if (outputs == nullptr || controls == nullptr) return fail(err, err_len, TD_ERR_ARG, "null peer pointer table");
    for (int r = 0; r < world; ++r)
        if (outputs[r] == nullptr || controls[r] == nullptr) return fail(err, err_len, TD_ERR_ARG, "null peer pointer");
    if (B * Q > 0 && (!memory || !value_weight || !sampling_locations || !attention_weights ||
                      (L * P > 0 && (!spatial_shapes || !level_start_index))))
        return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    const int64_t D = HD / H;
    const size_t e = dtype_size(dtype);
    const long long row_bytes = D * (long long)e;
    const long long G = row_bytes / 16;
    // the vector sampler's conditions (the value is this call's own head-major projection)
    if (row_bytes % 16 != 0 || row_bytes > 512 || (G & (G - 1)) != 0)
        return fail(err, err_len, TD_ERR_ARG, "the peer gather needs D * element size = 16, 32, ... 512 bytes");
    for (int r = 0; r < world; ++r)
        if (!aligned16(outputs[r])) return fail(err, err_len, TD_ERR_ARG, "peer outputs must be 16-byte aligned");
    const size_t need = td_project_workspace_bytes(dtype, B, N, HD);
    if (B * Q > 0 && (workspace == nullptr || workspace_bytes < need))
        return fail(err, err_len, TD_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need,
                    workspace_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* value = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
    return dispatch(dtype, [&](auto tag) -> int {
        using T = decltype(tag);
        T* v = static_cast<T*>(value);
        const bool project = B * Q > 0 && N > 0;
        if (project) {
            if (int rc = launch_proj<T>(static_cast<const T*>(memory), static_cast<const T*>(value_weight),
                                        static_cast<const T*>(value_bias), v, B, N, C, H, HD, 1, s, err, err_len,
                                        true))
                return rc;
        }
        SampleArgs<T> a;
        a.value = v; a.loc = static_cast<const T*>(sampling_locations);
        a.attn = static_cast<const T*>(attention_weights);
        a.out = nullptr; a.shapes = spatial_shapes; a.starts = level_start_index; a.prod = ProducerIn<T>{};
        a.rows = B * Q * H; a.s_img = H * N * D; a.s_tok = D; a.s_head = N * D; a.n_tok = N;
        a.mask = value_padding_mask;
        a.Q = int(Q); a.H = int(H); a.D = int(D); a.L = int(L); a.P = int(P); a.G = int(G);
        const bool wide = row_bytes % 32 == 0 && row_bytes >= 128;
        if (wide) a.G = int(row_bytes / 32);
        const bool no_alloc = B * H * N * D * (long long)e > (64LL << 20);
        PeerOut<T> po;
        PeerCtrl pc;
        for (int r = 0; r < kMaxPeers; ++r) {
            po.out[r] = r < world ? static_cast<T*>(outputs[r]) : nullptr;
            pc.p[r] = r < world ? static_cast<unsigned*>(controls[r]) : nullptr;
        }
        po.row0 = first_image * Q * H; po.world = world; po.rank = rank;
        if (a.rows > 0) {
            const unsigned grid = unsigned((a.rows + kSampleWarps - 1) / kSampleWarps);
            const size_t smem = sample_vec_smem<T>(int(L), int(P));
            DeviceFacts f;
            if (int rc = device_facts(&f, err, err_len)) return rc;
            // the same form and depth as launch_sampler's, so that the gathered rows equal the unfused path's
            const bool pair = sample_pair_form(a.rows, a.G, L, P, f.sm_count);
            const int depth = sample_batch_depth(int(4 * L * P), a.G, wide, a.rows, f.sm_count, pair ? 16 : 32);
            auto peer_launch = [&](auto k_wide, auto k_noalloc) -> cudaError_t {
                constexpr bool W = decltype(k_wide)::value, NA = decltype(k_noalloc)::value;
                const dim3 g(grid), blk(kSampleWarps * 32);
                if (pair) {
                    const dim3 g2(unsigned((a.rows + 2 * kSampleWarps - 1) / (2 * kSampleWarps)));
                    a.S_pad = sample_pair_slots(int(L), int(P), a.G, depth);
                    const size_t ps = sample_pair_smem<T>(a.S_pad);
                    if (depth == 3)
                        return launch_kernel(sample_peer_kernel<T, W, NA, 3, 2>, g2, blk, ps, s, project, a, po);
                    if (depth == 4)
                        return launch_kernel(sample_peer_kernel<T, W, NA, 4, 2>, g2, blk, ps, s, project, a, po);
                    if constexpr (!W)
                        if (depth == 6)
                            return launch_kernel(sample_peer_kernel<T, W, NA, 6, 2>, g2, blk, ps, s, project, a, po);
                    return cudaErrorInvalidValue;
                }
                if (depth == 3) return launch_kernel(sample_peer_kernel<T, W, NA, 3>, g, blk, smem, s, project, a, po);
                if (depth == 4) return launch_kernel(sample_peer_kernel<T, W, NA, 4>, g, blk, smem, s, project, a, po);
                if constexpr (!W)
                    return launch_kernel(sample_peer_kernel<T, W, NA, 6>, g, blk, smem, s, project, a, po);
                return cudaErrorInvalidValue;
            };
            const cudaError_t ce = wide       ? peer_launch(std::true_type{}, std::true_type{})
                                   : no_alloc ? peer_launch(std::false_type{}, std::true_type{})
                                              : peer_launch(std::false_type{}, std::false_type{});
            if (ce != cudaSuccess)
                return fail(err, err_len, TD_ERR_CUDA, "sample_peer_kernel launch: %s", cudaGetErrorString(ce));
            g_launches.fetch_add(1, std::memory_order_relaxed);
            if (int rc = check_launch(err, err_len, "sample_peer_kernel")) return rc;
        }
        if (world == 1) return int(TD_OK);
        // a rank with an empty shard still signals its peers and waits for theirs
        const cudaError_t ce = launch_kernel(peer_signal_wait_kernel, dim3(1), dim3(32), 0, s, true, pc, world, rank,
                                             1, kSpinLimitCycles);
        if (ce != cudaSuccess)
            return fail(err, err_len, TD_ERR_CUDA, "peer_signal_wait_kernel launch: %s", cudaGetErrorString(ce));
        g_launches.fetch_add(1, std::memory_order_relaxed);
        return check_launch(err, err_len, "peer_signal_wait_kernel");
    });
}

int td_test_peer_wait(void* control, int world, int rank, long long limit_cycles, void* stream, char* err,
                      size_t err_len) {
    if (control == nullptr || world < 2 || world > kMaxPeers || rank < 0 || rank >= world || limit_cycles <= 0)
        return fail(err, err_len, TD_ERR_ARG, "bad peer wait arguments");
    PeerCtrl pc;
    for (int r = 0; r < kMaxPeers; ++r) pc.p[r] = r == rank ? static_cast<unsigned*>(control) : nullptr;
    const cudaError_t ce = launch_kernel(peer_signal_wait_kernel, dim3(1), dim3(32), 0,
                                         static_cast<cudaStream_t>(stream), false, pc, world, rank, 0, limit_cycles);
    if (ce != cudaSuccess)
        return fail(err, err_len, TD_ERR_CUDA, "peer_signal_wait_kernel launch: %s", cudaGetErrorString(ce));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "peer_signal_wait_kernel");
}

size_t td_layer_workspace_bytes(int dtype, int order, int64_t B, int64_t Q, int64_t N, int64_t H, int64_t HD,
                                int64_t L, int64_t P, int output_proj) {
    const size_t e = dtype_size(dtype);
    if (e == 0 || (order != TD_ORDER_PROJECT && order != TD_ORDER_FUSED) || B < 0 || Q < 0 || N < 0 || H < 0 ||
        HD < 0 || L < 0 || P < 0)
        return 0;
    return layer_workspace(e, order, B, Q, N, H, HD, L, P, output_proj != 0).bytes;
}

int td_layer_forward(int dtype, int order, const void* query, int64_t Cq, const void* reference_points, int ref_dim,
                     const void* sampling_weight, const void* sampling_bias, const void* memory,
                     const void* value_weight, const void* value_bias, const uint8_t* value_padding_mask,
                     const int64_t* spatial_shapes, const int64_t* level_start_index, const void* output_weight,
                     const void* output_bias, int64_t C_out, void* out, int64_t B, int64_t Q, int64_t N, int64_t C,
                     int64_t H, int64_t HD, int64_t L, int64_t P, void* workspace, size_t workspace_bytes,
                     void* stream, char* err, size_t err_len) {
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (order != TD_ORDER_PROJECT && order != TD_ORDER_FUSED)
        return fail(err, err_len, TD_ERR_ARG, "order must be TD_ORDER_PROJECT or TD_ORDER_FUSED, got %d", order);
    if (int rc = check_geometry(B, Q, N, H, L, P, err, err_len)) return rc;
    if (L <= 0 || P <= 0) return fail(err, err_len, TD_ERR_ARG, "the layer needs at least one level and one point");
    if (C <= 0 || Cq <= 0 || HD <= 0)
        return fail(err, err_len, TD_ERR_ARG, "channels and value_weight rows must be positive");
    if (HD % H != 0) return fail(err, err_len, TD_ERR_ARG, "value_weight rows must be a multiple of the head count");
    if (ref_dim != 2 && ref_dim != 4)
        return fail(err, err_len, TD_ERR_ARG, "reference points must have 2 (x, y) or 4 (cx, cy, w, h) coordinates");
    if (output_weight != nullptr && C_out <= 0)
        return fail(err, err_len, TD_ERR_ARG, "the output projection needs C_out > 0");
    if (output_weight == nullptr && output_bias != nullptr)
        return fail(err, err_len, TD_ERR_ARG, "output_bias needs output_weight");
    if (order == TD_ORDER_FUSED && C > TD_MAX_CHANNELS)
        return fail(err, err_len, TD_ERR_ARG, "channels must be <= %d", TD_MAX_CHANNELS);
    if (Cq > INT32_MAX || C > INT32_MAX || HD > INT32_MAX || C_out > INT32_MAX || B * Q > INT32_MAX)
        return fail(err, err_len, TD_ERR_ARG, "size too large");
    if (B * Q == 0) return TD_OK;
    if (!query || !reference_points || !sampling_weight || !memory || !value_weight || !spatial_shapes ||
        !level_start_index || !out)
        return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    const size_t e = dtype_size(dtype);
    const LayerWorkspace w = layer_workspace(e, order, B, Q, N, H, HD, L, P, output_weight != nullptr);
    if (workspace == nullptr || workspace_bytes < w.bytes)
        return fail(err, err_len, TD_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", w.bytes,
                    workspace_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned char* ws = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
    const int64_t D = HD / H, LP3 = 3 * H * L * P;
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        T* proj = reinterpret_cast<T*>(ws + w.proj);
        T* target = output_weight != nullptr ? reinterpret_cast<T*>(ws + w.mid) : static_cast<T*>(out);
        const T* ref = static_cast<const T*>(reference_points);
        // the query projection: offsets and attention logits of every (batch, query) row
        const ProjShape jq{query, sampling_weight, sampling_bias, proj, 1, B * Q, Cq, 1, LP3, 0};
        auto query_proj = [&] {
            return launch_proj<T>(static_cast<const T*>(query), static_cast<const T*>(sampling_weight),
                                  static_cast<const T*>(sampling_bias), proj, 1, B * Q, Cq, 1, LP3, 0, s, err,
                                  err_len, true);
        };
        if (order == TD_ORDER_PROJECT) {
            // 1. the value projection (head-major) and the query projection, in one tcgen05 launch when both fit it
            // (the query tiles take SMs the value tiles leave idle), else one after the other; 2. the sampler, whose
            // corner prologue runs the producer on the query projection (see sample_vec_kernel)
            T* value = reinterpret_cast<T*>(ws + w.value);
            bool paired = false;
            if (N > 0) {
                const ProjShape jv{memory, value_weight, value_bias, value, B, N, C, H, HD, 1};
                if (int rc = launch_proj_pair<T>(jv, jq, s, true, &paired, err, err_len)) return rc;
            }
            if (!paired) {
                if (int rc = query_proj()) return rc;
                if (N > 0) {
                    if (int rc = launch_proj<T>(static_cast<const T*>(memory), static_cast<const T*>(value_weight),
                                                static_cast<const T*>(value_bias), value, B, N, C, H, HD, 1, s, err,
                                                err_len, true))
                        return rc;
                }
            }
            ProducerIn<T> prod;
            prod.proj = proj; prod.ref = ref; prod.ref_dim = ref_dim; prod.wait_first = paired ? 1 : 0;
            if (output_weight != nullptr) {
                // output_proj in the sampler's own kernel, where the plan and the shapes allow it
                const int rc = launch_sample_outproj<T>(
                    value, H * N * D, D, N * D, spatial_shapes, level_start_index, nullptr, nullptr,
                    static_cast<const T*>(output_weight), static_cast<const T*>(output_bias), static_cast<T*>(out),
                    C_out, B, Q, N, H, D, L, P, s, err, err_len, N > 0, value_padding_mask, prod);
                if (rc != kNotApplicable) return rc;
            }
            // with no value projection in between, the sampler follows the query projection in plain stream order
            if (int rc = launch_sampler<T>(value, H * N * D, D, N * D, spatial_shapes, level_start_index, nullptr,
                                           nullptr, target, B, Q, N, H, D, L, P, s, err, err_len, N > 0,
                                           value_padding_mask, prod))
                return rc;
        } else {
            // 1. the query projection, 2. locations and weights, 3. the fused gather-then-project kernel
            if (int rc = query_proj()) return rc;
            T* loc = reinterpret_cast<T*>(ws + w.loc);
            T* attn = reinterpret_cast<T*>(ws + w.attn);
            if (int rc = launch_producer<T>(proj, ref, ref_dim, spatial_shapes, loc, attn, B, Q, H, L, P, s, err,
                                            err_len))
                return rc;
            if (int rc = launch_fused<T>(static_cast<const T*>(memory), static_cast<const T*>(value_weight),
                                         static_cast<const T*>(value_bias), spatial_shapes, level_start_index, loc,
                                         attn, target, B, Q, N, C, H, D, L, P, s, err, err_len, value_padding_mask))
                return rc;
        }
        if (output_weight == nullptr) return int(TD_OK);
        // then the output projection of the attention result
        return launch_proj<T>(target, static_cast<const T*>(output_weight), static_cast<const T*>(output_bias),
                              static_cast<T*>(out), 1, B * Q, HD, 1, C_out, 0, s, err, err_len, true);
    });
}

size_t td_project_ex_workspace_bytes(int dtype, int64_t B, int64_t Q, int64_t N, int64_t HD, int output_proj) {
    const size_t e = dtype_size(dtype);
    if (e == 0 || B < 0 || Q < 0 || N < 0 || HD < 0) return 0;
    const size_t value = (size_t(B) * size_t(N) * size_t(HD) * e + 255) & ~size_t(255);
    const size_t mid = output_proj ? size_t(B) * size_t(Q) * size_t(HD) * e : 0;
    return value + mid + 256;
}

int td_project_forward_ex(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                          const int64_t* spatial_shapes, const int64_t* level_start_index,
                          const void* sampling_locations, const void* attention_weights,
                          const uint8_t* value_padding_mask, const void* output_weight, const void* output_bias,
                          int64_t C_out, void* out, int64_t B, int64_t Q, int64_t N, int64_t C, int64_t H,
                          int64_t HD, int64_t L, int64_t P, void* workspace, size_t workspace_bytes, void* stream,
                          char* err, size_t err_len) {
    if (output_weight == nullptr) {
        if (output_bias != nullptr) return fail(err, err_len, TD_ERR_ARG, "output_bias needs output_weight");
        return td_project_forward_masked(dtype, memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                         sampling_locations, attention_weights, value_padding_mask, out, B, Q, N, C,
                                         H, HD, L, P, workspace, workspace_bytes, stream, err, err_len);
    }
    if (dtype_size(dtype) == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (int rc = check_geometry(B, Q, N, H, L, P, err, err_len)) return rc;
    if (C <= 0 || HD <= 0) return fail(err, err_len, TD_ERR_ARG, "channels and value_weight rows must be positive");
    if (HD % H != 0) return fail(err, err_len, TD_ERR_ARG, "value_weight rows must be a multiple of the head count");
    if (C_out <= 0 || C_out > INT32_MAX || HD > INT32_MAX)
        return fail(err, err_len, TD_ERR_ARG, "output_proj needs 0 < C_out < 2^31");
    if (B * Q == 0) return TD_OK;
    if (!memory || !value_weight || !sampling_locations || !attention_weights || !out ||
        (L * P > 0 && (!spatial_shapes || !level_start_index)))
        return fail(err, err_len, TD_ERR_ARG, "null tensor pointer");
    const size_t need = td_project_ex_workspace_bytes(dtype, B, Q, N, HD, 1);
    if (workspace == nullptr || workspace_bytes < need)
        return fail(err, err_len, TD_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need,
                    workspace_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t D = HD / H;
    unsigned char* ws =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
    const size_t value_bytes = (size_t(B) * size_t(N) * size_t(HD) * dtype_size(dtype) + 255) & ~size_t(255);
    return dispatch(dtype, [&](auto tag) {
        using T = decltype(tag);
        T* v = reinterpret_cast<T*>(ws);
        T* mid = reinterpret_cast<T*>(ws + value_bytes);
        if (N > 0) {
            if (int rc = launch_proj<T>(static_cast<const T*>(memory), static_cast<const T*>(value_weight),
                                        static_cast<const T*>(value_bias), v, B, N, C, H, HD, 1, s, err, err_len,
                                        true))
                return rc;
        }
        {
            // output_proj in the sampler's own kernel, where the plan and the shapes allow it
            const int rc = launch_sample_outproj<T>(
                v, H * N * D, D, N * D, spatial_shapes, level_start_index, static_cast<const T*>(sampling_locations),
                static_cast<const T*>(attention_weights), static_cast<const T*>(output_weight),
                static_cast<const T*>(output_bias), static_cast<T*>(out), C_out, B, Q, N, H, D, L, P, s, err,
                err_len, N > 0, value_padding_mask);
            if (rc != kNotApplicable) return rc;
        }
        if (int rc = launch_sampler<T>(v, H * N * D, D, N * D, spatial_shapes, level_start_index,
                                       static_cast<const T*>(sampling_locations),
                                       static_cast<const T*>(attention_weights), mid, B, Q, N, H, D, L, P, s, err,
                                       err_len, N > 0, value_padding_mask))
            return rc;
        return launch_proj<T>(mid, static_cast<const T*>(output_weight), static_cast<const T*>(output_bias),
                              static_cast<T*>(out), 1, B * Q, HD, 1, C_out, 0, s, err, err_len, true);
    });
}

}  // extern "C"

// Scratch of td_project_forward_noalloc: the projected value of one call. A host-side name for device memory, so
// host code only ever passes the address cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[TD_NOALLOC_SCRATCH_BYTES];

namespace td {
namespace {
// The scratch array's device address per device, stored only once a lookup has succeeded (a failed lookup leaves
// nullptr, and the next call tries again).
std::atomic<void*> g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mutex;

int scratch_address(cudaStream_t stream, void** out, char* err, size_t err_len) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(err, err_len, TD_ERR_CUDA, "device index %d out of range", dev);
    void* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
    if (p == nullptr) {
        std::lock_guard<std::mutex> lock(g_scratch_mutex);
        p = g_scratch_ptr[dev].load(std::memory_order_acquire);
        if (p == nullptr) {
            cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
            e = cudaStreamIsCapturing(stream, &capturing);
            if (e != cudaSuccess) {
                cudaGetLastError();
                return fail(err, err_len, TD_ERR_CUDA, "cudaStreamIsCapturing: %s", cudaGetErrorString(e));
            }
            if (capturing != cudaStreamCaptureStatusNone)
                return fail(err, err_len, TD_ERR_CUDA,
                            "the first td_project_forward_noalloc call on device %d looks up its scratch array "
                            "and must come before any stream capture on that device",
                            dev);
            e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || p == nullptr) {
                cudaGetLastError();  // not sticky: leave no error behind for the next launch check
                return fail(err, err_len, TD_ERR_CUDA, "cudaGetSymbolAddress of the scratch array on device %d: %s",
                            dev, cudaGetErrorString(e));
            }
            g_scratch_ptr[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
    return TD_OK;
}
}  // namespace
}  // namespace td

extern "C" {

int td_project_forward_noalloc(int dtype, const void* memory, const void* value_weight, const void* value_bias,
                               const int64_t* spatial_shapes, const int64_t* level_start_index,
                               const void* sampling_locations, const void* attention_weights, void* out,
                               int64_t B, int64_t Q, int64_t N, int64_t C, int64_t H, int64_t HD, int64_t L,
                               int64_t P, void* stream, char* err, size_t err_len) {
    // argument checks first (the same as td_project_forward's), so that a bad call never reaches the device
    const size_t e = dtype_size(dtype);
    if (e == 0) return fail(err, err_len, TD_ERR_ARG, "unsupported dtype code %d", dtype);
    if (int rc = check_geometry(B, Q, N, H, L, P, err, err_len)) return rc;
    if (C <= 0 || HD <= 0) return fail(err, err_len, TD_ERR_ARG, "channels and value_weight rows must be positive");
    if (HD % H != 0) return fail(err, err_len, TD_ERR_ARG, "value_weight rows must be a multiple of the head count");
    if (B * Q == 0) return TD_OK;
    // B * N * HD * e + 256 with every product checked, so that absurd sizes cannot wrap below the limit
    size_t need = 0;
    const bool wraps = __builtin_mul_overflow(size_t(B), size_t(N), &need) ||
                       __builtin_mul_overflow(need, size_t(HD), &need) || __builtin_mul_overflow(need, e, &need) ||
                       __builtin_add_overflow(need, size_t(256), &need);
    if (wraps)
        return fail(err, err_len, TD_ERR_WORKSPACE,
                    "the allocation-free project order holds at most %zu bytes of projected value, this call needs "
                    "more than SIZE_MAX (B * N * H * D elements)",
                    size_t(TD_NOALLOC_SCRATCH_BYTES));
    if (need > TD_NOALLOC_SCRATCH_BYTES)
        return fail(err, err_len, TD_ERR_WORKSPACE,
                    "the allocation-free project order holds at most %zu bytes of projected value, this call "
                    "needs %zu (B * N * H * D elements plus 256 bytes of alignment)",
                    size_t(TD_NOALLOC_SCRATCH_BYTES), need);
    void* scratch = nullptr;
    if (int rc = scratch_address(static_cast<cudaStream_t>(stream), &scratch, err, err_len)) return rc;
    return td_project_forward(dtype, memory, value_weight, value_bias, spatial_shapes, level_start_index,
                              sampling_locations, attention_weights, out, B, Q, N, C, H, HD, L, P, scratch,
                              TD_NOALLOC_SCRATCH_BYTES, stream, err, err_len);
}

int td_probe_row_gather(const void* buf, int64_t rows, int row_bytes, int wide, int64_t visits, unsigned seed,
                        void* sink, size_t sink_bytes, int grid, void* stream, char* err, size_t err_len) {
    const int word = wide ? 32 : 16;
    if (row_bytes < word || row_bytes > 512 || (row_bytes & (row_bytes - 1)) != 0)
        return fail(err, err_len, TD_ERR_ARG, "row_bytes must be a power of two from %d to 512", word);
    if (buf == nullptr || sink == nullptr || rows <= 0 || grid <= 0 || visits < 0)
        return fail(err, err_len, TD_ERR_ARG, "need a buffer, a sink, rows > 0 and grid > 0");
    if ((reinterpret_cast<uintptr_t>(buf) & uintptr_t(word - 1)) != 0)
        return fail(err, err_len, TD_ERR_ARG, "buf must be %d-byte aligned", word);
    if (sink_bytes < size_t(grid) * kProbeThreads * 16 || !aligned16(sink))
        return fail(err, err_len, TD_ERR_ARG, "sink needs grid * %d 16-byte words, 16-byte aligned", kProbeThreads);
    const long long chunk = (long long)grid * (kProbeThreads / 32) * (32 / (row_bytes / word)) * (wide ? 4 : 8);
    if (visits % chunk != 0)
        return fail(err, err_len, TD_ERR_ARG, "visits must be a multiple of %lld for this grid", chunk);
    ProbeArgs a;
    a.buf = static_cast<const unsigned char*>(buf);
    a.rows = (unsigned long long)rows;
    a.visits = visits;
    a.row_bytes = row_bytes;
    a.seed = seed;
    a.sink = static_cast<uint4*>(sink);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const cudaError_t e = wide ? launch_kernel(row_gather_probe_kernel<true>, dim3(grid), dim3(kProbeThreads), 0, s,
                                               false, a)
                               : launch_kernel(row_gather_probe_kernel<false>, dim3(grid), dim3(kProbeThreads), 0,
                                               s, false, a);
    if (e != cudaSuccess)
        return fail(err, err_len, TD_ERR_CUDA, "row_gather_probe_kernel launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch(err, err_len, "row_gather_probe_kernel");
}

int td_test_starve_next_grad_gemm(long long spin_limit_cycles) {
    if (spin_limit_cycles <= 0 || spin_limit_cycles > kSpinLimitCycles) return TD_ERR_ARG;
    g_starve_next.store(spin_limit_cycles);
    return TD_OK;
}

int td_device_info(int device, int* sm_count, int* cc_major, int* cc_minor, char* err, size_t err_len) {
    cudaError_t e = cudaDeviceGetAttribute(sm_count, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(cc_major, cudaDevAttrComputeCapabilityMajor, device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(cc_minor, cudaDevAttrComputeCapabilityMinor, device);
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "device %d: %s", device, cudaGetErrorString(e));
    return TD_OK;
}

int td_set_kernel_policy(int policy) {
    if (policy != TD_POLICY_BEST && policy != TD_POLICY_CUDA_CORES) return -1;
    return g_policy.exchange(policy);
}

int td_set_output_proj_plan(int plan) {
    if (plan != TD_OUTPROJ_AUTO && plan != TD_OUTPROJ_CHAINED && plan != TD_OUTPROJ_CLUSTER) return -1;
    return g_outproj_plan.exchange(plan);
}

int td_device_error(int clear, unsigned int* code, char* err, size_t err_len) {
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v));
    if (e == cudaSuccess && clear) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    }
    if (e != cudaSuccess) return fail(err, err_len, TD_ERR_CUDA, "device error word: %s", cudaGetErrorString(e));
    if (code != nullptr) *code = v;
    return TD_OK;
}

uint64_t td_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* td_version(void) { return "0.1.1+b200"; }

}  // extern "C"
