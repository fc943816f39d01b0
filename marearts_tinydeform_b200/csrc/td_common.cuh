// td_common.cuh -- element types, 16-byte vector loads, and the bilinear corner rule shared by every kernel.
//
// The corner rule is the operator's definition of sampling (grid_sample, bilinear, zero padding,
// align_corners=False), in the form upstream's CUDA kernel evaluates it (csrc/ma_deform_fused.cu:79-100):
//   x = clamp(loc_x * w_l - 0.5, -2, w_l + 1), y likewise with h_l; x0 = floor(x), fx = x - x0;
//   corner (dx, dy) has token start_l + (y0 + dy) * w_l + (x0 + dx) and weight attn * (dx ? fx : 1 - fx) * (dy ? ...)
//   and counts only when it lies inside the level's map and inside [0, N).
// The clamp keeps far-away, infinite and NaN locations from overflowing the int conversion; they sample nothing.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace td {

constexpr int kMaxLevelPoints = 64;   // levels x points per head
constexpr int kMaxCorners = kMaxLevelPoints * 4;
constexpr int kMaxLevels = 64;

// Accumulator type and elements per 16-byte vector for each storage type.
template <typename T> struct Elem;
template <> struct Elem<float> { using acc = float; static constexpr int kVec = 4; };
template <> struct Elem<__half> { using acc = float; static constexpr int kVec = 8; };
template <> struct Elem<__nv_bfloat16> { using acc = float; static constexpr int kVec = 8; };
template <> struct Elem<double> { using acc = double; static constexpr int kVec = 2; };

__device__ __forceinline__ float to_acc(float v) { return v; }
__device__ __forceinline__ float to_acc(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_acc(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ double to_acc(double v) { return v; }

template <typename T> __device__ __forceinline__ T from_acc(typename Elem<T>::acc v);
template <> __device__ __forceinline__ float from_acc<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_acc<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ double from_acc<double>(double v) { return v; }

// Read-only 16-byte load, widened to the accumulator type.
template <typename T>
__device__ __forceinline__ void load16(const T* p, typename Elem<T>::acc* o);

template <>
__device__ __forceinline__ void load16<float>(const float* p, float* o) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}
template <>
__device__ __forceinline__ void load16<__half>(const __half* p, float* o) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        o[2 * i] = f.x; o[2 * i + 1] = f.y;
    }
}
template <>
__device__ __forceinline__ void load16<__nv_bfloat16>(const __nv_bfloat16* p, float* o) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        o[2 * i] = f.x; o[2 * i + 1] = f.y;
    }
}
template <>
__device__ __forceinline__ void load16<double>(const double* p, double* o) {
    const double2 v = __ldg(reinterpret_cast<const double2*>(p));
    o[0] = v.x; o[1] = v.y;
}

// Widen a raw 16-byte vector (already loaded) to kVec accumulators.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& v, typename Elem<T>::acc* o);

template <>
__device__ __forceinline__ void unpack16<float>(const uint4& v, float* o) {
    o[0] = __uint_as_float(v.x); o[1] = __uint_as_float(v.y); o[2] = __uint_as_float(v.z); o[3] = __uint_as_float(v.w);
}
template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& v, float* o) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        o[2 * i] = f.x; o[2 * i + 1] = f.y;
    }
}
template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& v, float* o) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        o[2 * i] = f.x; o[2 * i + 1] = f.y;
    }
}
template <>
__device__ __forceinline__ void unpack16<double>(const uint4& v, double* o) {
    o[0] = __hiloint2double(int(v.y), int(v.x));
    o[1] = __hiloint2double(int(v.w), int(v.z));
}

// Narrow kVec accumulators to T and store them as one 16-byte vector.
template <typename T>
__device__ __forceinline__ void store16(T* p, const typename Elem<T>::acc* v);

template <>
__device__ __forceinline__ void store16<float>(float* p, const float* v) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
template <>
__device__ __forceinline__ void store16<__half>(__half* p, const float* v) {
    uint4 o;
    uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(p) = o;
}
template <>
__device__ __forceinline__ void store16<__nv_bfloat16>(__nv_bfloat16* p, const float* v) {
    uint4 o;
    uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(p) = o;
}
template <>
__device__ __forceinline__ void store16<double>(double* p, const double* v) {
    *reinterpret_cast<double2*>(p) = make_double2(v[0], v[1]);
}

// Coordinate arithmetic is float32 for the 16/32-bit types (as upstream) and float64 for float64 inputs.
template <typename T> struct Coord { using type = float; };
template <> struct Coord<double> { using type = double; };

__device__ __forceinline__ float cmin(float a, float b) { return fminf(a, b); }
__device__ __forceinline__ float cmax(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ double cmin(double a, double b) { return fmin(a, b); }
__device__ __forceinline__ double cmax(double a, double b) { return fmax(a, b); }
__device__ __forceinline__ float cfloor(float a) { return floorf(a); }
__device__ __forceinline__ double cfloor(double a) { return floor(a); }

// Level geometry as the kernels keep it in shared memory.
struct Level {
    int h, w;
    long long start;
};

// Load the (height, width, first token) of every level into shared memory. Negative or oversized sizes are
// clamped to [0, 2^30] so the corner arithmetic below cannot overflow; such levels sample nothing or stay in
// range through the [0, N) test.
__device__ __forceinline__ void load_levels(const int64_t* __restrict__ shapes, const int64_t* __restrict__ starts,
                                            int L, Level* lv) {
    for (int l = threadIdx.x; l < L; l += blockDim.x) {
        long long h = shapes[2 * l], w = shapes[2 * l + 1];
        h = h < 0 ? 0 : (h > (1LL << 30) ? (1LL << 30) : h);
        w = w < 0 ? 0 : (w > (1LL << 30) ? (1LL << 30) : w);
        lv[l].h = int(h);
        lv[l].w = int(w);
        lv[l].start = starts[l];
    }
}

// The geometry of level l read straight from the device arrays (same clamping as load_levels), for kernels that
// fetch it together with the sampling locations instead of staging it first.
__device__ __forceinline__ Level level_at(const int64_t* __restrict__ shapes, const int64_t* __restrict__ starts,
                                          int l) {
    long long h = shapes[2 * l], w = shapes[2 * l + 1];
    Level lv;
    lv.h = int(h < 0 ? 0 : (h > (1LL << 30) ? (1LL << 30) : h));
    lv.w = int(w < 0 ? 0 : (w > (1LL << 30) ? (1LL << 30) : w));
    lv.start = starts[l];
    return lv;
}

// The level of sampling point j (points are level-major, P per level): a shift when P is a power of two (the usual
// 4, 8 or 16), where a division by the runtime P costs ~20 instructions in every corner prologue.
__device__ __forceinline__ int level_of(int j, int P) {
    return P > 0 && (P & (P - 1)) == 0 ? j >> (__ffs(P) - 1) : j / P;
}

// The four bilinear corners of one sampling point. tok[k] = -1 marks a corner outside the map (it contributes
// nothing, as zero padding); inside corners carry attn * bilinear weight, which may itself be 0. mask_b (the value
// padding mask of the image, one byte per token, nonzero = padded; or null) turns a corner on a padded token into
// an outside one: its value row counts as zero, as Deformable-DETR's masked_fill after the value projection makes
// it (bias included).
template <typename CT>
__device__ __forceinline__ void corners4(CT lx, CT ly, CT a, const Level& lv, long long n_tok, int* tok, CT* wt,
                                         const uint8_t* mask_b = nullptr) {
    const CT x = cmin(cmax(lx * CT(lv.w) - CT(0.5), CT(-2)), CT(lv.w) + CT(1));
    const CT y = cmin(cmax(ly * CT(lv.h) - CT(0.5), CT(-2)), CT(lv.h) + CT(1));
    const CT xf = cfloor(x), yf = cfloor(y);
    const int x0 = int(xf), y0 = int(yf);
    const CT fx = x - xf, fy = y - yf;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int dx = k & 1, dy = k >> 1, xi = x0 + dx, yi = y0 + dy;
        const long long t = lv.start + (long long)yi * lv.w + xi;
        bool in = xi >= 0 && xi < lv.w && yi >= 0 && yi < lv.h && t >= 0 && t < n_tok;
        if (in && mask_b != nullptr) in = mask_b[t] == 0;
        tok[k] = in ? int(t) : -1;
        wt[k] = in ? a * (dx ? fx : CT(1) - fx) * (dy ? fy : CT(1) - fy) : CT(0);
    }
}

// Corners of sample j (level j / P) of row bqh, read straight from sampling_locations / attention_weights.
template <typename T>
__device__ __forceinline__ void row_corners(const T* __restrict__ loc, const T* __restrict__ attn, const Level* lv,
                                            int LP, int P, long long n_tok, long long bqh, int j, int* tok,
                                            typename Coord<T>::type* wt, const uint8_t* mask_b = nullptr) {
    using CT = typename Coord<T>::type;
    const long long i = bqh * LP + j;
    const CT lx = CT(to_acc(loc[2 * i])), ly = CT(to_acc(loc[2 * i + 1]));
    const CT a = CT(to_acc(attn[i]));
    corners4<CT>(lx, ly, a, lv[j / P], n_tok, tok, wt, mask_b);
}

}  // namespace td
