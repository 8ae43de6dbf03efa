// Device helpers shared by the neighbor-list kernels.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "tnr_plan.h"

namespace tnr {

constexpr unsigned kFullMask = 0xffffffffu;

template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
    using type = float4;
};
template <>
struct Vec4<double> {
    using type = double4;
};
template <typename T>
using vec4_t = typename Vec4<T>::type;

// ---- IEEE round-to-nearest arithmetic without contraction -----------------
// The decisive cutoff predicate must evaluate the reference's expression
// (tonari csrc/core/neighbors_cpu.cpp:247-260) operation by operation; nvcc
// would otherwise fuse multiply-adds.
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }

// Target index stored in the fourth lane of a ghost record.
__device__ __forceinline__ float index_to_lane(int32_t v, float) { return __int_as_float(v); }
__device__ __forceinline__ double index_to_lane(int32_t v, double) {
    return __longlong_as_double(static_cast<long long>(v));
}
__device__ __forceinline__ int32_t lane_to_index(float v) { return __float_as_int(v); }
__device__ __forceinline__ int32_t lane_to_index(double v) {
    return static_cast<int32_t>(__double_as_longlong(v));
}

// ---- order-preserving keys for atomic min / max of floating values --------
__device__ __forceinline__ int32_t order_key(float v) {
    const int32_t bits = __float_as_int(v);
    return bits >= 0 ? bits : bits ^ 0x7fffffff;
}
__device__ __forceinline__ long long order_key(double v) {
    const long long bits = __double_as_longlong(v);
    return bits >= 0 ? bits : bits ^ 0x7fffffffffffffffLL;
}

// One component of the public displacement, in the reference's order:
// (p_t - p_s) + S0*cell[0][c] + S1*cell[1][c] + S2*cell[2][c].
template <typename T>
__device__ __forceinline__ T exact_component(T target, T source, const long long (&shift)[3],
                                             const T* cell, int c) {
    T value = sub_rn(target, source);
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        value = add_rn(value, mul_rn(static_cast<T>(shift[a]), cell[3 * a + c]));
    }
    return value;
}

template <typename T>
__device__ __forceinline__ T exact_norm2(T x, T y, T z) {
    return add_rn(add_rn(mul_rn(x, x), mul_rn(y, y)), mul_rn(z, z));
}

// Pair identity rule, tonari csrc/core/pair_policy.h:42-79.
__device__ __forceinline__ bool canonical_shift(const long long (&shift)[3]) {
    if (shift[0] != 0) return shift[0] < 0;
    if (shift[1] != 0) return shift[1] < 0;
    if (shift[2] != 0) return shift[2] < 0;
    return true;
}

__device__ __forceinline__ bool keep_identity(int64_t source, int64_t target,
                                              const long long (&shift)[3], bool half,
                                              bool include_self) {
    const bool zero = shift[0] == 0 && shift[1] == 0 && shift[2] == 0;
    if (source == target && zero) return include_self;
    if (!half) return true;
    if (source != target) return source < target;
    return canonical_shift(shift);
}

// Image k of a structure with the given repeats, enumerated x-major, then y,
// then z (tonari csrc/core/geometry.cpp:229-237).
__device__ __forceinline__ void decode_image(int32_t k, const int32_t (&repeats)[3],
                                             int32_t (&image)[3]) {
    const int32_t ny = 2 * repeats[1] + 1;
    const int32_t nz = 2 * repeats[2] + 1;
    const int32_t yz = ny * nz;
    const int32_t x = k / yz;
    const int32_t rem = k - x * yz;
    const int32_t y = rem / nz;
    image[0] = x - repeats[0];
    image[1] = y - repeats[1];
    image[2] = rem - y * nz - repeats[2];
}

// Cartesian bin coordinate of a point; identical code in every kernel so the
// binning, scatter and stencil passes agree bit for bit.
template <typename T>
__device__ __forceinline__ int32_t bin_axis(T value, T origin, T inv_edge, int32_t dim) {
    const T u = mul_rn(sub_rn(value, origin), inv_edge);
    int32_t b = static_cast<int32_t>(floor(u));
    b = b < 0 ? 0 : b;
    return b >= dim ? dim - 1 : b;
}

// Index of the structure containing `atom`: the b with
// batch_ptr[b] <= atom < batch_ptr[b+1] (skipping empty structures).
// The search may be narrowed to [lo, hi) when the answer is known to be there.
__device__ __forceinline__ int32_t structure_of(const int64_t* __restrict__ batch_ptr,
                                                int64_t batch, int64_t atom, int64_t lo = 0,
                                                int64_t hi = -1) {
    if (hi < 0) hi = batch;  // answer in [lo, hi)
    while (hi - lo > 1) {
        const int64_t mid = (lo + hi) >> 1;
        if (batch_ptr[mid] <= atom) lo = mid; else hi = mid;
    }
    return static_cast<int32_t>(lo);
}

// Position of `value` in a nondecreasing prefix array of length count+1:
// the k with prefix[k] <= value < prefix[k+1].
// The search may be narrowed to [lo, hi) when the answer is known to be there.
__device__ __forceinline__ int32_t segment_of(const int64_t* __restrict__ prefix, int32_t count,
                                              int64_t value, int32_t lo = 0, int32_t hi = -1) {
    if (hi < 0) hi = count;
    while (hi - lo > 1) {
        const int32_t mid = (lo + hi) >> 1;
        if (prefix[mid] <= value) lo = mid; else hi = mid;
    }
    return lo;
}

// The same search by a whole warp (all 32 lanes call it with equal
// arguments): the largest k in [lo, hi) with prefix[k] <= value, given
// prefix[lo] <= value and prefix nondecreasing.  Each step narrows the range
// 32-fold with one load per lane, so a block's first structure is found in
// a few dependent loads instead of one per halving.
__device__ __forceinline__ int64_t warp_last_le(const int64_t* __restrict__ prefix, int64_t lo,
                                                int64_t hi, int64_t value) {
    const int lane = threadIdx.x & 31;
    while (hi - lo > 1) {
        const int64_t step = (hi - lo + 31) / 32;
        const int64_t k = lo + lane * step;
        const bool le = k < hi && prefix[k] <= value;
        const unsigned ballot = __ballot_sync(0xffffffffu, le);
        lo += static_cast<int64_t>(31 - __clz(ballot)) * step;
        hi = min(lo + step, hi);
    }
    return lo;
}

}  // namespace tnr
