// Device helpers shared by the CUDA translation units: element decode for
// the reference's low storage, index nests, ordered float keys and block
// reductions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace fb {

// Element offset of `linear` inside a row-major nest (index_of,
// compute-cuda/src/kernels.cu:5-13).  Fully unrolled so the nest stays in
// kernel-parameter space.
__device__ __forceinline__ uint64_t nest_offset(const Nest& n, uint64_t linear) {
    uint64_t off = 0;
#pragma unroll
    for (int d = FB_MAX_RANK - 1; d >= 0; --d) {
        if (d < (int)n.rank) {
            const uint64_t dim = n.dims[d];
            off += (linear % dim) * n.strides[d];
            linear /= dim;
        }
    }
    return off;
}

// decode_low (compute-cuda/src/low_precision.cu:17-24): BF16 is the high
// half of an f32; F16 converts exactly.  Subnormals are preserved.
__device__ __forceinline__ float bf16_bits_to_float(uint16_t bits) { return __uint_as_float((uint32_t)bits << 16); }
__device__ __forceinline__ float f16_bits_to_float(uint16_t bits) { return __half2float(__ushort_as_half(bits)); }

template <typename T>
struct Elem;
template <>
struct Elem<float> {
    static __device__ __forceinline__ float load(const float* p) { return __ldg(p); }
    // Four consecutive elements from a 16-byte aligned address.
    static __device__ __forceinline__ float4 load4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
};
template <>
struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float load(const __nv_bfloat16* p) {
        return bf16_bits_to_float(__ldg(reinterpret_cast<const unsigned short*>(p)));
    }
    static __device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
        return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                           __uint_as_float(u.y & 0xffff0000u));
    }
};
template <>
struct Elem<__half> {
    static __device__ __forceinline__ float load(const __half* p) {
        return f16_bits_to_float(__ldg(reinterpret_cast<const unsigned short*>(p)));
    }
    static __device__ __forceinline__ float4 load4(const __half* p) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
        return make_float4(f16_bits_to_float((uint16_t)(u.x & 0xffff)), f16_bits_to_float((uint16_t)(u.x >> 16)),
                           f16_bits_to_float((uint16_t)(u.y & 0xffff)), f16_bits_to_float((uint16_t)(u.y >> 16)));
    }
};

// Total-order key of an f32 (reduce_float_key, compute-cuda/src/reductions.cu:
// 31-34): unsigned comparison of keys orders -0 < +0 and preserves bits.
// Three-input min/max that propagate NaN (sm_100 forms).
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
    float d;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ float min3_nan(float a, float b, float c) {
    float d;
    asm("min.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ uint32_t order_key(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// encode_low (compute-cuda/src/low_precision.cu:6-16): nearest-even.
__device__ __forceinline__ uint16_t encode_bf16(float value) {
    const uint32_t bits = __float_as_uint(value);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x0040u);
    return (uint16_t)((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}
__device__ __forceinline__ uint16_t encode_f16(float value) { return __half_as_ushort(__float2half_rn(value)); }
// Two values to a 16-bit pair (lo in the low half).  BF16: one nearest-even
// cvt for both (the same rounding as encode_bf16 for every non-NaN value,
// subnormals included); a NaN keeps encode_bf16's result (payload high bits,
// quiet bit set) instead of the cvt's canonical NaN.
__device__ __forceinline__ uint32_t encode_low_pair(float lo, float hi, uint32_t dtype) {
    if (dtype != FB_BF16) return (uint32_t)encode_f16(lo) | ((uint32_t)encode_f16(hi) << 16);
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    if (lo != lo) r = (r & 0xffff0000u) | encode_bf16(lo);
    if (hi != hi) r = (r & 0x0000ffffu) | ((uint32_t)encode_bf16(hi) << 16);
    return r;
}

// 2^x on the special-function unit (PTX ex2.approx.ftz: relative error about
// 2^-22; subnormal results flush to zero; -inf -> 0, NaN -> NaN).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// tanh form of GELU, 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), as
// x / (1 + exp(-2u)): the same value without the cancellation of 1 + tanh
// for large negative x.  exp on the special-function unit and a fast divide
// (relative error about 1e-5 before the 16-bit rounding that follows every
// use; x -> -inf gives -0, x -> +inf gives x), cheap enough for a GEMM
// epilogue to apply it at the tensor cores' pace.
__device__ __forceinline__ float gelu_tanh(float x) {
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;
    const float u = k0 * fmaf(k1 * x, x * x, x);
    return __fdividef(x, 1.0f + ex2_approx(u * -2.885390081777927f));  // -2 log2(e)
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int d = 16; d; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int d = 16; d; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    return v;
}
// Three-input maximum that ignores NaN operands (NaN only when all are NaN).
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int d = 16; d; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
    return v;
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int d = 16; d; d >>= 1) {
        const uint64_t o = __shfl_xor_sync(0xffffffffu, v, d);
        v = o > v ? o : v;
    }
    return v;
}

// Block-wide reductions over all threads; every thread gets the result.
// `scratch` holds one slot per warp and is free again on return.
template <int BLOCK>
__device__ __forceinline__ double block_sum(double v, double* scratch) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < BLOCK / 32; ++w) t += scratch[w];  // fixed order: deterministic
    __syncthreads();
    return t;
}
template <int BLOCK>
__device__ __forceinline__ float block_max(float v, float* scratch) {
    v = warp_max(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = scratch[0];
#pragma unroll
    for (int w = 1; w < BLOCK / 32; ++w) t = fmaxf(t, scratch[w]);
    __syncthreads();
    return t;
}
template <int BLOCK>
__device__ __forceinline__ uint64_t block_max_u64(uint64_t v, uint64_t* scratch) {
    v = warp_max_u64(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    uint64_t t = scratch[0];
#pragma unroll
    for (int w = 1; w < BLOCK / 32; ++w) t = scratch[w] > t ? scratch[w] : t;
    __syncthreads();
    return t;
}

}  // namespace fb
