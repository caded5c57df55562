// Elementwise glue between the hot-path operators, for composite workloads
// (an encoder forward that chains convolution, layer norm and attention needs
// residual additions and an activation between them).
//
//   add          out = a + b in f32, operands with arbitrary strides (stride 0
//                broadcasts), as the reference's `binary` kernel with its add
//                op (compute-cuda/src/kernels.cu:29-58).
//   gelu_to_low  the tanh form of GELU, 0.5 x (1 + tanh(sqrt(2/pi) (x +
//                0.044715 x^3))), as the reference's host activation
//                (tensor-core/src/host_tensor/activation.rs:9-20), evaluated in
//                f32 (in the equivalent form x / (1 + exp(-2u)), which does not
//                cancel for negative x) and rounded once to f16/bf16 (round to nearest even, as
//                encode_low in compute-cuda/src/low_precision.cu:6-16), so the
//                activation feeds the next tensor-core contraction directly.
// Both are memory-bound; the destination is contiguous and written once.
#include <cuda_runtime.h>

#include "device_common.cuh"
#include "kernels.h"

namespace fb {
namespace {

constexpr int BLOCK = 256;

__global__ void add_kernel(const float* a, uint64_t a_off, Nest an, const float* b, uint64_t b_off, Nest bn, float* out,
                           uint64_t out_off, Nest on, uint64_t count) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x)
        out[out_off + nest_offset(on, i)] = __fadd_rn(a[a_off + nest_offset(an, i)], b[b_off + nest_offset(bn, i)]);
}

// Every view has the output's dims (broadcast axes with stride 0) and a
// contiguous innermost axis whose length is a multiple of four, each run
// 16-byte aligned: one decomposition of the index per four elements serves
// all three views (in 32-bit arithmetic when the element count allows).
template <typename I>
__global__ void add_vec4_kernel(const float* a, Nest an, const float* b, Nest bn, float* out, Nest on, I count4) {
    for (I t = (I)blockIdx.x * blockDim.x + threadIdx.x; t < count4; t += (I)gridDim.x * blockDim.x) {
        I lin = t * 4;
        uint64_t oa = 0, ob = 0, oo = 0;
#pragma unroll
        for (int d = FB_MAX_RANK - 1; d >= 0; --d) {
            if (d < (int)on.rank) {
                const I dim = (I)on.dims[d];
                const uint64_t c = lin % dim;
                lin /= dim;
                oa += c * an.strides[d];
                ob += c * bn.strides[d];
                oo += c * on.strides[d];
            }
        }
        const float4 x = *reinterpret_cast<const float4*>(a + oa), y = *reinterpret_cast<const float4*>(b + ob);
        *reinterpret_cast<float4*>(out + oo) =
            make_float4(__fadd_rn(x.x, y.x), __fadd_rn(x.y, y.y), __fadd_rn(x.z, y.z), __fadd_rn(x.w, y.w));
    }
}

// Both operands dense and the same shape: four elements per thread.
__global__ void add_dense_kernel(const float4* a, const float4* b, float4* out, uint64_t count4) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count4; i += (uint64_t)gridDim.x * blockDim.x) {
        const float4 x = a[i], y = b[i];
        out[i] = make_float4(__fadd_rn(x.x, y.x), __fadd_rn(x.y, y.y), __fadd_rn(x.z, y.z), __fadd_rn(x.w, y.w));
    }
}

// 0.5 x (1 + tanh(u)) evaluated as x / (1 + exp(-2u)), the same function:
// the sum 1 + tanh(u) cancels catastrophically in f32 for u below about -4,
// the quotient keeps full relative precision (and is exactly -0 once exp
// overflows, where the f64 form also rounds to zero).
__global__ void gelu_to_low_kernel(const float* in, uint64_t in_off, Nest n, uint16_t* out, uint32_t dtype,
                                   uint64_t count) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x) {
        const float g = gelu_tanh(in[in_off + nest_offset(n, i)]);
        out[i] = dtype == FB_BF16 ? encode_bf16(g) : encode_f16(g);
    }
}

__global__ void gelu_to_low_vec8_kernel(const float* in, uint64_t in_off, Nest n, uint16_t* out, uint32_t dtype,
                                        uint64_t runs) {
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < runs; t += (uint64_t)gridDim.x * blockDim.x) {
        const float4* src = reinterpret_cast<const float4*>(in + in_off + nest_offset(n, t * 8));
        const float4 a = src[0], b = src[1];
        reinterpret_cast<uint4*>(out)[t] =
            make_uint4(encode_low_pair(gelu_tanh(a.x), gelu_tanh(a.y), dtype), encode_low_pair(gelu_tanh(a.z), gelu_tanh(a.w), dtype),
                       encode_low_pair(gelu_tanh(b.x), gelu_tanh(b.y), dtype), encode_low_pair(gelu_tanh(b.z), gelu_tanh(b.w), dtype));
    }
}

unsigned grid_of(uint64_t work) {
    const uint64_t cap = (uint64_t)sm_count() * 16;
    const uint64_t blocks = (work + BLOCK - 1) / BLOCK;
    return (unsigned)(blocks == 0 ? 1 : (blocks < cap ? blocks : cap));
}

}  // namespace

bool add_vec4_ok(const float* a, const Nest& an, const float* b, const Nest& bn, const float* out, const Nest& on) {
    const uint32_t r = on.rank;
    if (r == 0 || an.rank != r || bn.rank != r || on.dims[r - 1] % 4 != 0) return false;
    for (const Nest* n : {&an, &bn, &on}) {
        if (n->strides[r - 1] != 1) return false;
        for (uint32_t d = 0; d < r; ++d) {
            if (n->dims[d] != on.dims[d]) return false;
            if (d + 1 < r && n->strides[d] % 4 != 0) return false;
        }
    }
    auto al = [](const float* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
    return al(a) && al(b) && al(out);
}

int launch_add(const float* a, uint64_t a_off, const Nest& an, const float* b, uint64_t b_off, const Nest& bn, float* out,
               uint64_t out_off, const Nest& on, uint64_t count, bool dense, void* stream) {
    if (count == 0) return FB_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const char* name = "add_kernel";
    if (dense) {
        name = "add_dense_kernel";
        add_dense_kernel<<<grid_of(count / 4), BLOCK, 0, st>>>(reinterpret_cast<const float4*>(a + a_off),
                                                              reinterpret_cast<const float4*>(b + b_off),
                                                              reinterpret_cast<float4*>(out + out_off), count / 4);
    } else if (add_vec4_ok(a + a_off, an, b + b_off, bn, out + out_off, on)) {
        name = "add_vec4_kernel";
        if (count < (1ull << 32))
            add_vec4_kernel<uint32_t><<<grid_of(count / 4), BLOCK, 0, st>>>(a + a_off, an, b + b_off, bn, out + out_off, on,
                                                                           (uint32_t)(count / 4));
        else
            add_vec4_kernel<uint64_t><<<grid_of(count / 4), BLOCK, 0, st>>>(a + a_off, an, b + b_off, bn, out + out_off, on,
                                                                           count / 4);
    } else {
        add_kernel<<<grid_of(count), BLOCK, 0, st>>>(a, a_off, an, b, b_off, bn, out, out_off, on, count);
    }
    count_launch(name);
    return launch_status("add");
}

int launch_gelu_to_low(const float* in, uint64_t in_off, const Nest& n, uint16_t* out, uint32_t dtype, uint64_t count,
                       void* stream) {
    if (count == 0) return FB_OK;
    if (vec8_ok(n, in, in_off, out)) {
        const uint64_t runs = count / 8;
        gelu_to_low_vec8_kernel<<<grid_of(runs), BLOCK, 0, static_cast<cudaStream_t>(stream)>>>(in, in_off, n, out, dtype,
                                                                                                 runs);
    } else {
        gelu_to_low_kernel<<<grid_of(count), BLOCK, 0, static_cast<cudaStream_t>(stream)>>>(in, in_off, n, out, dtype,
                                                                                            count);
    }
    count_launch(vec8_ok(n, in, in_off, out) ? "gelu_to_low_vec8_kernel" : "gelu_to_low_kernel");
    return launch_status("gelu");
}

}  // namespace fb
