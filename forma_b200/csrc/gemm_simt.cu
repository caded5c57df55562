// Low-precision GEMM for every layout the tensor-core path does not take
// (any strides, any M / N / K, broadcast batches): 16 x 16 output tiles, 16 x
// 16 operand tiles staged in shared memory, f32 fused multiply-add over K in
// order, f32 output or one nearest-even rounding to 16 bits.  The reference
// computes these products with cuBLAS (compute-cuda/src/matmul.rs:144-162);
// parity is the bf16 tensor-core tolerance, not bit equality.
#include <cuda_runtime.h>

#include "device_common.cuh"
#include "kernels.h"

namespace fb {
namespace {

constexpr int T16 = 16;

__device__ __forceinline__ float load_low(const uint16_t* p, uint64_t i, uint32_t dtype) {
    return dtype == FB_BF16 ? bf16_bits_to_float(p[i]) : f16_bits_to_float(p[i]);
}

__global__ void __launch_bounds__(T16 * T16) gemm_simt_kernel(GemmArgs g, uint64_t n_tiles, uint64_t tiles) {
    __shared__ float As[T16][T16 + 1], Bs[T16][T16 + 1];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const uint16_t* A0 = static_cast<const uint16_t*>(g.a);
    const uint16_t* B0 = static_cast<const uint16_t*>(g.b);
    for (uint64_t bz = blockIdx.y; bz < g.batch; bz += gridDim.y) {
        const uint64_t ao = g.a_off + nest_offset(g.a_batch, bz);
        const uint64_t bo = g.b_off + nest_offset(g.b_batch, bz);
        const uint64_t oo = g.o_off + nest_offset(g.o_batch, bz);
        for (uint64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
            const uint64_t m0 = (t / n_tiles) * T16, n0 = (t % n_tiles) * T16;
            float acc = 0.0f;
            for (uint64_t k0 = 0; k0 < g.K; k0 += T16) {
                const uint64_t am = m0 + ty, ak = k0 + tx;
                As[ty][tx] = (am < g.M && ak < g.K) ? load_low(A0, ao + am * g.a_sm + ak * g.a_sk, g.dtype) : 0.0f;
                const uint64_t bk = k0 + ty, bn = n0 + tx;
                Bs[ty][tx] = (bk < g.K && bn < g.N) ? load_low(B0, bo + bk * g.b_sk + bn * g.b_sn, g.dtype) : 0.0f;
                __syncthreads();
#pragma unroll
                for (int kk = 0; kk < T16; ++kk) acc = fmaf(As[ty][kk], Bs[kk][tx], acc);
                __syncthreads();
            }
            const uint64_t m = m0 + ty, n = n0 + tx;
            if (m < g.M && n < g.N) {
                const uint64_t i = oo + m * g.o_sm + n * g.o_sn;
                if (g.out_low == FB_BF16)
                    static_cast<uint16_t*>(g.out)[i] = encode_bf16(acc);
                else if (g.out_low)
                    static_cast<uint16_t*>(g.out)[i] = encode_f16(acc);
                else
                    static_cast<float*>(g.out)[i] = acc;
            }
        }
    }
}

}  // namespace

int launch_gemm_simt(const GemmArgs& g, void* stream) {
    if (g.M == 0 || g.N == 0 || g.batch == 0) return FB_OK;
    const uint64_t n_tiles = (g.N + T16 - 1) / T16, m_tiles = (g.M + T16 - 1) / T16;
    const uint64_t tiles = m_tiles * n_tiles;
    const uint64_t cap = (uint64_t)sm_count() * 8;
    const unsigned gx = (unsigned)(tiles < cap ? tiles : cap);
    const unsigned gy = (unsigned)(g.batch < 65535 ? g.batch : 65535);
    gemm_simt_kernel<<<dim3(gx, gy), dim3(T16, T16), 0, static_cast<cudaStream_t>(stream)>>>(g, n_tiles, tiles);
    count_launch("gemm_simt_kernel");
    return launch_status("gemm");
}

}  // namespace fb
