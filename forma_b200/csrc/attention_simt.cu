// General scaled dot-product attention on CUDA cores.
//
// Covers every geometry the trait allows (masks, grouped heads, broadcast
// batches, strided views, signed causal offsets, any depth).  One warp owns a
// query row; keys are visited in tiles of 32 with one key per lane.  Scores,
// the online-softmax state and the PV accumulator are f64, as in the
// reference (compute-cuda/src/attention.cu:31-123), but the accumulator lives
// in shared memory instead of an output-sized global f64 buffer that the
// reference re-reads and re-writes every tile.
#include <cuda_runtime.h>

#include "device_common.cuh"
#include "kernels.h"

namespace fb {
namespace {

struct RowBases {
    uint64_t q, k, v, m, o, query_index;
};

__device__ __forceinline__ RowBases attention_bases(const AttnArgs& a, uint64_t row) {
    RowBases b{a.q_offset, a.k_offset, a.v_offset, a.m_offset, a.o_offset, 0};
    uint64_t rem = row;
#pragma unroll
    for (int d = FB_MAX_RANK - 1; d >= 0; --d) {
        if (d < (int)a.row_rank) {
            const uint64_t dim = a.row_dims[d];
            const uint64_t c = rem % dim;
            rem /= dim;
            if (d == (int)a.row_rank - 1) b.query_index = c;
            const uint64_t kvc = d == (int)a.row_rank - 2 ? c / a.group_size : c;
            b.q += c * a.q_row_strides[d];
            b.k += kvc * a.k_row_strides[d];
            b.v += kvc * a.v_row_strides[d];
            b.m += c * a.m_row_strides[d];
            b.o += c * a.o_row_strides[d];
        }
    }
    return b;
}

template <typename T>
__global__ void attention_simt_kernel(AttnArgs a, int warps_per_block) {
    extern __shared__ double smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    double* acc = smem + (uint64_t)warp * (a.value_depth + 32 + (a.depth + 1) / 2);
    double* wts = acc + a.value_depth;
    float* qrow = reinterpret_cast<float*>(wts + 32);
    const T* Q = static_cast<const T*>(a.q);
    const T* K = static_cast<const T*>(a.k);
    const T* V = static_cast<const T*>(a.v);
    const double excluded = -__longlong_as_double(0x7ff0000000000000ll);
    for (uint64_t row = (uint64_t)blockIdx.x * warps_per_block + warp; row < a.rows;
         row += (uint64_t)gridDim.x * warps_per_block) {
        const RowBases b = attention_bases(a, row);
        for (uint64_t d = lane; d < a.depth; d += 32) qrow[d] = Elem<T>::load(Q + b.q + d * a.q_stride_d);
        for (uint64_t d = lane; d < a.value_depth; d += 32) acc[d] = 0.0;
        __syncwarp();
        double maximum = excluded, denominator = 0.0;
        for (uint64_t begin = 0; begin < a.keys; begin += 32) {
            const uint64_t key = begin + lane;
            bool allowed = key < a.keys;
            if (allowed && a.causal) allowed = (long long)key - (long long)b.query_index <= (long long)a.causal_offset;
            double bias = 0.0;
            if (allowed && a.mask_kind == FB_MASK_KEEP)
                allowed = static_cast<const uint32_t*>(a.mask)[b.m + key * a.m_stride_key] != 0u;
            if (allowed && a.mask_kind == FB_MASK_ADDITIVE) {
                bias = (double)static_cast<const float*>(a.mask)[b.m + key * a.m_stride_key];
                allowed = bias != excluded;
            }
            double score = excluded;
            if (allowed) {
                double dot = 0.0;
                const T* kp = K + b.k + key * a.k_stride_key;
                for (uint64_t d = 0; d < a.depth; ++d)
                    dot += (double)qrow[d] * (double)Elem<T>::load(kp + d * a.k_stride_d);
                score = dot * (double)a.scale + bias;
            }
            double tile_max = score;
#pragma unroll
            for (int s = 16; s; s >>= 1) {
                const double o = __shfl_xor_sync(0xffffffffu, tile_max, s);
                tile_max = o > tile_max ? o : tile_max;
            }
            if (tile_max == excluded) continue;  // nothing visible in this tile
            const double next = maximum > tile_max ? maximum : tile_max;
            // An all-excluded prefix must not evaluate -inf - (-inf).
            const double alpha = denominator == 0.0 ? 0.0 : exp(maximum - next);
            maximum = next;
            const double w = score == excluded ? 0.0 : exp(score - maximum);
            denominator = denominator * alpha + warp_sum(w);
            wts[lane] = w;
            __syncwarp();
            for (uint64_t d = lane; d < a.value_depth; d += 32) {
                double r = acc[d] * alpha;
                for (int j = 0; j < 32; ++j) {
                    const double wj = wts[j];
                    // Zero weights cover excluded keys, tails and underflow:
                    // V is not read for them.
                    if (wj != 0.0) r += wj * (double)Elem<T>::load(V + b.v + (begin + j) * a.v_stride_key + d * a.v_stride_d);
                }
                acc[d] = r;
            }
            __syncwarp();
        }
        __syncwarp();
        for (uint64_t d = lane; d < a.value_depth; d += 32)
            a.out[b.o + d * a.o_stride_d] = denominator == 0.0 ? 0.0f : (float)(acc[d] / denominator);
        __syncwarp();
    }
}

}  // namespace

int launch_attention_simt(const AttnArgs& a, void* stream) {
    if (a.rows == 0) return FB_OK;
    const uint64_t per_warp = (a.value_depth + 32 + (a.depth + 1) / 2) * sizeof(double);
    const uint64_t limit = 200 * 1024;
    if (per_warp > limit) return FB_ERR_UNSUPPORTED;
    int warps = (int)std::min<uint64_t>(4, limit / per_warp);
    const uint64_t smem = per_warp * warps;
    const uint64_t cap = (uint64_t)sm_count() * 16;
    const uint64_t blocks = std::min<uint64_t>((a.rows + warps - 1) / warps, cap);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    switch (a.dtype) {
        case FB_F32:
            e = cudaFuncSetAttribute(attention_simt_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            attention_simt_kernel<float><<<(unsigned)blocks, warps * 32, smem, s>>>(a, warps);
            break;
        case FB_BF16:
            e = cudaFuncSetAttribute(attention_simt_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem);
            attention_simt_kernel<__nv_bfloat16><<<(unsigned)blocks, warps * 32, smem, s>>>(a, warps);
            break;
        case FB_F16:
            e = cudaFuncSetAttribute(attention_simt_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            attention_simt_kernel<__half><<<(unsigned)blocks, warps * 32, smem, s>>>(a, warps);
            break;
        default: return FB_ERR_DTYPE;
    }
    count_launch();
    if (e != cudaSuccess) return FB_ERR_DRIVER;
    return launch_status("kernel launch");
}

}  // namespace fb
