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

// Online softmax of one query row over keys [k_begin, k_end), warp-wide:
// leaves the unnormalised accumulator in acc[0, value_depth) (f64, shared
// memory) and returns the running maximum and denominator (0 when every key
// of the range is excluded).
struct RowState {
    double maximum, denominator;
};

template <typename T>
__device__ RowState attend_range(const AttnArgs& a, const RowBases& b, uint64_t k_begin, uint64_t k_end, double* acc,
                                 double* wts, const float* qrow) {
    const int lane = threadIdx.x & 31;
    const T* K = static_cast<const T*>(a.k);
    const T* V = static_cast<const T*>(a.v);
    const double excluded = -__longlong_as_double(0x7ff0000000000000ll);
    double maximum = excluded, denominator = 0.0;
    for (uint64_t begin = k_begin; begin < k_end; begin += 32) {
        const uint64_t key = begin + lane;
        bool allowed = key < k_end;
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
            for (uint64_t d = 0; d < a.depth; ++d) dot += (double)qrow[d] * (double)Elem<T>::load(kp + d * a.k_stride_d);
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
    return {maximum, denominator};
}

template <typename T>
__device__ __forceinline__ void load_query(const AttnArgs& a, const RowBases& b, double* acc, float* qrow) {
    const int lane = threadIdx.x & 31;
    const T* Q = static_cast<const T*>(a.q);
    for (uint64_t d = lane; d < a.depth; d += 32) qrow[d] = Elem<T>::load(Q + b.q + d * a.q_stride_d);
    for (uint64_t d = lane; d < a.value_depth; d += 32) acc[d] = 0.0;
    __syncwarp();
}

template <typename T>
__global__ void attention_simt_kernel(AttnArgs a, int warps_per_block) {
    extern __shared__ double smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    double* acc = smem + (uint64_t)warp * (a.value_depth + 32 + (a.depth + 1) / 2);
    double* wts = acc + a.value_depth;
    float* qrow = reinterpret_cast<float*>(wts + 32);
    for (uint64_t row = (uint64_t)blockIdx.x * warps_per_block + warp; row < a.rows;
         row += (uint64_t)gridDim.x * warps_per_block) {
        const RowBases b = attention_bases(a, row);
        load_query<T>(a, b, acc, qrow);
        const RowState st = attend_range<T>(a, b, 0, a.keys, acc, wts, qrow);
        __syncwarp();
        for (uint64_t d = lane; d < a.value_depth; d += 32)
            a.out[b.o + d * a.o_stride_d] = st.denominator == 0.0 ? 0.0f : (float)(acc[d] / st.denominator);
        __syncwarp();
    }
}

// Split-key form for few query rows over many keys (decode): warp w takes
// (row, part) = (w / parts, w % parts), keys [part * part_keys, +part_keys),
// and leaves {maximum, denominator, acc[value_depth]} (f64) in its workspace
// record; attention_merge_kernel then combines a row's parts.
template <typename T>
__global__ void attention_part_kernel(AttnArgs a, int warps_per_block, uint32_t parts, uint64_t part_keys, double* ws) {
    extern __shared__ double smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    double* acc = smem + (uint64_t)warp * (a.value_depth + 32 + (a.depth + 1) / 2);
    double* wts = acc + a.value_depth;
    float* qrow = reinterpret_cast<float*>(wts + 32);
    const uint64_t total = a.rows * parts;
    for (uint64_t w = (uint64_t)blockIdx.x * warps_per_block + warp; w < total; w += (uint64_t)gridDim.x * warps_per_block) {
        const uint64_t row = w / parts, part = w % parts;
        const RowBases b = attention_bases(a, row);
        load_query<T>(a, b, acc, qrow);
        const uint64_t k0 = part * part_keys, k1 = k0 + part_keys < a.keys ? k0 + part_keys : a.keys;
        const RowState st = attend_range<T>(a, b, k0, k1, acc, wts, qrow);
        __syncwarp();
        double* rec = ws + w * (a.value_depth + 2);
        if (lane == 0) {
            rec[0] = st.maximum;
            rec[1] = st.denominator;
        }
        for (uint64_t d = lane; d < a.value_depth; d += 32) rec[2 + d] = acc[d];
        __syncwarp();
    }
}

// One warp per row: O = sum_p acc_p e^(m_p - M) / sum_p l_p e^(m_p - M) over
// the parts with a nonzero denominator (M their largest maximum); rows with
// no visible key are 0, as in the unsplit kernel.
__global__ void attention_merge_kernel(AttnArgs a, uint32_t parts, const double* ws) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    const uint64_t stride = a.value_depth + 2;
    for (uint64_t row = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < a.rows; row += warps) {
        const double* recs = ws + row * parts * stride;
        double M = -__longlong_as_double(0x7ff0000000000000ll);
        for (uint32_t p = 0; p < parts; ++p)
            if (recs[p * stride + 1] != 0.0 && recs[p * stride] > M) M = recs[p * stride];
        double L = 0.0;
        for (uint32_t p = 0; p < parts; ++p) {
            const double l = recs[p * stride + 1];
            if (l != 0.0) L += l * exp(recs[p * stride] - M);
        }
        const RowBases b = attention_bases(a, row);
        for (uint64_t d = lane; d < a.value_depth; d += 32) {
            double o = 0.0;
            for (uint32_t p = 0; p < parts; ++p) {
                const double l = recs[p * stride + 1];
                if (l != 0.0) o += recs[p * stride + 2 + d] * exp(recs[p * stride] - M);
            }
            a.out[b.o + d * a.o_stride_d] = L == 0.0 ? 0.0f : (float)(o / L);
        }
    }
}

}  // namespace

int launch_attention_decode(const AttnArgs& a, void* stream) {
    // Few query rows per head over many keys: parts of about 256 keys (at
    // most 64 per row, at least 2), workspace at most 64 MB.
    const uint64_t lq = a.row_rank ? a.row_dims[a.row_rank - 1] : 1;
    if (a.rows == 0 || lq > 64 || a.keys < 512) return FB_ERR_UNSUPPORTED;
    const uint64_t rec = (a.value_depth + 2) * sizeof(double);
    uint64_t parts = std::min<uint64_t>(64, (a.keys + 255) / 256);
    while (parts >= 2 && a.rows * parts * rec > (64ull << 20)) parts /= 2;
    if (parts < 2) return FB_ERR_UNSUPPORTED;
    const uint64_t part_keys = (a.keys + parts - 1) / parts;
    parts = (a.keys + part_keys - 1) / part_keys;
    const uint64_t per_warp = (a.value_depth + 32 + (a.depth + 1) / 2) * sizeof(double);
    const uint64_t limit = 200 * 1024;
    if (per_warp > limit) return FB_ERR_UNSUPPORTED;
    double* ws = static_cast<double*>(scratch(stream, a.rows * parts * rec, SCRATCH_ATTN_SPLIT));
    if (!ws) return FB_ERR_DRIVER;
    const int warps = (int)std::min<uint64_t>(4, limit / per_warp);
    const uint64_t smem = per_warp * warps;
    const uint64_t cap = (uint64_t)sm_count() * 16;
    const uint64_t blocks = std::min<uint64_t>((a.rows * parts + warps - 1) / warps, cap);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    switch (a.dtype) {
        case FB_F32:
            e = cudaFuncSetAttribute(attention_part_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            attention_part_kernel<float><<<(unsigned)blocks, warps * 32, smem, s>>>(a, warps, (uint32_t)parts, part_keys, ws);
            break;
        case FB_BF16:
            e = cudaFuncSetAttribute(attention_part_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem);
            attention_part_kernel<__nv_bfloat16><<<(unsigned)blocks, warps * 32, smem, s>>>(a, warps, (uint32_t)parts,
                                                                                         part_keys, ws);
            break;
        case FB_F16:
            e = cudaFuncSetAttribute(attention_part_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            attention_part_kernel<__half><<<(unsigned)blocks, warps * 32, smem, s>>>(a, warps, (uint32_t)parts, part_keys, ws);
            break;
        default: return FB_ERR_DTYPE;
    }
    count_launch("attention_part_kernel");
    if (e != cudaSuccess) return FB_ERR_DRIVER;
    if (cudaGetLastError() != cudaSuccess) return launch_status("kernel launch");
    const unsigned mblocks = (unsigned)std::min<uint64_t>((a.rows + 3) / 4, (uint64_t)sm_count() * 16);
    attention_merge_kernel<<<mblocks, 128, 0, s>>>(a, (uint32_t)parts, ws);
    count_launch("attention_merge_kernel");
    return launch_status("kernel launch");
}

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
    count_launch("attention_simt_kernel");
    if (e != cudaSuccess) return FB_ERR_DRIVER;
    return launch_status("kernel launch");
}

}  // namespace fb
