// Row reductions, argmax, statistics and the global-sum partial.
//
// Every operation is a pass over "rows" (the kept coordinates) of "columns"
// (the contracted coordinates).  One 256-thread block owns a row at a time
// and the grid strides over rows, sized to a multiple of the SM count.  For
// the dominant case - contiguous rows of an f32 matrix - columns are read
// with 128-bit loads, several in flight per thread, and statistics keep the
// whole row in registers so softmax and layer norm read HBM once and write
// once (the reference reads the input three times and keeps f64 partials in
// global memory: compute-cuda/src/statistics.cu:139-208).  Other layouts use
// the same kernels with per-element nest addressing.
//
// Arithmetic: sums, products and moments accumulate in f64; min, max and
// argmax compare total-order keys so they are exact and order-independent.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "async.cuh"
#include "device_common.cuh"
#include "kernels.h"

namespace fb {
namespace {

__device__ uint32_t g_reduce_status;  // DeviceStatus of this translation unit

constexpr int BLOCK = 256;

template <typename T>
__device__ __forceinline__ const T* row_base(const Rows& in, uint64_t row) {
    const T* p = reinterpret_cast<const T*>(in.data) + in.offset;
    return p + (in.contiguous_rows ? row * in.row_stride : nest_offset(in.outer, row));
}

template <typename T>
__device__ __forceinline__ float row_elem(const Rows& in, const T* base, uint64_t c) {
    return Elem<T>::load(base + (in.contiguous_rows ? c : nest_offset(in.inner, c)));
}

__device__ __forceinline__ uint64_t out_index(const RowOut& o, uint64_t row) {
    return o.offset + (o.contiguous ? row : nest_offset(o.nest, row));
}

// Four consecutive results of a contiguous row, as f32 or rounded 16-bit.
__device__ __forceinline__ void store_row4(const ElemOut& eo, uint64_t row, uint64_t col, float4 v) {
    const uint64_t i = eo.offset + row * eo.row_stride + col;
    if (eo.dtype == FB_F32) {
        *reinterpret_cast<float4*>(eo.data + i) = v;
    } else {
        *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(eo.data) + i) =
            make_uint2(encode_low_pair(v.x, v.y, eo.dtype), encode_low_pair(v.z, v.w, eo.dtype));
    }
}

__device__ __forceinline__ float* elem_out(const ElemOut& o, uint64_t row, uint64_t c) {
    if (o.contiguous_rows) return o.data + o.offset + row * o.row_stride + c;
    return o.data + o.offset + nest_offset(o.outer, row) + nest_offset(o.inner, c);
}

// Per-thread state of one reduction.
struct Acc {
    double sum;
    uint64_t best;  // (key << 32) | (0xffffffff - column): max = largest key, lowest column
};

__device__ __forceinline__ void acc_add(Acc& a, uint32_t op, float x, uint64_t c) {
    if (op == ROW_SUM || op == ROW_MEAN) {
        a.sum += (double)x;
    } else if (op == ROW_PRODUCT) {
        a.sum *= (double)x;
    } else {
        uint32_t k = order_key(x);
        if (op == ROW_MIN) k = ~k;
        const uint64_t packed = ((uint64_t)k << 32) | (uint64_t)(0xffffffffu - (uint32_t)c);
        a.best = packed > a.best ? packed : a.best;
    }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(BLOCK) reduce_rows_kernel(Rows in, RowOut out, uint32_t op) {
    __shared__ double s_sum[BLOCK / 32];
    __shared__ uint64_t s_best[BLOCK / 32];
    __shared__ double s_prod[BLOCK];
    for (uint64_t row = blockIdx.x; row < in.rows; row += gridDim.x) {
        const T* base = row_base<T>(in, row);
        Acc a{op == ROW_PRODUCT ? 1.0 : 0.0, 0};
        uint64_t c0 = 0;
        if (VEC == 4) {
            // 128-bit (f32) or 64-bit (low) loads, four vectors in flight.
            const uint64_t nvec = in.cols / 4;
            uint64_t v = threadIdx.x;
            for (; v + 3 * BLOCK < nvec; v += 4 * BLOCK) {
                float4 x[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) x[u] = Elem<T>::load4(base + (v + u * BLOCK) * 4);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint64_t c = (v + u * BLOCK) * 4;
                    acc_add(a, op, x[u].x, c);
                    acc_add(a, op, x[u].y, c + 1);
                    acc_add(a, op, x[u].z, c + 2);
                    acc_add(a, op, x[u].w, c + 3);
                }
            }
            for (; v < nvec; v += BLOCK) {
                const float4 x = Elem<T>::load4(base + v * 4);
                acc_add(a, op, x.x, v * 4);
                acc_add(a, op, x.y, v * 4 + 1);
                acc_add(a, op, x.z, v * 4 + 2);
                acc_add(a, op, x.w, v * 4 + 3);
            }
            c0 = nvec * 4;
        }
        for (uint64_t c = c0 + threadIdx.x; c < in.cols; c += BLOCK) acc_add(a, op, row_elem<T>(in, base, c), c);

        if (op == ROW_PRODUCT) {
            // Products have no warp shuffle identity worth special-casing: a
            // shared-memory tree in fixed order.
            s_prod[threadIdx.x] = a.sum;
            __syncthreads();
            for (int s = BLOCK / 2; s; s >>= 1) {
                if (threadIdx.x < s) s_prod[threadIdx.x] *= s_prod[threadIdx.x + s];
                __syncthreads();
            }
            if (threadIdx.x == 0) static_cast<float*>(out.data)[out_index(out, row)] = (float)s_prod[0];
            __syncthreads();
        } else if (op == ROW_SUM || op == ROW_MEAN) {
            const double t = block_sum<BLOCK>(a.sum, s_sum);
            if (threadIdx.x == 0)
                static_cast<float*>(out.data)[out_index(out, row)] =
                    op == ROW_MEAN ? (float)(t / (double)in.cols) : (float)t;
        } else {
            const uint64_t b = block_max_u64<BLOCK>(a.best, s_best);
            if (threadIdx.x == 0) {
                uint32_t k = (uint32_t)(b >> 32);
                if (op == ROW_ARGMAX)
                    static_cast<uint32_t*>(out.data)[out_index(out, row)] = 0xffffffffu - (uint32_t)(b & 0xffffffffu);
                else
                    static_cast<float*>(out.data)[out_index(out, row)] = key_value(op == ROW_MIN ? ~k : k);
            }
        }
    }
}

// u32 reductions (TensorReduceBackend::reduce_u32): wrapping sum/product.
__global__ void __launch_bounds__(BLOCK) reduce_rows_u32_kernel(Rows in, RowOut out, uint32_t op) {
    __shared__ uint32_t s[BLOCK];
    for (uint64_t row = blockIdx.x; row < in.rows; row += gridDim.x) {
        const uint32_t* base = reinterpret_cast<const uint32_t*>(in.data) + in.offset +
                               (in.contiguous_rows ? row * in.row_stride : nest_offset(in.outer, row));
        uint32_t a = op == ROW_PRODUCT ? 1u : (op == ROW_MIN ? 0xffffffffu : 0u);
        for (uint64_t c = threadIdx.x; c < in.cols; c += BLOCK) {
            const uint32_t x = __ldg(base + (in.contiguous_rows ? c : nest_offset(in.inner, c)));
            a = op == ROW_SUM ? a + x : op == ROW_PRODUCT ? a * x : op == ROW_MIN ? min(a, x) : max(a, x);
        }
        s[threadIdx.x] = a;
        __syncthreads();
        for (int w = BLOCK / 2; w; w >>= 1) {
            if (threadIdx.x < w) {
                const uint32_t x = s[threadIdx.x], y = s[threadIdx.x + w];
                s[threadIdx.x] = op == ROW_SUM ? x + y : op == ROW_PRODUCT ? x * y : op == ROW_MIN ? min(x, y) : max(x, y);
            }
            __syncthreads();
        }
        if (threadIdx.x == 0) static_cast<uint32_t*>(out.data)[out_index(out, row)] = s[0];
        __syncthreads();
    }
}

// Statistics over rows (TensorStatsBackend).  NV > 0 keeps the row in
// registers: NV float4 per thread, so rows of up to 4*NV*BLOCK columns are read
// from HBM exactly once and written once with 128-bit stores (input and output
// rows contiguous and 16-byte aligned).  NV == 0 re-reads the row from memory
// for each pass and addresses any strided layout.
//   softmax      exp(x - max) / sum exp(x - max)
//   log-softmax  (x - max) - log(sum)
//   logsumexp    max + log(sum)
//   moments      mean = sum x / n, var = sum (x - mean)^2 / n (f64, centred)
//   layer norm   (x - mean) / sqrt(var + eps)
// exp is CUDA's expf on the f32 shift, as in compute-cuda/src/statistics.cu:151;
// every sum is f64.
template <typename T, int NV>
__global__ void __launch_bounds__(BLOCK) stats_rows_kernel(Rows in, ElemOut out, RowOut oa, RowOut ob, uint32_t op,
                                                           float eps) {
    __shared__ double s_sum[BLOCK / 32];
    __shared__ float s_max[BLOCK / 32];
    const bool exp_family = op == STATS_SOFTMAX || op == STATS_LOG_SOFTMAX || op == STATS_LOGSUMEXP;
    for (uint64_t row = blockIdx.x; row < in.rows; row += gridDim.x) {
        const T* base = row_base<T>(in, row);
        const uint64_t n = in.cols;
        float4 cache[NV > 0 ? NV : 1];
        if constexpr (NV > 0) {
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                const uint64_t v = threadIdx.x + (uint64_t)j * BLOCK;
                cache[j] = v * 4 < n ? Elem<T>::load4(base + v * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        // Applies f to every element this thread owns.
        auto each = [&](auto&& f) {
            if constexpr (NV > 0) {
#pragma unroll
                for (int j = 0; j < NV; ++j) {
                    if ((threadIdx.x + (uint64_t)j * BLOCK) * 4 < n) {
                        f(cache[j].x);
                        f(cache[j].y);
                        f(cache[j].z);
                        f(cache[j].w);
                    }
                }
            } else {
                for (uint64_t c = threadIdx.x; c < n; c += BLOCK) f(row_elem<T>(in, base, c));
            }
        };
        // Writes g(x) for every element this thread owns.
        auto emit = [&](auto&& g) {
            if constexpr (NV > 0) {
                float* orow = out.data + out.offset + row * out.row_stride;
#pragma unroll
                for (int j = 0; j < NV; ++j) {
                    const uint64_t c = (threadIdx.x + (uint64_t)j * BLOCK) * 4;
                    if (c < n)
                        *reinterpret_cast<float4*>(orow + c) =
                            make_float4(g(cache[j].x), g(cache[j].y), g(cache[j].z), g(cache[j].w));
                }
            } else {
                for (uint64_t c = threadIdx.x; c < n; c += BLOCK) *elem_out(out, row, c) = g(row_elem<T>(in, base, c));
            }
        };
        if (exp_family) {
            float m = -__int_as_float(0x7f800000);
            each([&](float x) { m = fmaxf(m, x); });
            m = block_max<BLOCK>(m, s_max);
            double s = 0.0;
            each([&](float x) { s += (double)expf(x - m); });
            s = block_sum<BLOCK>(s, s_sum);
            if (op == STATS_SOFTMAX) {
                const double inv = 1.0 / s;
                emit([&](float x) { return (float)((double)expf(x - m) * inv); });
            } else if (op == STATS_LOG_SOFTMAX) {
                // (x - max) - log(sum): subtracting the shift first keeps the
                // result exact for huge offsets (max + log(sum) would round).
                const double ls = log(s);
                emit([&](float x) { return (float)(((double)x - (double)m) - ls); });
            } else if (threadIdx.x == 0) {
                static_cast<float*>(oa.data)[out_index(oa, row)] = (float)((double)m + log(s));
            }
        } else {
            double s = 0.0;
            each([&](float x) { s += (double)x; });
            const double mean = block_sum<BLOCK>(s, s_sum) / (double)n;
            double q = 0.0;
            each([&](float x) {
                const double d = (double)x - mean;
                q += d * d;
            });
            const double var = block_sum<BLOCK>(q, s_sum) / (double)n;
            if (op == STATS_LAYER_NORM) {
                const double inv = 1.0 / sqrt(var + (double)eps);
                emit([&](float x) { return (float)(((double)x - mean) * inv); });
            } else if (threadIdx.x == 0) {
                static_cast<float*>(oa.data)[out_index(oa, row)] = (float)mean;
                static_cast<float*>(ob.data)[out_index(ob, row)] = (float)var;
            }
        }
    }
}

// Streamed row engine for contiguous rows (the row-reduction workload).
//
// Rows are copied HBM -> shared memory by cp.async.bulk into a ring of
// `stages` row buffers, each completing on its own mbarrier, so the next rows
// are always in flight while the current one is reduced: the block never
// waits on an HBM round trip between rows.  Each thread then takes NV float4
// of the row into registers (conflict-free 16-byte shared loads), the stage is
// released, and the operation runs on registers with block-wide f64 / key
// reductions.  Elementwise results leave with 128-bit coalesced stores.
template <typename T>
__device__ __forceinline__ float4 smem_load4(const unsigned char* row, uint64_t v) {
    if constexpr (sizeof(T) == 4) {
        return *reinterpret_cast<const float4*>(row + v * 16);
    } else {
        const uint2 u = *reinterpret_cast<const uint2*>(row + v * 8);
        if constexpr (std::is_same<T, __nv_bfloat16>::value)
            return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                               __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
        else
            return make_float4(f16_bits_to_float((uint16_t)(u.x & 0xffff)), f16_bits_to_float((uint16_t)(u.x >> 16)),
                               f16_bits_to_float((uint16_t)(u.y & 0xffff)), f16_bits_to_float((uint16_t)(u.y >> 16)));
    }
}

// Operation codes of the streamed engine: RowOp values, then StatsOp + 16.
constexpr uint32_t STREAM_STATS = 16;

// Operation families, one kernel instantiation each, so that every family
// gets the registers (and so the blocks per SM) that its own code needs.
constexpr int FAM_SUM = 0;      // sum, mean
constexpr int FAM_EXTREME = 1;  // min, max, argmax
constexpr int FAM_EXP = 2;      // softmax, log-softmax, logsumexp
constexpr int FAM_MOMENTS = 3;  // moments, layer norm

// CAP: registers capped so that six (argmax) or five (moments: six spilled
// in its row loop) 128-thread blocks fit per SM; both hold more per-row state
// and measured faster with the extra blocks, the light reductions uncapped.
template <typename T, int NV, int TB, bool CAP, int FAM>
__global__ void __launch_bounds__(TB, CAP ? (FAM == FAM_MOMENTS ? 5 : 6) : 1) rows_stream_kernel(Rows in, uint32_t op, RowOut oa, RowOut ob, ElemOut eo,
                                                            float eps, uint32_t stages, uint32_t row_bytes) {
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    unsigned char* ring = smem + 128;
    // Per-warp partials, double-buffered by row parity so that one barrier per
    // block reduction suffices (a row's partials are never overwritten before
    // every thread has passed the next row's first barrier).
    __shared__ double s_d[2][2][TB / 32];
    __shared__ float s_f[2][TB / 32];
    __shared__ float s_e[2][TB / 32];
    __shared__ uint64_t s_k[2][TB / 32];
    __shared__ int s_abort;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint64_t first = blockIdx.x, step = gridDim.x;
    const uint64_t mine = first < in.rows ? (in.rows - 1 - first) / step + 1 : 0;
    const uint64_t n = in.cols;
    const double inv_n = 1.0 / (double)n;  // one division per thread, not per row
    const T* base = reinterpret_cast<const T*>(in.data) + in.offset;
    if (tid == 0) {
        for (uint32_t s = 0; s < stages; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
        s_abort = 0;
    }
    __syncthreads();
    auto issue = [&](uint64_t i) {
        const uint32_t s = (uint32_t)(i % stages);
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&full[s], row_bytes);
        bulk_g2s(ring + (uint64_t)s * row_bytes, base + (first + i * step) * in.row_stride, row_bytes, &full[s]);
    };
    if (tid == 0)
        for (uint64_t i = 0; i < mine && i < stages; ++i) issue(i);
    uint64_t aborted_at = ~0ull;
    for (uint64_t i = 0; i < mine; ++i) {
        const uint32_t s = (uint32_t)(i % stages), par = (uint32_t)(i & 1);
        if (!mbar_wait(&full[s], (uint32_t)((i / stages) & 1))) s_abort = 1;
        float4 c[NV];
        const unsigned char* rb = ring + (uint64_t)s * row_bytes;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const uint64_t v = tid + (uint64_t)j * TB;
            c[j] = v * 4 < n ? smem_load4<T>(rb, v) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const uint64_t row = first + i * step;
        // First barrier of the row: every thread has read stage s, so the
        // producer refills it, and the first partials are visible.
        auto barrier_release = [&]() {
            __syncthreads();
            if (tid == 0 && i + stages < mine && !s_abort) issue(i + stages);
        };
        auto valid = [&](int j) { return (tid + (uint64_t)j * TB) * 4 < n; };

        if constexpr (FAM == FAM_SUM) {
            double a = 0.0;
#pragma unroll
            for (int j = 0; j < NV; ++j)
                if (valid(j)) a += ((double)c[j].x + (double)c[j].y) + ((double)c[j].z + (double)c[j].w);
            a = warp_sum(a);
            if (lane == 0) s_d[0][par][warp] = a;
            barrier_release();
            if (s_abort) {
                aborted_at = i;
                break;
            }
            if (tid == 0) {
                double t = 0.0;
#pragma unroll
                for (int w = 0; w < TB / 32; ++w) t += s_d[0][par][w];
                static_cast<float*>(oa.data)[out_index(oa, row)] = op == ROW_MEAN ? (float)(t / (double)n) : (float)t;
            }
        } else if constexpr (FAM == FAM_EXTREME) {
            // Keys in column order per thread: a strictly greater key wins,
            // so each thread keeps its lowest column among equal keys.
            const uint32_t flip = op == ROW_MIN ? 0xffffffffu : 0u;
            uint32_t bk = 0, bc = 0;
            // This thread's extreme with NaN-propagating three-input min/max
            // (half an instruction per element).  Unless it is NaN or a zero,
            // numeric order and key order agree on this thread's elements (only
            // NaNs and the two zeros differ), so its key is the thread's best
            // key, and argmax needs just the first column equal to it.
            // Threads holding a NaN or a zero extreme run the full key scan.
            const bool is_min = op == ROW_MIN;
            float m = is_min ? __int_as_float(0x7f800000) : -__int_as_float(0x7f800000);
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                if (!valid(j)) continue;
                if (is_min)
                    m = min3_nan(min3_nan(m, c[j].x, c[j].y), c[j].z, c[j].w);
                else
                    m = max3_nan(max3_nan(m, c[j].x, c[j].y), c[j].z, c[j].w);
            }
            if (m != m || m == 0.0f) {
#pragma unroll
                for (int j = 0; j < NV; ++j) {
                    if (!valid(j)) continue;
                    const uint32_t col = (uint32_t)((tid + (uint64_t)j * TB) * 4);
                    const float xs[4] = {c[j].x, c[j].y, c[j].z, c[j].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t k = order_key(xs[e]) ^ flip;
                        if (k > bk || (j == 0 && e == 0)) {
                            bk = k;
                            bc = col + e;
                        }
                    }
                }
            } else {
                bk = order_key(m) ^ flip;
                if (op == ROW_ARGMAX) {
                    // last match wins in a reverse scan = first column
#pragma unroll
                    for (int j = NV - 1; j >= 0; --j) {
                        if (!valid(j)) continue;
                        const uint32_t col = (uint32_t)((tid + (uint64_t)j * TB) * 4);
                        if (c[j].w == m) bc = col + 3;
                        if (c[j].z == m) bc = col + 2;
                        if (c[j].y == m) bc = col + 1;
                        if (c[j].x == m) bc = col;
                    }
                }
            }
            uint64_t best = ((uint64_t)bk << 32) | (uint64_t)(0xffffffffu - bc);
            if (!valid(0)) best = 0;
            best = warp_max_u64(best);
            if (lane == 0) s_k[par][warp] = best;
            barrier_release();
            if (s_abort) {
                aborted_at = i;
                break;
            }
            if (tid == 0) {
                uint64_t t = s_k[par][0];
#pragma unroll
                for (int w = 1; w < TB / 32; ++w) t = s_k[par][w] > t ? s_k[par][w] : t;
                const uint32_t k = (uint32_t)(t >> 32) ^ flip;
                if (op == ROW_ARGMAX)
                    static_cast<uint32_t*>(oa.data)[out_index(oa, row)] = 0xffffffffu - (uint32_t)(t & 0xffffffffu);
                else
                    static_cast<float*>(oa.data)[out_index(oa, row)] = key_value(k);
            }
        } else if constexpr (FAM == FAM_EXP) {
            // Row maximum (NaN operands ignored, as a NaN reaches every output
            // through the sum anyway), then exp(x - max) once per element as
            // 2^((x - max) log2 e) on the special-function unit, summed in f32
            // (all terms positive: relative error below 2^-19 for 4096
            // columns).  The reference takes expf of the f32 difference and
            // sums in f64 (statistics.cu:37-45, 89-91).
            float m = -__int_as_float(0x7f800000);
#pragma unroll
            for (int j = 0; j < NV; ++j)
                if (valid(j)) m = max3(max3(m, c[j].x, c[j].y), c[j].z, c[j].w);
            m = warp_max(m);
            if (lane == 0) s_f[par][warp] = m;
            barrier_release();
            if (s_abort) {
                aborted_at = i;
                break;
            }
            m = s_f[par][0];
#pragma unroll
            for (int w = 1; w < TB / 32; ++w) m = fmaxf(m, s_f[par][w]);
            // lane pairs: two values per add / multiply instruction
            const float2 nm2 = make_float2(-m, -m);
            const float2 l2e = make_float2(1.4426950408889634f, 1.4426950408889634f);
            float2 e2 = make_float2(0.0f, 0.0f);
            const bool keep = op == STREAM_STATS + STATS_SOFTMAX;
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                if (!valid(j)) continue;
                const float2 t01 = __fmul2_rn(__fadd2_rn(make_float2(c[j].x, c[j].y), nm2), l2e);
                const float2 t23 = __fmul2_rn(__fadd2_rn(make_float2(c[j].z, c[j].w), nm2), l2e);
                const float2 x01 = make_float2(ex2_approx(t01.x), ex2_approx(t01.y));
                const float2 x23 = make_float2(ex2_approx(t23.x), ex2_approx(t23.y));
                e2 = __fadd2_rn(e2, __fadd2_rn(x01, x23));
                if (keep) c[j] = make_float4(x01.x, x01.y, x23.x, x23.y);
            }
            float e = warp_sum_f(e2.x + e2.y);
            if (lane == 0) s_e[par][warp] = e;
            __syncthreads();
            e = 0.0f;
#pragma unroll
            for (int w = 0; w < TB / 32; ++w) e += s_e[par][w];
            if (op == STREAM_STATS + STATS_SOFTMAX) {
                const float inv = __frcp_rn(e);
                const float2 inv2 = make_float2(inv, inv);
#pragma unroll
                for (int j = 0; j < NV; ++j)
                    if (valid(j)) {
                        const float2 y01 = __fmul2_rn(make_float2(c[j].x, c[j].y), inv2);
                        const float2 y23 = __fmul2_rn(make_float2(c[j].z, c[j].w), inv2);
                        store_row4(eo, row, (tid + (uint64_t)j * TB) * 4, make_float4(y01.x, y01.y, y23.x, y23.y));
                    }
            } else if (op == STREAM_STATS + STATS_LOG_SOFTMAX) {
                // (x - max) - log(sum): both terms within an f32 ulp
                const float ls = logf(e);
                const float2 nls = make_float2(-ls, -ls);
#pragma unroll
                for (int j = 0; j < NV; ++j)
                    if (valid(j)) {
                        const float2 y01 = __fadd2_rn(__fadd2_rn(make_float2(c[j].x, c[j].y), nm2), nls);
                        const float2 y23 = __fadd2_rn(__fadd2_rn(make_float2(c[j].z, c[j].w), nm2), nls);
                        store_row4(eo, row, (tid + (uint64_t)j * TB) * 4, make_float4(y01.x, y01.y, y23.x, y23.y));
                    }
            } else if (tid == 0) {
                static_cast<float*>(oa.data)[out_index(oa, row)] = (float)((double)m + log((double)e));
            }
        } else {  // FAM_MOMENTS
            // Moments / layer norm in one pass and one block reduction.  Each
            // thread sums the deviations d = x - a from an anchor a (the mean
            // of the row's first four values, read from the staged row,
            // identical in every thread) and their squares, in f32 lane pairs
            // (two values per instruction) combined pairwise, then in f64
            // across lanes, warps and the block:
            //   D = sum d,  Q = sum d^2,  mean = a + D / n,  var = (Q - D^2 / n) / n.
            // Accepted when both error bounds leave a wide margin under the
            // 1e-5 tolerance (u = 2^-24; the f32 tree has depth L = 2 + log2(NV)
            // after the rounding of each d):
            //   mean:  (L + 1) u * sum |d| / n <= 2^-20 * max(|mean|, 1), with
            //          sum |d| <= sqrt(n Q) (Cauchy-Schwarz)
            //   var:   Q <= 4 * n * var  (cancellation factor <= 4; each f32
            //          partial of squares is within (L + 3) u, so var is
            //          within 4 (L + 3) u, <= 32u)
            // and everything is finite with a variance that cannot have
            // underflowed in f32; otherwise (NaN/inf inputs, constant rows,
            // deviations too large for the bounds) the row is redone exactly
            // in f64 with two passes, as the reference computes it
            // (statistics.cu:4-123).
            const float4 head = smem_load4<T>(rb, 0);
            const float anc = 0.25f * ((head.x + head.y) + (head.z + head.w));
            const float2 na2 = make_float2(-anc, -anc);
            float2 s2[NV], q2[NV];
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                if (!valid(j)) {
                    s2[j] = q2[j] = make_float2(0.0f, 0.0f);
                    continue;
                }
                const float2 d01 = __fadd2_rn(make_float2(c[j].x, c[j].y), na2);
                const float2 d23 = __fadd2_rn(make_float2(c[j].z, c[j].w), na2);
                s2[j] = __fadd2_rn(d01, d23);
                q2[j] = __ffma2_rn(d01, d01, __fmul2_rn(d23, d23));
            }
#pragma unroll
            for (int w = 1; w < NV; w *= 2)
#pragma unroll
                for (int j = 0; j + w < NV; j += 2 * w) {
                    s2[j] = __fadd2_rn(s2[j], s2[j + w]);
                    q2[j] = __fadd2_rn(q2[j], q2[j + w]);
                }
            double sd = (double)s2[0].x + (double)s2[0].y, qd = (double)q2[0].x + (double)q2[0].y;
            sd = warp_sum(sd);
            qd = warp_sum(qd);
            if (lane == 0) {
                s_d[0][par][warp] = sd;
                s_d[1][par][warp] = qd;
            }
            barrier_release();
            if (s_abort) {
                aborted_at = i;
                break;
            }
            double D = 0.0, Q = 0.0;
#pragma unroll
            for (int w = 0; w < TB / 32; ++w) {
                D += s_d[0][par][w];
                Q += s_d[1][par][w];
            }
            // Only multiplications, comparisons and one f32 square root per
            // row: D * (1/n) is within an f64 ulp of D / n, far below the f32
            // result, and the bound needs no more than an upper estimate.
            const double dn = (double)n;
            double mean = (double)anc + D * inv_n;
            double var = (Q - D * D * inv_n) * inv_n;
            constexpr double kL = NV >= 8 ? 6.0 : NV >= 4 ? 5.0 : NV >= 2 ? 4.0 : 3.0;  // 3 + log2(NV)
            constexpr double kLu = kL * 5.9604644775390625e-08;                           // (L + 1) * 2^-24
            const double big = 1.7976931348623157e308;
            // The f32 root (correctly rounded, of an argument rounded to f32)
            // is raised by 2^-20 to stay an upper bound; an argument past the
            // f32 range gives inf and the exact path.
            const double A = (double)sqrtf((float)(dn * Q)) * (1.0 + 9.5367431640625e-07);
            const bool fast = fabs(D) <= big && Q <= big && var > 1e-30 &&
                              kLu * A * inv_n <= 9.5367431640625e-07 * fmax(fabs(mean), 1.0) &&
                              Q <= 4.0 * dn * var;
            if (!fast) {
                // block-uniform fallback: exact f64 two-pass (the partials of
                // this parity are reused once every thread has read them)
                double e = 0.0;
#pragma unroll
                for (int j = 0; j < NV; ++j)
                    if (valid(j)) e += ((double)c[j].x + (double)c[j].y) + ((double)c[j].z + (double)c[j].w);
                e = warp_sum(e);
                __syncthreads();
                if (lane == 0) s_d[0][par][warp] = e;
                __syncthreads();
                e = 0.0;
#pragma unroll
                for (int w = 0; w < TB / 32; ++w) e += s_d[0][par][w];
                mean = e * inv_n;
                double q = 0.0;
#pragma unroll
                for (int j = 0; j < NV; ++j) {
                    if (!valid(j)) continue;
                    const double e0 = (double)c[j].x - mean, e1 = (double)c[j].y - mean;
                    const double e2 = (double)c[j].z - mean, e3 = (double)c[j].w - mean;
                    q += (e0 * e0 + e1 * e1) + (e2 * e2 + e3 * e3);
                }
                q = warp_sum(q);
                if (lane == 0) s_d[1][par][warp] = q;
                __syncthreads();
                q = 0.0;
#pragma unroll
                for (int w = 0; w < TB / 32; ++w) q += s_d[1][par][w];
                var = q * inv_n;
            }
            const float m32 = (float)mean;
            const double delta = mean - (double)m32;
            if (var < 0.0) var = 0.0;
            if (op == STREAM_STATS + STATS_LAYER_NORM) {
                const double inv = 1.0 / sqrt(var + (double)eps);
                // (x - mean) * inv = (x - m32) * inv - delta * inv: one FFMA
                const float invf = (float)inv, dinv = (float)(delta * inv);
                auto ln = [&](float x) { return fmaf(x - m32, invf, -dinv); };
#pragma unroll
                for (int j = 0; j < NV; ++j)
                    if (valid(j))
                        store_row4(eo, row, (tid + (uint64_t)j * TB) * 4,
                                   make_float4(ln(c[j].x), ln(c[j].y), ln(c[j].z), ln(c[j].w)));
            } else if (tid == 0) {
                static_cast<float*>(oa.data)[out_index(oa, row)] = (float)mean;
                static_cast<float*>(ob.data)[out_index(ob, row)] = (float)var;
            }
        }
    }
    if (aborted_at != ~0ull && tid == 0) {
        atomicOr(&g_reduce_status, 1u << DEV_ROWS_WAIT_TIMEOUT);
        // Drain the copies still in flight (bounded) before the block exits.
        for (uint64_t i = aborted_at; i < mine && i < aborted_at + stages; ++i)
            (void)mbar_wait(&full[i % stages], (uint32_t)((i / stages) & 1));
    }
}

// Short rows (at most 32 x 4 x NV columns) of the exp and moments families,
// one warp per row: the lanes read the row's float4s straight from global
// memory (coalesced, NV in flight per lane) and reduce with shuffles only, so
// a block holds eight rows at once and needs no barrier.  The arithmetic is
// the streamed engine's (exp2 of the f32 difference with f32 sums for the
// exp family; anchored f32 lane-pair moments with the same error bounds and
// exact f64 two-pass fallback for moments and layer norm); only the order in
// which the per-lane partials are combined differs.
constexpr int WARP_ROWS_TB = 256;

// FULL: the row is exactly 32 x 4 x NV columns (the encoder's 768), so no
// lane needs bounds checks; held to four blocks per SM (64 registers), which
// measured faster than the unchecked form's natural register count (C5 layer
// norm, 12608 x 768: 18.5 vs 19.5 us with the checks, 22.6 us uncapped).
template <typename T, int NV, int FAM, bool FULL>
__global__ void __launch_bounds__(WARP_ROWS_TB, FULL ? 4 : 1) rows_warp_kernel(Rows in, uint32_t op, RowOut oa, RowOut ob, ElemOut eo,
                                                                 float eps) {
    static_assert(FAM == FAM_EXP || FAM == FAM_MOMENTS, "exp and moments families only");
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (WARP_ROWS_TB / 32);
    const uint64_t n = in.cols;
    const double inv_n = 1.0 / (double)n;
    const T* base = reinterpret_cast<const T*>(in.data) + in.offset;
    for (uint64_t row = (uint64_t)blockIdx.x * (WARP_ROWS_TB / 32) + (threadIdx.x >> 5); row < in.rows; row += warps) {
        const unsigned char* rp = reinterpret_cast<const unsigned char*>(base + row * in.row_stride);
        auto valid = [&](int j) { return FULL || (lane + (uint64_t)j * 32) * 4 < n; };
        float4 c[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) c[j] = valid(j) ? smem_load4<T>(rp, lane + (uint64_t)j * 32) : make_float4(0.f, 0.f, 0.f, 0.f);
        if constexpr (FAM == FAM_EXP) {
            float m = -__int_as_float(0x7f800000);
#pragma unroll
            for (int j = 0; j < NV; ++j)
                if (valid(j)) m = max3(max3(m, c[j].x, c[j].y), c[j].z, c[j].w);
            m = warp_max(m);
            const float2 nm2 = make_float2(-m, -m);
            const float2 l2e = make_float2(1.4426950408889634f, 1.4426950408889634f);
            float2 e2 = make_float2(0.0f, 0.0f);
            const bool keep = op == STREAM_STATS + STATS_SOFTMAX;
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                if (!valid(j)) continue;
                const float2 t01 = __fmul2_rn(__fadd2_rn(make_float2(c[j].x, c[j].y), nm2), l2e);
                const float2 t23 = __fmul2_rn(__fadd2_rn(make_float2(c[j].z, c[j].w), nm2), l2e);
                const float2 x01 = make_float2(ex2_approx(t01.x), ex2_approx(t01.y));
                const float2 x23 = make_float2(ex2_approx(t23.x), ex2_approx(t23.y));
                e2 = __fadd2_rn(e2, __fadd2_rn(x01, x23));
                if (keep) c[j] = make_float4(x01.x, x01.y, x23.x, x23.y);
            }
            const float e = warp_sum_f(e2.x + e2.y);
            if (op == STREAM_STATS + STATS_SOFTMAX) {
                const float inv = __frcp_rn(e);
                const float2 inv2 = make_float2(inv, inv);
#pragma unroll
                for (int j = 0; j < NV; ++j)
                    if (valid(j)) {
                        const float2 y01 = __fmul2_rn(make_float2(c[j].x, c[j].y), inv2);
                        const float2 y23 = __fmul2_rn(make_float2(c[j].z, c[j].w), inv2);
                        store_row4(eo, row, (lane + (uint64_t)j * 32) * 4, make_float4(y01.x, y01.y, y23.x, y23.y));
                    }
            } else if (op == STREAM_STATS + STATS_LOG_SOFTMAX) {
                const float ls = logf(e);
                const float2 nls = make_float2(-ls, -ls);
#pragma unroll
                for (int j = 0; j < NV; ++j)
                    if (valid(j)) {
                        const float2 y01 = __fadd2_rn(__fadd2_rn(make_float2(c[j].x, c[j].y), nm2), nls);
                        const float2 y23 = __fadd2_rn(__fadd2_rn(make_float2(c[j].z, c[j].w), nm2), nls);
                        store_row4(eo, row, (lane + (uint64_t)j * 32) * 4, make_float4(y01.x, y01.y, y23.x, y23.y));
                    }
            } else if (lane == 0) {
                static_cast<float*>(oa.data)[out_index(oa, row)] = (float)((double)m + log((double)e));
            }
        } else {
            // Anchored moments (bounds as in rows_stream_kernel; the f32
            // tree over a lane's float4s has depth ceil(log2 NV), lanes and
            // the warp combine in f64).
            const float anc = 0.25f * ((__shfl_sync(0xffffffffu, c[0].x, 0) + __shfl_sync(0xffffffffu, c[0].y, 0)) +
                                       (__shfl_sync(0xffffffffu, c[0].z, 0) + __shfl_sync(0xffffffffu, c[0].w, 0)));
            const float2 na2 = make_float2(-anc, -anc);
            float2 s2[NV], q2[NV];
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                if (!valid(j)) {
                    s2[j] = q2[j] = make_float2(0.0f, 0.0f);
                    continue;
                }
                const float2 d01 = __fadd2_rn(make_float2(c[j].x, c[j].y), na2);
                const float2 d23 = __fadd2_rn(make_float2(c[j].z, c[j].w), na2);
                s2[j] = __fadd2_rn(d01, d23);
                q2[j] = __ffma2_rn(d01, d01, __fmul2_rn(d23, d23));
            }
#pragma unroll
            for (int w = 1; w < NV; w *= 2)
#pragma unroll
                for (int j = 0; j + w < NV; j += 2 * w) {
                    s2[j] = __fadd2_rn(s2[j], s2[j + w]);
                    q2[j] = __fadd2_rn(q2[j], q2[j + w]);
                }
            const double D = warp_sum((double)s2[0].x + (double)s2[0].y);
            const double Q = warp_sum((double)q2[0].x + (double)q2[0].y);
            const double dn = (double)n;
            double mean = (double)anc + D * inv_n;
            double var = (Q - D * D * inv_n) * inv_n;
            constexpr double kL = NV > 4 ? 6.0 : NV > 2 ? 5.0 : NV > 1 ? 4.0 : 3.0;  // 3 + ceil(log2 NV)
            constexpr double kLu = kL * 5.9604644775390625e-08;
            const double big = 1.7976931348623157e308;
            const double A = (double)sqrtf((float)(dn * Q)) * (1.0 + 9.5367431640625e-07);
            const bool fast = fabs(D) <= big && Q <= big && var > 1e-30 &&
                              kLu * A * inv_n <= 9.5367431640625e-07 * fmax(fabs(mean), 1.0) && Q <= 4.0 * dn * var;
            if (!fast) {  // warp-uniform: exact f64 two-pass
                double e = 0.0;
#pragma unroll
                for (int j = 0; j < NV; ++j)
                    if (valid(j)) e += ((double)c[j].x + (double)c[j].y) + ((double)c[j].z + (double)c[j].w);
                mean = warp_sum(e) * inv_n;
                double q = 0.0;
#pragma unroll
                for (int j = 0; j < NV; ++j) {
                    if (!valid(j)) continue;
                    const double e0 = (double)c[j].x - mean, e1 = (double)c[j].y - mean;
                    const double e2 = (double)c[j].z - mean, e3 = (double)c[j].w - mean;
                    q += (e0 * e0 + e1 * e1) + (e2 * e2 + e3 * e3);
                }
                var = warp_sum(q) * inv_n;
            }
            const float m32 = (float)mean;
            const double delta = mean - (double)m32;
            if (var < 0.0) var = 0.0;
            if (op == STREAM_STATS + STATS_LAYER_NORM) {
                // one f64 reciprocal square root (within an f64 ulp; its f32
                // rounding is that of the quotient 1 / sqrt but in vanishingly
                // rare ties)
                const double inv = rsqrt(var + (double)eps);
                const float invf = (float)inv, dinv = (float)(delta * inv);
                auto ln = [&](float x) { return fmaf(x - m32, invf, -dinv); };
                if (fast && eo.dtype != FB_F32) {
                    // The accepted sums were finite, so every input and every
                    // normalised value is finite: one nearest-even pack per
                    // pair rounds exactly as encode_low_pair does for non-NaN
                    // values, without its NaN fix-ups.
                    uint16_t* orow = reinterpret_cast<uint16_t*>(eo.data) + eo.offset + row * eo.row_stride;
                    const bool bf = eo.dtype == FB_BF16;
#pragma unroll
                    for (int j = 0; j < NV; ++j)
                        if (valid(j)) {
                            uint32_t w0, w1;
                            if (bf) {
                                asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w0) : "f"(ln(c[j].y)), "f"(ln(c[j].x)));
                                asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w1) : "f"(ln(c[j].w)), "f"(ln(c[j].z)));
                            } else {
                                asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(w0) : "f"(ln(c[j].y)), "f"(ln(c[j].x)));
                                asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(w1) : "f"(ln(c[j].w)), "f"(ln(c[j].z)));
                            }
                            *reinterpret_cast<uint2*>(orow + (lane + (uint64_t)j * 32) * 4) = make_uint2(w0, w1);
                        }
                } else {
#pragma unroll
                    for (int j = 0; j < NV; ++j)
                        if (valid(j))
                            store_row4(eo, row, (lane + (uint64_t)j * 32) * 4,
                                       make_float4(ln(c[j].x), ln(c[j].y), ln(c[j].z), ln(c[j].w)));
                }
            } else if (lane == 0) {
                static_cast<float*>(oa.data)[out_index(oa, row)] = (float)mean;
                static_cast<float*>(ob.data)[out_index(ob, row)] = (float)var;
            }
        }
    }
}

// Global f32 sum into one f64: grid-stride f64 partials per block, then the
// last block to finish folds the block partials in index order (so the
// result does not depend on block scheduling) and re-arms the counter.
template <int VEC>
__global__ void __launch_bounds__(BLOCK) sum_partial_kernel(Rows in, double* block_partials, unsigned* counter,
                                                            double* result) {
    __shared__ double s_sum[BLOCK / 32];
    __shared__ bool s_last;
    const float* base = reinterpret_cast<const float*>(in.data) + in.offset;
    const uint64_t n = in.cols;
    double acc = 0.0;
    const uint64_t tid = (uint64_t)blockIdx.x * BLOCK + threadIdx.x, step = (uint64_t)gridDim.x * BLOCK;
    uint64_t c0 = 0;
    if (VEC == 4) {
        const uint64_t nvec = n / 4;
        uint64_t v = tid;
        for (; v + 3 * step < nvec; v += 4 * step) {
            float4 x[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) x[u] = Elem<float>::load4(base + (v + u * step) * 4);
#pragma unroll
            for (int u = 0; u < 4; ++u) acc += ((double)x[u].x + (double)x[u].y) + ((double)x[u].z + (double)x[u].w);
        }
        for (; v < nvec; v += step) {
            const float4 x = Elem<float>::load4(base + v * 4);
            acc += ((double)x.x + (double)x.y) + ((double)x.z + (double)x.w);
        }
        c0 = nvec * 4;
    }
    for (uint64_t c = c0 + tid; c < n; c += step)
        acc += (double)Elem<float>::load(base + (in.contiguous_rows ? c : nest_offset(in.inner, c)));
    acc = block_sum<BLOCK>(acc, s_sum);
    if (threadIdx.x == 0) {
        block_partials[blockIdx.x] = acc;
        __threadfence();
        s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        double t = 0.0;
        for (unsigned b = threadIdx.x; b < gridDim.x; b += BLOCK) t += __ldcg(block_partials + b);
        t = block_sum<BLOCK>(t, s_sum);
        if (threadIdx.x == 0) {
            *result = t;
            *counter = 0u;
        }
    }
}

// Global f32 sum, streamed: the input is cut into 16 KB chunks dealt to the
// blocks round-robin (chunk b, b + grid, ...); each block streams its chunks
// HBM -> shared memory through a cp.async.bulk ring and every thread adds its
// float4s into one f64 across all its chunks (no per-chunk reduction, one
// barrier per chunk to release the ring slot).  The elements after the last
// full chunk are added by the last block with plain loads; the block partials
// are then folded in index order by the last block to finish.  The chunk
// assignment is fixed by the grid, so the result does not depend on block
// scheduling.
constexpr uint32_t kSumChunk = 4096;  // floats per chunk
constexpr int kSumTB = 128;
constexpr int kSumNV = kSumChunk / 4 / kSumTB;  // float4s per thread per chunk

__global__ void __launch_bounds__(kSumTB) sum_stream_kernel(const float* base, uint64_t chunks, uint64_t tail_n,
                                                           uint32_t stages, double* block_partials, unsigned* counter,
                                                           double* result) {
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    unsigned char* ring = smem + 128;
    __shared__ double s_sum[kSumTB / 32];
    __shared__ bool s_last;
    __shared__ int s_abort;
    constexpr uint32_t kBytes = kSumChunk * 4;
    const uint32_t tid = threadIdx.x;
    const uint64_t first = blockIdx.x, step = gridDim.x;
    const uint64_t mine = first < chunks ? (chunks - 1 - first) / step + 1 : 0;
    if (tid == 0) {
        for (uint32_t s = 0; s < stages; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
        s_abort = 0;
    }
    __syncthreads();
    auto issue = [&](uint64_t i) {
        const uint32_t s = (uint32_t)(i % stages);
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&full[s], kBytes);
        bulk_g2s(ring + (uint64_t)s * kBytes, base + (first + i * step) * kSumChunk, kBytes, &full[s]);
    };
    if (tid == 0)
        for (uint64_t i = 0; i < mine && i < stages; ++i) issue(i);
    double acc = 0.0;
    uint64_t aborted_at = ~0ull;
    for (uint64_t i = 0; i < mine; ++i) {
        const uint32_t s = (uint32_t)(i % stages);
        if (!mbar_wait(&full[s], (uint32_t)((i / stages) & 1))) s_abort = 1;
        const float4* rb = reinterpret_cast<const float4*>(ring + (uint64_t)s * kBytes);
        float4 x[kSumNV];
#pragma unroll
        for (int j = 0; j < kSumNV; ++j) x[j] = rb[tid + j * kSumTB];
        __syncthreads();  // every thread has read slot s
        if (s_abort) {
            aborted_at = i;
            break;
        }
        if (tid == 0 && i + stages < mine) issue(i + stages);
#pragma unroll
        for (int j = 0; j < kSumNV; ++j)
            acc += ((double)x[j].x + (double)x[j].y) + ((double)x[j].z + (double)x[j].w);
    }
    if (aborted_at != ~0ull && tid == 0) {
        atomicOr(&g_reduce_status, 1u << DEV_ROWS_WAIT_TIMEOUT);
        for (uint64_t i = aborted_at; i < mine && i < aborted_at + stages; ++i)
            (void)mbar_wait(&full[i % stages], (uint32_t)((i / stages) & 1));
    }
    if (blockIdx.x == gridDim.x - 1)
        for (uint64_t c = tid; c < tail_n; c += kSumTB) acc += (double)base[chunks * kSumChunk + c];
    // The finishing protocol runs even after a timeout (the status word
    // reports it), so that the counter is re-armed for the next call.
    acc = block_sum<kSumTB>(acc, s_sum);
    if (tid == 0) {
        block_partials[blockIdx.x] = acc;
        __threadfence();
        s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        double t = 0.0;
        for (unsigned b = tid; b < gridDim.x; b += kSumTB) t += __ldcg(block_partials + b);
        t = block_sum<kSumTB>(t, s_sum);
        if (tid == 0) {
            *result = t;
            *counter = 0u;
        }
    }
}

__global__ void finish_sum_kernel(const double* partial, float* out) { *out = (float)*partial; }

__global__ void fill_kernel(uint32_t* out, uint64_t count, uint32_t bits) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = bits;
}

template <typename E>
__global__ void copy_kernel(const E* in, uint64_t in_offset, Nest in_nest, E* out, uint64_t out_offset, Nest out_nest,
                            uint64_t count) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x)
        out[out_offset + nest_offset(out_nest, i)] = in[in_offset + nest_offset(in_nest, i)];
}

__global__ void cast_to_low_kernel(const float* in, uint64_t in_offset, Nest in_nest, uint16_t* out, uint32_t dtype,
                                   uint64_t count) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x) {
        const float x = in[in_offset + nest_offset(in_nest, i)];
        out[i] = dtype == FB_BF16 ? encode_bf16(x) : encode_f16(x);
    }
}

__global__ void cast_to_low_vec8_kernel(const float* in, uint64_t in_offset, Nest in_nest, uint16_t* out, uint32_t dtype,
                                        uint64_t runs) {
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < runs; t += (uint64_t)gridDim.x * blockDim.x) {
        const float4* src = reinterpret_cast<const float4*>(in + in_offset + nest_offset(in_nest, t * 8));
        const float4 a = src[0], b = src[1];
        reinterpret_cast<uint4*>(out)[t] = make_uint4(encode_low_pair(a.x, a.y, dtype), encode_low_pair(a.z, a.w, dtype),
                                                      encode_low_pair(b.x, b.y, dtype), encode_low_pair(b.z, b.w, dtype));
    }
}

unsigned grid_for(uint64_t work, unsigned per_sm = 8) {
    const uint64_t cap = (uint64_t)sm_count() * per_sm;
    uint64_t g = work < cap ? work : cap;
    return (unsigned)(g ? g : 1);
}

int check_launch(const char* kernel) {
    count_launch(kernel);
    return launch_status("kernel launch");
}

bool vec_ok(const Rows& in) {
    if (!in.contiguous_rows) return false;
    const uint64_t esz = in.dtype == FB_F32 || in.dtype == FB_U32 ? 4 : 2;
    const uintptr_t addr = reinterpret_cast<uintptr_t>(in.data) + in.offset * esz;
    return addr % (4 * esz) == 0 && (in.rows <= 1 || in.row_stride % 4 == 0);
}

template <typename T>
int reduce_typed(uint32_t op, const Rows& in, const RowOut& out, cudaStream_t s) {
    const unsigned g = grid_for(in.rows);
    if (vec_ok(in))
        reduce_rows_kernel<T, 4><<<g, BLOCK, 0, s>>>(in, out, op);
    else
        reduce_rows_kernel<T, 1><<<g, BLOCK, 0, s>>>(in, out, op);
    return check_launch("reduce_rows_kernel");
}

template <typename T>
int stats_typed(uint32_t op, const Rows& in, const ElemOut& out, const RowOut& a, const RowOut& b, float eps,
                cudaStream_t s) {
    const unsigned g = grid_for(in.rows);
    const bool elementwise = op == STATS_SOFTMAX || op == STATS_LOG_SOFTMAX || op == STATS_LAYER_NORM;
    const bool out_ok = !elementwise ||
                        (out.contiguous_rows && reinterpret_cast<uintptr_t>(out.data + out.offset) % 16 == 0 &&
                         (in.rows <= 1 || out.row_stride % 4 == 0));
    const bool cache = vec_ok(in) && in.cols % 4 == 0 && out_ok;
    const uint64_t per_pass = 4ull * BLOCK;
    if (cache && in.cols <= per_pass)
        stats_rows_kernel<T, 1><<<g, BLOCK, 0, s>>>(in, out, a, b, op, eps);
    else if (cache && in.cols <= 2 * per_pass)
        stats_rows_kernel<T, 2><<<g, BLOCK, 0, s>>>(in, out, a, b, op, eps);
    else if (cache && in.cols <= 4 * per_pass)
        stats_rows_kernel<T, 4><<<g, BLOCK, 0, s>>>(in, out, a, b, op, eps);
    else if (cache && in.cols <= 8 * per_pass)
        stats_rows_kernel<T, 8><<<g, BLOCK, 0, s>>>(in, out, a, b, op, eps);
    else
        stats_rows_kernel<T, 0><<<g, BLOCK, 0, s>>>(in, out, a, b, op, eps);
    return check_launch("stats_rows_kernel");
}

// Launches the streamed engine when the geometry allows it; returns
// FB_ERR_UNSUPPORTED otherwise.
template <typename T>
int stream_typed(uint32_t op, const Rows& in, const RowOut& a, const RowOut& b, const ElemOut& eo, float eps,
                 cudaStream_t st) {
    const uint64_t esz = sizeof(T);
    const uint64_t row_bytes = in.cols * esz;
    if (!in.contiguous_rows || in.cols == 0 || in.cols % 4 != 0 || row_bytes % 16 != 0) return FB_ERR_UNSUPPORTED;
    if (in.cols > 8ull * 4 * BLOCK) return FB_ERR_UNSUPPORTED;
    const uintptr_t addr = reinterpret_cast<uintptr_t>(in.data) + in.offset * esz;
    if (addr % 16 != 0 || (in.rows > 1 && (in.row_stride * esz) % 16 != 0)) return FB_ERR_UNSUPPORTED;
    const bool elementwise = op == STREAM_STATS + STATS_SOFTMAX || op == STREAM_STATS + STATS_LOG_SOFTMAX ||
                             op == STREAM_STATS + STATS_LAYER_NORM;
    const uint64_t oesz = eo.dtype == FB_F32 ? 4 : 2;
    if (elementwise && !(eo.contiguous_rows && (reinterpret_cast<uintptr_t>(eo.data) + eo.offset * oesz) % (4 * oesz) == 0 &&
                         (in.rows <= 1 || eo.row_stride % 4 == 0)))
        return FB_ERR_UNSUPPORTED;
    const uint64_t vec = in.cols / 4;
    // Short rows of the exp and moments families: one warp per row.
    const bool exp_fam = op == STREAM_STATS + STATS_SOFTMAX || op == STREAM_STATS + STATS_LOG_SOFTMAX ||
                         op == STREAM_STATS + STATS_LOGSUMEXP;
    const bool mom_fam = op == STREAM_STATS + STATS_MOMENTS || op == STREAM_STATS + STATS_LAYER_NORM;
    if ((exp_fam || mom_fam) && vec <= 8 * 32) {
        auto launch_w = [&](auto kernel) -> int {
            int per_sm = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, WARP_ROWS_TB, 0) != cudaSuccess || per_sm < 1)
                return FB_ERR_UNSUPPORTED;
            const uint64_t want = (in.rows + WARP_ROWS_TB / 32 - 1) / (WARP_ROWS_TB / 32);
            const uint64_t cap = (uint64_t)sm_count() * (uint64_t)per_sm;
            kernel<<<(unsigned)(want < cap ? want : cap), WARP_ROWS_TB, 0, st>>>(in, op, a, b, eo, eps);
            return check_launch("rows_warp_kernel");
        };
        auto by_nv = [&](auto fam_c) -> int {
            constexpr int F = decltype(fam_c)::value;
            if (vec == 32) return launch_w(rows_warp_kernel<T, 1, F, true>);
            if (vec == 64) return launch_w(rows_warp_kernel<T, 2, F, true>);
            if (vec == 128) return launch_w(rows_warp_kernel<T, 4, F, true>);
            if (vec == 192) return launch_w(rows_warp_kernel<T, 6, F, true>);
            if (vec <= 32) return launch_w(rows_warp_kernel<T, 1, F, false>);
            if (vec <= 64) return launch_w(rows_warp_kernel<T, 2, F, false>);
            if (vec <= 128) return launch_w(rows_warp_kernel<T, 4, F, false>);
            if (vec <= 192) return launch_w(rows_warp_kernel<T, 6, F, false>);
            return launch_w(rows_warp_kernel<T, 8, F, false>);
        };
        return exp_fam ? by_nv(std::integral_constant<int, FAM_EXP>{}) : by_nv(std::integral_constant<int, FAM_MOMENTS>{});
    }
    // Row reductions without an elementwise output (sum, min/max, argmax,
    // mean, moments, logsumexp) run 128-thread blocks with a short ring: more
    // rows in reduction at once per SM hides each row's reduce/barrier
    // latency.  Layer norm on long rows (more than 1024 columns) measured
    // faster with 256 threads and a deeper ring.
    const bool writes_row = op == STREAM_STATS + STATS_SOFTMAX || op == STREAM_STATS + STATS_LOG_SOFTMAX ||
                            op == STREAM_STATS + STATS_LAYER_NORM;
    // Since each operation family has its own registers, the exp family
    // (softmax, log-softmax) measured faster with 128 threads on long rows
    // too (4096 columns: 5.61 vs 5.47 TB/s); layer norm keeps 256.
    const uint32_t tb = vec > 128 && (vec <= (writes_row ? 256u : 8u * 128) || (exp_fam && vec <= 8u * 128)) ? 128 : 256;
    const int nv = vec <= tb ? 1 : vec <= 2 * tb ? 2 : vec <= 4 * tb ? 4 : 8;
    if ((uint64_t)nv * 4 * tb < in.cols) return FB_ERR_UNSUPPORTED;
    // Ring depth: enough rows in flight to cover HBM latency, within shared memory.
    uint32_t stages = row_bytes <= 4096 ? 8 : row_bytes <= 8192 ? 5 : 3;
    if (tb == 128) stages = row_bytes <= 4096 ? 4 : 2;
    auto launch = [&](auto kernel, uint32_t threads) -> int {
        const size_t smem = 128 + (size_t)stages * row_bytes;
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return FB_ERR_DRIVER;
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1)
            return FB_ERR_UNSUPPORTED;
        const uint64_t cap = (uint64_t)sm_count() * (uint64_t)per_sm;
        const unsigned grid = (unsigned)(in.rows < cap ? in.rows : cap);
        kernel<<<grid, threads, smem, st>>>(in, op, a, b, eo, eps, stages, (uint32_t)row_bytes);
        return check_launch("rows_stream_kernel");
    };
    const bool cap = op == ROW_ARGMAX || op == STREAM_STATS + STATS_MOMENTS;
    const int fam = op == ROW_SUM || op == ROW_MEAN                             ? FAM_SUM
                    : op == ROW_MIN || op == ROW_MAX || op == ROW_ARGMAX        ? FAM_EXTREME
                    : op == STREAM_STATS + STATS_SOFTMAX || op == STREAM_STATS + STATS_LOG_SOFTMAX ||
                              op == STREAM_STATS + STATS_LOGSUMEXP
                        ? FAM_EXP
                        : FAM_MOMENTS;
    auto with_nv = [&](auto tb_c, auto cap_c, auto fam_c) -> int {
        constexpr int TBc = decltype(tb_c)::value;
        constexpr bool CAPc = decltype(cap_c)::value;
        constexpr int F = decltype(fam_c)::value;
        switch (nv) {
            case 1: return launch(rows_stream_kernel<T, 1, TBc, CAPc, F>, TBc);
            case 2: return launch(rows_stream_kernel<T, 2, TBc, CAPc, F>, TBc);
            case 4: return launch(rows_stream_kernel<T, 4, TBc, CAPc, F>, TBc);
            default: return launch(rows_stream_kernel<T, 8, TBc, CAPc, F>, TBc);
        }
    };
    using I128 = std::integral_constant<int, 128>;
    using I256 = std::integral_constant<int, 256>;
    using Cap = std::true_type;
    using NoCap = std::false_type;
    auto with_fam = [&](auto fam_c) -> int {
        constexpr int F = decltype(fam_c)::value;
        if (tb == 128 && cap) {
            if constexpr (F == FAM_EXTREME || F == FAM_MOMENTS) return with_nv(I128{}, Cap{}, fam_c);
        }
        if (tb == 128) return with_nv(I128{}, NoCap{}, fam_c);
        return with_nv(I256{}, NoCap{}, fam_c);
    };
    switch (fam) {
        case FAM_SUM: return with_fam(std::integral_constant<int, FAM_SUM>{});
        case FAM_EXTREME: return with_fam(std::integral_constant<int, FAM_EXTREME>{});
        case FAM_EXP: return with_fam(std::integral_constant<int, FAM_EXP>{});
        default: return with_fam(std::integral_constant<int, FAM_MOMENTS>{});
    }
}

int stream_rows(uint32_t op, const Rows& in, const RowOut& a, const RowOut& b, const ElemOut& eo, float eps,
                cudaStream_t st) {
    switch (in.dtype) {
        case FB_F32: return stream_typed<float>(op, in, a, b, eo, eps, st);
        case FB_BF16: return stream_typed<__nv_bfloat16>(op, in, a, b, eo, eps, st);
        case FB_F16: return stream_typed<__half>(op, in, a, b, eo, eps, st);
        default: return FB_ERR_UNSUPPORTED;
    }
}

}  // namespace

uint32_t read_reduce_status() {
    uint32_t v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_reduce_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    cudaMemcpyToSymbol(g_reduce_status, &zero, sizeof(zero));
    return v;
}

int launch_reduce_rows(uint32_t op, const Rows& in, const RowOut& out, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (in.rows == 0) return FB_OK;
    if (op != ROW_PRODUCT && in.dtype != FB_U32) {
        const int r = stream_rows(op, in, out, RowOut{}, ElemOut{}, 0.0f, s);
        if (r != FB_ERR_UNSUPPORTED) return r;
    }
    switch (in.dtype) {
        case FB_F32: return reduce_typed<float>(op, in, out, s);
        case FB_BF16: return reduce_typed<__nv_bfloat16>(op, in, out, s);
        case FB_F16: return reduce_typed<__half>(op, in, out, s);
        case FB_U32:
            reduce_rows_u32_kernel<<<grid_for(in.rows), BLOCK, 0, s>>>(in, out, op);
            return check_launch("reduce_rows_u32_kernel");
        default: return FB_ERR_DTYPE;
    }
}

int launch_stats_rows(uint32_t op, const Rows& in, const ElemOut& out, const RowOut& a, const RowOut& b, float eps,
                      void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (in.rows == 0) return FB_OK;
    const int r = stream_rows(STREAM_STATS + op, in, a, b, out, eps, s);
    if (r != FB_ERR_UNSUPPORTED) return r;
    if (out.dtype != FB_F32) return FB_ERR_UNSUPPORTED;  // 16-bit rows: streamed engine only
    switch (in.dtype) {
        case FB_F32: return stats_typed<float>(op, in, out, a, b, eps, s);
        case FB_BF16: return stats_typed<__nv_bfloat16>(op, in, out, a, b, eps, s);
        case FB_F16: return stats_typed<__half>(op, in, out, a, b, eps, s);
        default: return FB_ERR_DTYPE;
    }
}

int launch_sum_partial(const Rows& in, double* partial, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Scratch layout: [u32 counter, padded to 256 bytes][block partials], the
    // same for both kernels so that the counter every call re-arms is shared.
    const float* base = reinterpret_cast<const float*>(in.data) + in.offset;
    if (in.rows == 1 && in.contiguous_rows && reinterpret_cast<uintptr_t>(base) % 16 == 0 &&
        in.cols >= (uint64_t)kSumChunk * (uint64_t)sm_count()) {
        const uint32_t stages = 2;
        const size_t smem = 128 + (size_t)stages * kSumChunk * 4;
        if (cudaFuncSetAttribute(sum_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return FB_ERR_DRIVER;
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sum_stream_kernel, kSumTB, smem) != cudaSuccess ||
            per_sm < 1)
            return FB_ERR_DRIVER;
        const uint64_t chunks = in.cols / kSumChunk;
        const uint64_t cap = (uint64_t)sm_count() * (uint64_t)per_sm;
        const unsigned g = (unsigned)(chunks < cap ? chunks : cap);
        char* scr = static_cast<char*>(scratch(stream, 256 + (uint64_t)g * sizeof(double), SCRATCH_SUM));
        if (!scr) return FB_ERR_DRIVER;
        sum_stream_kernel<<<g, kSumTB, smem, s>>>(base, chunks, in.cols % kSumChunk, stages,
                                                   reinterpret_cast<double*>(scr + 256),
                                                   reinterpret_cast<unsigned*>(scr), partial);
        return check_launch("sum_stream_kernel");
    }
    const unsigned g = (unsigned)sm_count() * 4;
    char* scr = static_cast<char*>(scratch(stream, 256 + (uint64_t)g * sizeof(double), SCRATCH_SUM));
    if (!scr) return FB_ERR_DRIVER;
    double* partials = reinterpret_cast<double*>(scr + 256);
    unsigned* counter = reinterpret_cast<unsigned*>(scr);
    if (vec_ok(in))
        sum_partial_kernel<4><<<g, BLOCK, 0, s>>>(in, partials, counter, partial);
    else
        sum_partial_kernel<1><<<g, BLOCK, 0, s>>>(in, partials, counter, partial);
    return check_launch("sum_partial_kernel");
}

// Global-sum partial without allocation.  Some callers cannot call
// cudaMalloc (engines that reserve the device's memory up front and route
// every allocation through their own pool, and latency-critical paths on
// which cudaMalloc's implicit device-wide synchronisation is not acceptable),
// so this variant keeps its block partials and finishing counter in a
// file-scope device array instead of library-allocated scratch.  The array is
// FB_SUM_STATIC_SCRATCH_BYTES per device and lives until the process exits;
// every call shares it and it keeps the last call's contents, so the counter
// is cleared at the start of each call and calls that overlap on the GPU
// race.  In host code the array's name is only a host-side stand-in, so its
// device address is looked up once per device (with that device current) and
// cached; the first call on each device performs that lookup and should
// therefore come before any stream capture.
namespace {
constexpr uint64_t kStaticCounterBytes = 256;
constexpr uint64_t kStaticPartials = (FB_SUM_STATIC_SCRATCH_BYTES - kStaticCounterBytes) / sizeof(double);
constexpr uint64_t kStaticBlockElems = 1ull << 18;  // elements per block of the static variant

static __device__ __align__(256) unsigned char g_sum_static_scratch[FB_SUM_STATIC_SCRATCH_BYTES];

std::mutex g_static_mutex;
void* g_static_addr[64] = {};

// Device address of g_sum_static_scratch on the current device.
int static_sum_scratch(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FB_ERR_DRIVER;
    std::lock_guard<std::mutex> lock(g_static_mutex);
    if (!g_static_addr[dev]) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_sum_static_scratch) != cudaSuccess || !ptr) return FB_ERR_DRIVER;
        g_static_addr[dev] = ptr;
    }
    *out = g_static_addr[dev];
    return FB_OK;
}
}  // namespace

uint64_t static_sum_max_elements() { return kStaticPartials * kStaticBlockElems; }

int launch_sum_partial_static(const Rows& in, double* partial, void* stream) {
    const uint64_t count = in.cols;
    const uint64_t needed = count == 0 ? 1 : (count + kStaticBlockElems - 1) / kStaticBlockElems;
    if (needed > kStaticPartials) return FB_ERR_INVALID_INPUT;
    // The kernel is grid-stride: at least four blocks per SM (as the
    // allocating path launches) so small inputs get the full bandwidth, one
    // per 2^18 elements beyond that, never more partials than the array holds.
    const uint64_t floor_blocks = std::min<uint64_t>((uint64_t)sm_count() * 4, kStaticPartials);
    const uint64_t blocks = std::max(needed, floor_blocks);
    void* base = nullptr;
    const int rc = static_sum_scratch(&base);
    if (rc != FB_OK) return rc;
    double* partials = static_cast<double*>(base);
    unsigned* counter =
        reinterpret_cast<unsigned*>(static_cast<char*>(base) + FB_SUM_STATIC_SCRATCH_BYTES - kStaticCounterBytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(counter, 0, sizeof(unsigned), s) != cudaSuccess) return FB_ERR_DRIVER;
    if (vec_ok(in))
        sum_partial_kernel<4><<<(unsigned)blocks, BLOCK, 0, s>>>(in, partials, counter, partial);
    else
        sum_partial_kernel<1><<<(unsigned)blocks, BLOCK, 0, s>>>(in, partials, counter, partial);
    return check_launch("sum_partial_kernel");
}

// One thread waits on an mbarrier that nothing arrives at, with the same
// bounded wait every kernel here uses but a caller-chosen limit; the wait
// gives up, the timeout is recorded in the status word and the kernel
// returns.  No copy or MMA is in flight, so nothing needs draining.
__global__ void selftest_wait_kernel(uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_barrier_init();
    if (!mbar_wait_for(&bar, 0, limit_ns)) atomicOr(&g_reduce_status, 1u << DEV_SELFTEST_TIMEOUT);
}

int launch_selftest_wait(uint64_t limit_ns, void* stream) {
    selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns);
    return check_launch("selftest_wait_kernel");
}

int launch_finish_sum(const double* partial, float* out, void* stream) {
    finish_sum_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(partial, out);
    return check_launch("finish_sum_kernel");
}

int launch_fill(void* data, uint64_t count, uint32_t bits, void* stream) {
    if (count == 0) return FB_OK;
    fill_kernel<<<grid_for((count + BLOCK - 1) / BLOCK), BLOCK, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint32_t*>(data), count, bits);
    return check_launch("fill_kernel");
}

int launch_copy(const void* in, uint32_t elem_bytes, uint64_t in_offset, const Nest& in_nest, void* out,
                uint64_t out_offset, const Nest& out_nest, uint64_t count, void* stream) {
    if (count == 0) return FB_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned g = grid_for((count + BLOCK - 1) / BLOCK);
    if (elem_bytes == 4)
        copy_kernel<uint32_t><<<g, BLOCK, 0, s>>>(static_cast<const uint32_t*>(in), in_offset, in_nest,
                                                  static_cast<uint32_t*>(out), out_offset, out_nest, count);
    else
        copy_kernel<uint16_t><<<g, BLOCK, 0, s>>>(static_cast<const uint16_t*>(in), in_offset, in_nest,
                                                  static_cast<uint16_t*>(out), out_offset, out_nest, count);
    return check_launch("copy_kernel");
}

int launch_cast_to_low(const float* in, uint64_t in_offset, const Nest& in_nest, uint16_t* out, uint32_t dtype,
                       uint64_t count, void* stream) {
    if (count == 0) return FB_OK;
    if (vec8_ok(in_nest, in, in_offset, out)) {
        const uint64_t runs = count / 8;
        cast_to_low_vec8_kernel<<<grid_for((runs + BLOCK - 1) / BLOCK, 16), BLOCK, 0,
                                  static_cast<cudaStream_t>(stream)>>>(in, in_offset, in_nest, out, dtype, runs);
        return check_launch("cast_to_low_vec8_kernel");
    }
    cast_to_low_kernel<<<grid_for((count + BLOCK - 1) / BLOCK), BLOCK, 0, static_cast<cudaStream_t>(stream)>>>(
        in, in_offset, in_nest, out, dtype, count);
    return check_launch("cast_to_low_kernel");
}

}  // namespace fb
