// Launch interface between the C ABI (api.cpp) and the CUDA translation
// units.  Everything here is plain data: the ABI layer validates and
// canonicalises descriptors, the launchers only enqueue work.
#pragma once

#include <cstdint>
#include <initializer_list>
#include <string>

#include "../../include/forma_b200.h"

namespace fb {

// An index nest: logical row-major coordinates over `dims` mapped to an
// element offset through `strides` (the reference's index_of walk,
// compute-cuda/src/kernels.cu:5-13, with the dims resident in kernel
// parameters instead of an uploaded u64 descriptor).
struct Nest {
    uint32_t rank = 0;
    uint64_t dims[FB_MAX_RANK] = {};
    uint64_t strides[FB_MAX_RANK] = {};
};

// A row-structured view of a reduction or statistics operand: row r, column
// c lives at `offset + outer(r) + inner(c)`.  When `contiguous_rows` is set
// the inner nest is one stride-1 axis of `cols` elements and the outer nest
// one axis of stride `row_stride`.
struct Rows {
    const void* data = nullptr;
    uint32_t dtype = FB_F32;
    uint64_t offset = 0;
    uint64_t rows = 0, cols = 0;
    Nest outer, inner;
    bool contiguous_rows = false;
    uint64_t row_stride = 0;
};

// Destination of one value per row (reductions, logsumexp, moments).
struct RowOut {
    void* data = nullptr;
    uint64_t offset = 0;
    Nest nest;  // over rows
    bool contiguous = false;
};

// Destination with the input's geometry (softmax, log-softmax, layer norm).
struct ElemOut {
    float* data = nullptr;  // storage base (16-bit storage when dtype is F16/BF16)
    uint64_t offset = 0;
    Nest outer, inner;
    bool contiguous_rows = false;
    uint64_t row_stride = 0;
    // FB_F32, or FB_F16/FB_BF16: rounded once (nearest even) on store; only
    // the streamed row engine writes 16-bit rows (others: FB_ERR_UNSUPPORTED)
    uint32_t dtype = FB_F32;
};

enum RowOp : uint32_t {
    ROW_SUM = 0,
    ROW_PRODUCT = 1,
    ROW_MIN = 2,
    ROW_MAX = 3,
    ROW_MEAN = 4,
    ROW_ARGMAX = 5,
};

enum StatsOp : uint32_t {
    STATS_SOFTMAX = 0,
    STATS_LOG_SOFTMAX = 1,
    STATS_LAYER_NORM = 2,
    STATS_LOGSUMEXP = 3,
    STATS_MOMENTS = 4,
};

// Library-owned scratch for the calling (device, stream, slot); grows on
// demand and lives until process exit.  Each slot serves one purpose so that
// buffers used within one call (or carrying state between calls, like the
// global sum's re-armed counter) never alias.  Returns nullptr on failure.
enum ScratchSlot : int {
    SCRATCH_SUM = 0,          // global-sum block partials + finishing counter
    SCRATCH_CONV_RESULT = 1,  // f32 convolution result before low rounding
    SCRATCH_CONV_WEIGHT = 2,  // weights gathered into [O, kh, kw, C] or [O, C, kh, kw]
    SCRATCH_CONV_PATCH = 3,   // non-overlapping patches gathered into [N*P*Q, C*kh*kw]
    SCRATCH_STATS = 4,        // f32 statistics result before low rounding
    SCRATCH_ATTN_SPLIT = 5,   // split-key attention partials (f64 per row and key range)
    SCRATCH_ATTN_RESULT = 6,  // f32 attention result before low rounding
    SCRATCH_COLLECTIVE = 7,   // the global sum's f64 partial, all-reduced in place
    SCRATCH_SLOTS = 8,
};
void* scratch(void* stream, uint64_t bytes, int slot);
int sm_count();
// Records one enqueued launch of `kernel`: counted by fb_launch_count and
// appended to this host thread's fb_last_route.
void count_launch(const char* kernel);
// "base<p0,p1,...>": the name of a template instantiation for count_launch.
std::string kernel_name(const char* base, std::initializer_list<int> params);
// Starts a new route record for this host thread (every entry point calls it).
void begin_route();
// Launches this host thread has enqueued (prepared programs count theirs).
uint64_t thread_launch_count();
// In-place NCCL sum of `count` doubles on `stream` (collective.cpp); the
// communicator must belong to the current device.
int nccl_all_reduce_sum_f64(double* buf, uint64_t count, void* comm, void* stream);
// Records the pending CUDA error (if any) with `what` as this thread's driver
// error detail and returns FB_OK when there was none, FB_ERR_DRIVER otherwise.
int launch_status(const char* what);

// Per translation unit: reads and clears the device status word.
uint32_t read_reduce_status();
uint32_t read_gemm_status();
uint32_t read_attention_status();

// ---- reductions / statistics (reduce.cu) ----
int launch_reduce_rows(uint32_t op, const Rows& in, const RowOut& out, void* stream);
int launch_stats_rows(uint32_t op, const Rows& in, const ElemOut& out, const RowOut& out_a, const RowOut& out_b,
                      float epsilon, void* stream);
int launch_sum_partial(const Rows& in, double* partial, void* stream);
int launch_finish_sum(const double* partial, float* out, void* stream);
// The no-allocation variant: scratch in a static device array (reduce.cu).
int launch_sum_partial_static(const Rows& in, double* partial, void* stream);
uint64_t static_sum_max_elements();
// One CTA whose bounded wait on an mbarrier nobody arrives at gives up after
// `limit_ns` and records DEV_SELFTEST_TIMEOUT (fb_selftest_bounded_wait).
int launch_selftest_wait(uint64_t limit_ns, void* stream);
// Writes `count` elements of `value` (f32 or u32 bits) into a dense-permuted output.
int launch_fill(void* data, uint64_t count, uint32_t bits, void* stream);
// Copies a strided view into a (dense-permuted) output of the same logical shape.
int launch_copy(const void* in, uint32_t elem_bytes, uint64_t in_offset, const Nest& in_nest, void* out,
                uint64_t out_offset, const Nest& out_nest, uint64_t count, void* stream);
// Rounds f32 (strided) into F16/BF16 contiguous storage, nearest-even.
// An f32 -> 16-bit elementwise pass may move 8 elements per thread (two
// float4 loads, one 16-byte store) when the nest's innermost axis is
// contiguous with a multiple of 8 elements and every run starts 16-byte
// aligned on both sides.
inline bool vec8_ok(const Nest& n, const float* in, uint64_t in_offset, const uint16_t* out) {
    if (n.rank == 0 || n.strides[n.rank - 1] != 1 || n.dims[n.rank - 1] % 8 != 0) return false;
    for (uint32_t d = 0; d + 1 < n.rank; ++d)
        if (n.strides[d] % 4 != 0) return false;
    return reinterpret_cast<uintptr_t>(in + in_offset) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0;
}

// ---- elementwise glue (glue.cu) ----
int launch_add(const float* a, uint64_t a_off, const Nest& an, const float* b, uint64_t b_off, const Nest& bn, float* out,
               uint64_t out_off, const Nest& on, uint64_t count, bool dense, void* stream);
int launch_gelu_to_low(const float* in, uint64_t in_off, const Nest& n, uint16_t* out, uint32_t dtype, uint64_t count,
                       void* stream);
int launch_cast_to_low(const float* in, uint64_t in_offset, const Nest& in_nest, uint16_t* out, uint32_t dtype,
                       uint64_t count, void* stream);

// ---- convolution (conv_simt.cu, conv_tc.cu) ----
struct ConvArgs {
    const void* input = nullptr;
    const void* weight = nullptr;
    float* output = nullptr;
    uint32_t dtype = FB_F32;  // input/weight dtype
    uint32_t spatial = 0;
    uint64_t in_offset = 0, w_offset = 0, out_offset = 0;
    uint64_t batch = 0, channels_per_group = 0, outputs_per_group = 0, out_channels = 0;
    uint64_t in_stride_n = 0, in_stride_c = 0, w_stride_o = 0, w_stride_c = 0;
    uint64_t out_stride_n = 0, out_stride_c = 0;
    uint64_t in_dims[3] = {1, 1, 1}, out_dims[3] = {1, 1, 1}, k_dims[3] = {1, 1, 1};
    uint64_t in_strides[3] = {0, 0, 0}, w_strides[3] = {0, 0, 0}, out_strides[3] = {0, 0, 0};
    uint64_t stride[3] = {1, 1, 1}, dilation[3] = {1, 1, 1}, pad[3] = {0, 0, 0};
    uint64_t out_count = 0;
    // 0: `output` is f32.  FB_BF16 / FB_F16: `output` points at 16-bit storage
    // and the result is rounded once (conv_low); only the tensor-core path
    // accepts this, the others return FB_ERR_UNSUPPORTED for it.
    uint32_t out_low = 0;
    // Epilogue of the tensor-core path (the others return FB_ERR_UNSUPPORTED
    // when either is set): act 1 applies the tanh GELU to each f32 sum before
    // it is stored or rounded; accumulate 1 adds each f32 sum to the f32
    // output already in memory (output += conv).
    uint32_t act = 0, accumulate = 0;
};
int launch_conv_direct(const ConvArgs& a, void* stream);
// Returns FB_ERR_UNSUPPORTED when the geometry has no tiled kernel.
int launch_conv2d_f32_tiled(const ConvArgs& a, void* stream);
int launch_conv_tc(const ConvArgs& a, void* stream);

// ---- low-precision GEMM (conv_tc.cu tensor cores, gemm_simt.cu any layout) ----
struct GemmArgs {
    const void* a = nullptr;  // left  [batch..., M, K]
    const void* b = nullptr;  // right [batch..., K, N]
    void* out = nullptr;      // [batch..., M, N]
    uint32_t dtype = FB_BF16; // operands
    uint32_t out_low = 0;     // 0: f32 output; FB_BF16 / FB_F16: rounded once
    uint64_t M = 0, N = 0, K = 0;
    uint64_t a_off = 0, b_off = 0, o_off = 0;
    uint64_t a_sm = 0, a_sk = 0, b_sk = 0, b_sn = 0, o_sm = 0, o_sn = 0;  // element strides
    uint64_t batch = 1;                 // batch index count
    Nest a_batch, b_batch, o_batch;     // batch index -> element offset (stride 0 broadcasts)
};
// Returns FB_ERR_UNSUPPORTED when the layout or sizes have no tensor-core form.
int launch_gemm_tc(const GemmArgs& g, void* stream);
int launch_gemm_simt(const GemmArgs& g, void* stream);

// ---- attention (attention_simt.cu, attention_tc.cu) ----
struct AttnArgs {
    const void* q = nullptr;
    const void* k = nullptr;
    const void* v = nullptr;
    const void* mask = nullptr;
    float* out = nullptr;   // f32 rows, or 16-bit rows (o_offset in 2-byte elements) when out_low != 0
    uint32_t out_low = 0;   // 0, or FB_BF16 / FB_F16: rows rounded once (nearest even); tensor-core path only
    uint32_t dtype = FB_F32;
    uint32_t mask_kind = FB_MASK_NONE;
    // Row nest over [batch..., heads, queries] with per-operand strides; K/V
    // strides on the query axis are zero and their head coordinate is the
    // query head divided by `group_size`.
    uint32_t row_rank = 0;
    uint64_t row_dims[FB_MAX_RANK] = {};
    uint64_t q_row_strides[FB_MAX_RANK] = {}, k_row_strides[FB_MAX_RANK] = {};
    uint64_t v_row_strides[FB_MAX_RANK] = {}, m_row_strides[FB_MAX_RANK] = {};
    uint64_t o_row_strides[FB_MAX_RANK] = {};
    uint64_t q_offset = 0, k_offset = 0, v_offset = 0, m_offset = 0, o_offset = 0;
    uint64_t q_stride_d = 0, k_stride_key = 0, k_stride_d = 0, v_stride_key = 0, v_stride_d = 0;
    uint64_t m_stride_key = 0, o_stride_d = 0;
    uint64_t rows = 0, keys = 0, depth = 0, value_depth = 0, group_size = 1;
    float scale = 1.0f;
    bool causal = false;
    int32_t causal_offset = 0;
};
int launch_attention_simt(const AttnArgs& a, void* stream);
// Split-key attention for at most 64 query rows per head over >= 512 keys;
// FB_ERR_UNSUPPORTED for other shapes.
int launch_attention_decode(const AttnArgs& a, void* stream);
int launch_attention_tc(const AttnArgs& a, void* stream);

}  // namespace fb
