// The extern "C" entry points declared in include/forma_b200.h.
//
// Each entry point follows the shape of the compute-cuda trait impl it
// replaces: validate descriptors and plan (same error classes and order as
// the reference), take the reference's empty/singleton shortcuts, then
// canonicalise strided layouts into index nests and enqueue the kernels on
// the caller's stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "host.h"
#include "kernels.h"

namespace fb {
const char* last_error_cstr();

namespace {

std::atomic<uint64_t> g_launches{0};
thread_local std::string g_driver_error;
// Kernels enqueued by the current (or most recent) entry-point call of this
// host thread, ';'-separated in launch order.
thread_local std::string g_route;
thread_local uint64_t g_thread_launches = 0;

struct ScratchBlock {
    void* ptr = nullptr;
    uint64_t bytes = 0;
};
std::mutex g_scratch_mutex;
std::map<std::tuple<int, void*, int>, ScratchBlock> g_scratch;

#define FB_TRY(expr)                                          \
    do {                                                      \
        ::fb::Error _e = (expr);                              \
        if (_e.status != FB_OK) return fail(_e.status, _e.detail); \
    } while (0)

int launched(int status, const char* what) {
    if (status == FB_OK) return FB_OK;
    if (status == FB_ERR_DRIVER) {
        cudaError_t e = cudaGetLastError();
        std::string detail = g_driver_error.empty() ? std::string(cudaGetErrorString(e)) : g_driver_error;
        g_driver_error.clear();
        return fail(status, std::string(what) + ": " + detail);
    }
    return fail(status, what);
}

// Builds an index nest over `axes` (in the given order) of a strided view:
// unit axes are dropped and adjacent axes whose strides nest row-major are
// merged, which preserves the row-major linearisation of the coordinates.
Nest make_nest(const Dims& dims, const Dims& strides, const std::vector<uint32_t>& axes) {
    std::vector<std::pair<uint64_t, uint64_t>> list;  // (dim, stride)
    for (uint32_t a : axes) {
        if (dims[a] == 1) continue;
        if (!list.empty() && list.back().second == strides[a] * dims[a]) {
            list.back().first *= dims[a];
            list.back().second = strides[a];
        } else {
            list.push_back({dims[a], strides[a]});
        }
    }
    Nest n;
    n.rank = (uint32_t)list.size();
    for (size_t i = 0; i < list.size(); ++i) {
        n.dims[i] = list[i].first;
        n.strides[i] = list[i].second;
    }
    return n;
}

std::vector<uint32_t> all_axes(size_t rank) {
    std::vector<uint32_t> v(rank);
    for (size_t i = 0; i < rank; ++i) v[i] = (uint32_t)i;
    return v;
}

// Splits a view into rows (kept axes) x columns (contracted axes).
Rows make_rows(const View& v, const std::vector<uint32_t>& axes) {
    std::vector<uint32_t> kept, red(axes.begin(), axes.end());
    std::sort(red.begin(), red.end());
    for (uint32_t i = 0; i < v.dims.size(); ++i)
        if (std::find(red.begin(), red.end(), i) == red.end()) kept.push_back(i);
    Rows r;
    r.data = v.data;
    r.dtype = v.dtype;
    r.offset = v.offset;
    r.outer = make_nest(v.dims, v.strides, kept);
    r.inner = make_nest(v.dims, v.strides, red);
    r.rows = 1;
    for (uint32_t a : kept) r.rows *= v.dims[a];
    r.cols = 1;
    for (uint32_t a : red) r.cols *= v.dims[a];
    const bool inner_unit = r.inner.rank == 0 || (r.inner.rank == 1 && r.inner.strides[0] == 1);
    r.contiguous_rows = inner_unit && r.outer.rank <= 1;
    r.row_stride = r.outer.rank == 1 ? r.outer.strides[0] : 0;
    return r;
}

RowOut make_row_out(const View& o) {
    RowOut out;
    out.data = o.data;
    out.offset = o.offset;
    out.nest = make_nest(o.dims, o.strides, all_axes(o.dims.size()));
    out.contiguous = out.nest.rank == 0 || (out.nest.rank == 1 && out.nest.strides[0] == 1);
    return out;
}

ElemOut make_elem_out(const View& o, const std::vector<uint32_t>& axes) {
    Rows r = make_rows(o, axes);
    ElemOut e;
    e.data = static_cast<float*>(o.data);
    e.offset = o.offset;
    e.outer = r.outer;
    e.inner = r.inner;
    e.contiguous_rows = r.contiguous_rows;
    e.row_stride = r.row_stride;
    return e;
}

int copy_view(const View& in, const View& out, void* stream) {
    Nest a = make_nest(in.dims, in.strides, all_axes(in.dims.size()));
    Nest b = make_nest(out.dims, out.strides, all_axes(out.dims.size()));
    return launched(launch_copy(in.data, (uint32_t)dtype_size(in.dtype), in.offset, a, out.data, out.offset, b,
                                in.count, stream),
                    "copy");
}

// Fills a dense-permuted output: its storage block starts at `offset`.
int fill_view(const View& out, uint32_t bits, void* stream) {
    return launched(launch_fill(static_cast<char*>(out.data) + out.offset * 4, out.count, bits, stream), "fill");
}

std::vector<uint32_t> axes_vec(const uint32_t* axes, uint32_t n) {
    if (!axes || n == 0) return {};
    return std::vector<uint32_t>(axes, axes + n);
}

uint32_t f32_bits(float f) {
    uint32_t b;
    std::memcpy(&b, &f, 4);
    return b;
}

// ------------------------------------------------------------ reductions

int reduce_impl(uint32_t op, const fb_tensor* input, const uint32_t* axes_p, uint32_t n_axes, int32_t keep,
                fb_tensor* output, void* stream, uint32_t want_dtype, bool mean) {
    View in, out;
    FB_TRY(view_of(input, "input", &in));
    if (in.dtype != want_dtype) return fail(FB_ERR_DTYPE, "reduction input dtype mismatch");
    std::vector<uint32_t> axes = axes_vec(axes_p, n_axes);
    Dims shape;
    FB_TRY(reduction_shape(mean ? FB_REDUCE_SUM : op, in.dims, axes, keep != 0, mean, &shape));
    FB_TRY(check_output(output, "output", shape, want_dtype, &out));
    if (axes.empty()) return copy_view(in, out, stream);  // identity (materialize)
    if (out.count == 0) return FB_OK;
    if (in.count == 0) {
        // Empty contraction with a nonempty output: sum 0, product 1.
        const uint32_t one = want_dtype == FB_F32 ? f32_bits(1.0f) : 1u;
        return fill_view(out, op == FB_REDUCE_PRODUCT && !mean ? one : 0u, stream);
    }
    Rows rows = make_rows(in, axes);
    RowOut ro = make_row_out(out);
    return launched(launch_reduce_rows(mean ? ROW_MEAN : op, rows, ro, stream), "reduce");
}

// ------------------------------------------------------------ statistics

int normalize_impl(uint32_t op, const fb_tensor* input, const uint32_t* axes_p, uint32_t n_axes, float eps,
                   fb_tensor* output, void* stream) {
    View in, out;
    FB_TRY(view_of(input, "input", &in));
    if (in.dtype != FB_F32 && !is_low(in.dtype)) return fail(FB_ERR_DTYPE, "statistics input must be f32, f16 or bf16");
    std::vector<uint32_t> axes = axes_vec(axes_p, n_axes);
    FB_TRY(validate_axes(in.dims, axes));  // normalization_shape
    if (op == STATS_LAYER_NORM && (!std::isfinite(eps) || eps <= 0.0f))
        return fail(FB_ERR_INVALID_EPSILON, "normalization epsilon must be finite and strictly positive");
    // An output of the input's 16-bit dtype is the reference's `_low` form
    // (the f32 result cast once to low storage: low_statistics.rs:59-108).
    // An f32 input may also take a 16-bit output (same single rounding; for
    // programs that feed the result to a low-precision contraction).
    const bool low_out = output && is_low(output->dtype) && (output->dtype == in.dtype || in.dtype == FB_F32);
    FB_TRY(check_output(output, "output", in.dims, low_out ? output->dtype : FB_F32, &out));
    if (low_out && !is_contiguous(out)) return fail(FB_ERR_INVALID_INPUT, "low statistics output must be contiguous");
    if (in.count == 0) return FB_OK;
    Dims reduced;
    FB_TRY(reduce_dims(in.dims, axes, false, &reduced));
    uint64_t rows;
    FB_TRY(numel(reduced, &rows));
    Rows r = make_rows(in, axes);
    RowOut none;
    if (low_out && rows != in.count) {
        // rounded in the streamed row engine's store when it takes the rows
        ElemOut e = make_elem_out(out, axes);
        e.dtype = out.dtype;
        const int st = launch_stats_rows(op, r, e, none, none, eps, stream);
        if (st != FB_ERR_UNSUPPORTED) return launched(st, "statistics");
    }
    // f32 result: the output itself, or scratch before the low rounding
    View res = out;
    if (low_out) {
        float* buf = static_cast<float*>(scratch(stream, out.count * 4 + 256, SCRATCH_STATS));
        if (!buf) return fail(FB_ERR_DRIVER, "scratch allocation failed");
        res.data = buf;
        res.offset = 0;
        res.dtype = FB_F32;  // contiguous, like `out`
    }
    int st;
    if (rows == in.count) {
        // Singleton groups: softmax 1, log-softmax and layer norm 0
        // (compute-cuda/src/statistics.rs:104-126).
        st = fill_view(res, op == STATS_SOFTMAX ? f32_bits(1.0f) : 0u, stream);
    } else {
        ElemOut e = make_elem_out(res, axes);
        st = launched(launch_stats_rows(op, r, e, none, none, eps, stream), "statistics");
    }
    if (st != FB_OK || !low_out) return st;
    Nest rn = make_nest(res.dims, res.strides, all_axes(res.dims.size()));
    return launched(launch_cast_to_low(static_cast<float*>(res.data), 0, rn,
                                       static_cast<uint16_t*>(out.data) + out.offset, out.dtype, out.count, stream),
                    "cast");
}

int row_stats_impl(uint32_t op, const fb_tensor* input, const uint32_t* axes_p, uint32_t n_axes, int32_t keep,
                   fb_tensor* out_a, fb_tensor* out_b, void* stream) {
    View in, a, b;
    FB_TRY(view_of(input, "input", &in));
    if (in.dtype != FB_F32 && !is_low(in.dtype)) return fail(FB_ERR_DTYPE, "statistics input must be f32, f16 or bf16");
    std::vector<uint32_t> axes = axes_vec(axes_p, n_axes);
    Dims shape;
    FB_TRY(reduction_shape(FB_REDUCE_SUM, in.dims, axes, keep != 0, true, &shape));  // statistics_shape
    FB_TRY(check_output(out_a, op == STATS_MOMENTS ? "mean" : "output", shape, FB_F32, &a));
    if (op == STATS_MOMENTS) FB_TRY(check_output(out_b, "variance", shape, FB_F32, &b));
    if (a.count == 0) return FB_OK;
    if (a.count == in.count) {
        // Singleton groups preserve the input exactly (reshape in the
        // reference); the variance is zero.  Low inputs are widened exactly.
        if (in.dtype == FB_F32) {
            int s = copy_view(in, a, stream);
            if (s != FB_OK) return s;
        } else {
            // Widen low storage exactly: the max of a one-element group is
            // the element itself, bit for bit.
            Rows rr = make_rows(in, {});
            RowOut ro = make_row_out(a);
            int s = launched(launch_reduce_rows(ROW_MAX, rr, ro, stream), "widen");
            if (s != FB_OK) return s;
        }
        return op == STATS_MOMENTS ? fill_view(b, 0u, stream) : FB_OK;
    }
    Rows r = make_rows(in, axes);
    RowOut ra = make_row_out(a);
    RowOut rb = op == STATS_MOMENTS ? make_row_out(b) : RowOut{};
    ElemOut none;
    return launched(launch_stats_rows(op, r, none, ra, rb, 0.0f, stream), "statistics");
}

// ------------------------------------------------------------ convolution

// Launch arguments of a convolution: input/weight views, the output (or f32
// result) view and the plan's geometry.
ConvArgs conv_args(const View& in, const View& w, const View& res, const ConvPlan& plan) {
    ConvArgs a;
    a.input = in.data;
    a.weight = w.data;
    a.output = static_cast<float*>(res.data);
    a.dtype = in.dtype;
    a.spatial = plan.spatial_rank;
    a.in_offset = in.offset;
    a.w_offset = w.offset;
    a.out_offset = res.offset;
    a.batch = plan.output[0];
    a.channels_per_group = plan.channels_per_group;
    a.outputs_per_group = plan.outputs_per_group;
    a.out_channels = plan.output[1];
    a.in_stride_n = in.strides[0];
    a.in_stride_c = in.strides[1];
    a.w_stride_o = w.strides[0];
    a.w_stride_c = w.strides[1];
    a.out_stride_n = res.strides[0];
    a.out_stride_c = res.strides[1];
    a.out_count = res.count;
    for (uint32_t d = 0; d < plan.spatial_rank; ++d) {
        a.in_dims[d] = in.dims[d + 2];
        a.out_dims[d] = plan.output[d + 2];
        a.k_dims[d] = w.dims[d + 2];
        a.in_strides[d] = in.strides[d + 2];
        a.w_strides[d] = w.strides[d + 2];
        a.out_strides[d] = res.strides[d + 2];
        a.stride[d] = plan.strides[d];
        a.dilation[d] = plan.dilations[d];
        a.pad[d] = plan.pad_before[d];
    }
    return a;
}

// True when the view's elements fill a dense block in some axis order (a
// contiguous tensor or a permuted view of one, e.g. channels-last).
bool dense_permutation(const View& v) {
    std::vector<std::pair<uint64_t, uint64_t>> ax;
    for (size_t i = 0; i < v.dims.size(); ++i)
        if (v.dims[i] > 1) ax.push_back({v.strides[i], v.dims[i]});
    std::sort(ax.begin(), ax.end());
    uint64_t expect = 1;
    for (auto& e : ax) {
        if (e.first != expect) return false;
        expect *= e.second;
    }
    return true;
}

// Epilogues of the glue entry points: none, GELU before the low rounding
// (fb_conv_low_gelu), or accumulation into the f32 output
// (fb_conv_low_f32_accumulate).
enum ConvEpilogue : uint32_t { CONV_EPI_NONE = 0, CONV_EPI_GELU = 1, CONV_EPI_ACCUMULATE = 2 };

int conv_impl(const fb_tensor* input, const fb_tensor* weight, const fb_conv_options* options, fb_tensor* output,
              void* stream, bool low, bool round_low, uint32_t epi = CONV_EPI_NONE) {
    View in, w, out;
    FB_TRY(view_of(input, "input", &in));
    FB_TRY(view_of(weight, "weight", &w));
    if (low) {
        if (!is_low(in.dtype) || !is_low(w.dtype)) return fail(FB_ERR_DTYPE, "low convolution needs f16/bf16 operands");
        if (in.dtype != w.dtype)
            return fail(FB_ERR_LOW_DTYPE_MISMATCH, "low-precision dtypes must match");  // check_low_dtypes first
    } else if (in.dtype != FB_F32 || w.dtype != FB_F32) {
        return fail(FB_ERR_DTYPE, "convolution needs f32 operands");
    }
    ConvPlan plan;
    FB_TRY(conv_plan(in.dims, w.dims, options, &plan));
    const uint32_t out_dtype = round_low ? in.dtype : FB_F32;
    FB_TRY(check_output(output, "output", plan.output, out_dtype, &out));
    if (out.count == 0) return FB_OK;
    // The reference bounds active coordinates to u32 (compute-cuda/src/
    // convolution.rs:108-143).
    for (auto d : in.dims)
        if (d > 0xffffffffull) return fail(FB_ERR_INVALID_INPUT, "CUDA convolution coordinate exceeds u32");
    for (auto d : w.dims)
        if (d > 0xffffffffull) return fail(FB_ERR_INVALID_INPUT, "CUDA convolution coordinate exceeds u32");
    for (auto d : plan.output)
        if (d > 0xffffffffull) return fail(FB_ERR_INVALID_INPUT, "CUDA convolution coordinate exceeds u32");
    for (uint32_t d = 0; d < plan.spatial_rank; ++d)
        for (uint64_t v : {plan.strides[d], plan.dilations[d], plan.pad_before[d], plan.pad_after[d]})
            if (v > 0xffffffffull) return fail(FB_ERR_INVALID_INPUT, "CUDA convolution coordinate exceeds u32");

    // conv_low on the tensor-core path rounds in the GEMM epilogue and writes
    // the 16-bit output directly (the GELU and accumulate epilogues likewise
    // act on the f32 sums there); every other path computes an f32 result
    // (in scratch for conv_low and the epilogues) and finishes it in a
    // separate pass.
    if (epi == CONV_EPI_ACCUMULATE) {
        // The output is read and written while the input and weights are
        // still being read: it may not share memory with either.
        auto span = [](const View& v, uint64_t esz) {
            uint64_t hi = v.offset;
            for (size_t i = 0; i < v.dims.size(); ++i) hi += (v.dims[i] - 1) * v.strides[i];
            const uintptr_t base = reinterpret_cast<uintptr_t>(v.data);
            return std::make_pair(base + v.offset * esz, base + (hi + 1) * esz);
        };
        const auto o = span(out, 4), x = span(in, 2), k = span(w, 2);
        auto meet = [&](std::pair<uintptr_t, uintptr_t> a) { return a.first < o.second && o.first < a.second; };
        if (out.count > 0 && ((in.count > 0 && meet(x)) || (w.count > 0 && meet(k))))
            return fail(FB_ERR_INVALID_INPUT, "accumulated output overlaps the convolution's input or weight");
    }
    const bool via_scratch = round_low || epi == CONV_EPI_ACCUMULATE;
    if (via_scratch && in.count > 0 && plan.channels_per_group > 0) {
        ConvArgs d = conv_args(in, w, out, plan);
        d.output = static_cast<float*>(out.data);
        d.out_low = round_low ? out.dtype : 0;
        d.act = epi == CONV_EPI_GELU ? 1 : 0;
        d.accumulate = epi == CONV_EPI_ACCUMULATE ? 1 : 0;
        const int st = launch_conv_tc(d, stream);
        if (st != FB_ERR_UNSUPPORTED) return launched(st, "convolution");
    }
    if (epi == CONV_EPI_ACCUMULATE && (in.count == 0 || plan.channels_per_group == 0)) return FB_OK;  // adds zeros
    // f32 result buffer: the output itself, or scratch before the finishing
    // pass.  The scratch copy takes the output's own memory order when that
    // is a dense block (contiguous or permuted, e.g. channels-last), so the
    // finishing pass maps memory position to memory position.
    float* result = nullptr;
    View res = out;
    const bool out_dense = dense_permutation(out);
    if (round_low && !out_dense) return fail(FB_ERR_INVALID_INPUT, "low convolution output must be a dense block");
    if (via_scratch) {
        result = static_cast<float*>(scratch(stream, out.count * 4 + 256, SCRATCH_CONV_RESULT));
        if (!result) return fail(FB_ERR_DRIVER, "scratch allocation failed");
        res.data = result;
        res.offset = 0;
        res.dtype = FB_F32;
        if (out_dense) {
            res.strides = out.strides;
        } else {
            res.strides.assign(res.dims.size(), 0);
            uint64_t s = 1;
            for (size_t i = res.dims.size(); i-- > 0;) {
                res.strides[i] = s;
                s *= res.dims[i];
            }
        }
    }
    if (in.count == 0 || plan.channels_per_group == 0) {
        // No input values: every window sums nothing (zeros).
        if (!round_low) return fill_view(res, 0u, stream);
        int s = fill_view(res, 0u, stream);
        if (s != FB_OK) return s;
    } else {
        ConvArgs a = conv_args(in, w, res, plan);
        int s = FB_ERR_UNSUPPORTED;
        if (!low) s = launch_conv2d_f32_tiled(a, stream);
        if (low) s = launch_conv_tc(a, stream);
        if (s == FB_ERR_UNSUPPORTED) s = launch_conv_direct(a, stream);
        s = launched(s, "convolution");
        if (s != FB_OK) return s;
    }
    if (epi == CONV_EPI_ACCUMULATE) {
        // output += result (the output is its own first operand)
        float* o = static_cast<float*>(out.data);
        Nest on = make_nest(out.dims, out.strides, all_axes(out.dims.size()));
        Nest rn = make_nest(res.dims, res.strides, all_axes(res.dims.size()));
        const bool dense = is_contiguous(out) && out.count % 4 == 0 && reinterpret_cast<uintptr_t>(o + out.offset) % 16 == 0 &&
                           reinterpret_cast<uintptr_t>(result) % 16 == 0;
        return launched(launch_add(o, out.offset, on, result, 0, rn, o, out.offset, on, out.count, dense, stream), "add");
    }
    if (round_low) {
        // scratch and output share one memory order: a dense position-wise pass
        Nest flat = make_nest(Dims{out.count}, Dims{1}, all_axes(1));
        if (epi == CONV_EPI_GELU)
            return launched(launch_gelu_to_low(result, 0, flat, static_cast<uint16_t*>(out.data) + out.offset, out.dtype,
                                               out.count, stream),
                            "gelu");
        return launched(launch_cast_to_low(result, 0, flat, static_cast<uint16_t*>(out.data) + out.offset, out.dtype,
                                           out.count, stream),
                        "cast");
    }
    return FB_OK;
}

// ------------------------------------------------------------ attention

int attention_impl(const fb_tensor* q, const fb_tensor* k, const fb_tensor* v, uint32_t mask_kind,
                   const fb_tensor* mask, fb_attention_options options, fb_tensor* output, void* stream, bool low,
                   bool round_low = false) {
    View qv, kv, vv, mv, out;
    FB_TRY(view_of(q, "query", &qv));
    FB_TRY(view_of(k, "key", &kv));
    FB_TRY(view_of(v, "value", &vv));
    if (low) {
        if (!is_low(qv.dtype) || !is_low(kv.dtype) || !is_low(vv.dtype))
            return fail(FB_ERR_DTYPE, "low attention needs f16/bf16 operands");
        if (qv.dtype != kv.dtype || qv.dtype != vv.dtype)
            return fail(FB_ERR_LOW_DTYPE_MISMATCH, "low-precision dtypes must match");
    } else if (qv.dtype != FB_F32 || kv.dtype != FB_F32 || vv.dtype != FB_F32) {
        return fail(FB_ERR_DTYPE, "attention needs f32 operands");
    }
    if (mask_kind > FB_MASK_ADDITIVE) return fail(FB_ERR_INVALID_INPUT, "unknown attention mask kind");
    const Dims* mask_dims = nullptr;
    if (mask_kind != FB_MASK_NONE) {
        FB_TRY(view_of(mask, "mask", &mv));
        if (mv.dtype != (mask_kind == FB_MASK_KEEP ? (uint32_t)FB_U32 : (uint32_t)FB_F32))
            return fail(FB_ERR_DTYPE, "attention mask dtype mismatch");
        mask_dims = &mv.dims;
    }
    AttentionPlan plan;
    FB_TRY(attention_plan(qv.dims, kv.dims, vv.dims, mask_dims, options, &plan));
    FB_TRY(check_output(output, "output", plan.output, round_low ? qv.dtype : (uint32_t)FB_F32, &out));
    if (out.count == 0) return FB_OK;
    // attention_low (compute-cuda/src/program/builder_attention.rs:29-42):
    // the f32 attention rounded once to the operands' 16-bit type.  The
    // tensor-core kernel rounds in its epilogue; the other kernels compute
    // f32 rows into scratch laid out in the output's own memory order, and
    // a position-wise cast finishes them.
    View res = out;
    if (round_low) {  // check_output admits dense blocks only: scratch offsets 0..count-1
        float* result = static_cast<float*>(scratch(stream, out.count * 4 + 256, SCRATCH_ATTN_RESULT));
        if (!result) return fail(FB_ERR_DRIVER, "scratch allocation failed");
        res.data = result;
        res.offset = 0;
        res.dtype = FB_F32;
    }
    auto finish = [&](int st) {
        if (st != FB_OK || !round_low) return st;
        Nest flat = make_nest(Dims{out.count}, Dims{1}, all_axes(1));
        return launched(launch_cast_to_low(static_cast<const float*>(res.data), 0, flat,
                                           static_cast<uint16_t*>(out.data) + out.offset, out.dtype, out.count, stream),
                        "cast");
    };
    if (plan.keys == 0) return finish(fill_view(res, 0u, stream));

    // Canonical layouts (compute-cuda/src/attention_dispatch.rs:9-18): rank-2
    // operands gain a zero-stride head axis, batches broadcast with stride 0.
    auto canonical = [&](const View& t, const Dims& promoted) {
        Dims strides = t.strides;
        if (t.dims.size() == 2) strides.insert(strides.begin(), 0);
        const size_t lead = plan.batch.size() + 3 - promoted.size();
        Dims s(plan.batch.size() + 3, 0);
        for (size_t i = 0; i < promoted.size(); ++i)
            s[lead + i] = promoted[i] == 1 && i < promoted.size() - 3 ? 0 : strides[i];
        // Unit head/sequence/depth axes keep their stride: indices stay 0.
        return s;
    };
    Dims qs = canonical(qv, plan.query), ks = canonical(kv, plan.key), vs = canonical(vv, plan.value);
    const size_t r = plan.batch.size() + 3;
    AttnArgs a;
    a.q = qv.data;
    a.k = kv.data;
    a.v = vv.data;
    a.out = static_cast<float*>(out.data);
    a.out_low = round_low ? out.dtype : 0;
    a.dtype = qv.dtype;
    a.mask_kind = mask_kind;
    a.row_rank = (uint32_t)(r - 1);
    if (a.row_rank > FB_MAX_RANK) return fail(FB_ERR_INVALID_INPUT, "attention rank too large");
    // Output strides in canonical form (a rank-2 output has no head axis).
    Dims os(r, 0);
    if (out.dims.size() == 2) {
        os[r - 2] = out.strides[0];
        os[r - 1] = out.strides[1];
    } else {
        for (size_t i = 0; i < r; ++i) os[i] = out.strides[i];
    }
    Dims ms(r, 0);
    if (mask_kind != FB_MASK_NONE) {
        const size_t lead = r - mv.dims.size();
        for (size_t i = 0; i < mv.dims.size(); ++i) ms[lead + i] = mv.dims[i] == 1 ? 0 : mv.strides[i];
        a.mask = mv.data;
        a.m_offset = mv.offset;
    }
    for (size_t i = 0; i + 1 < r; ++i) {
        a.row_dims[i] = plan.canonical_output[i];
        a.q_row_strides[i] = qs[i];
        a.k_row_strides[i] = i == r - 2 ? 0 : ks[i];
        a.v_row_strides[i] = i == r - 2 ? 0 : vs[i];
        a.m_row_strides[i] = ms[i];
        a.o_row_strides[i] = os[i];
    }
    a.q_offset = qv.offset;
    a.k_offset = kv.offset;
    a.v_offset = vv.offset;
    a.o_offset = out.offset;
    a.q_stride_d = qs[r - 1];
    a.k_stride_key = ks[r - 2];
    a.k_stride_d = ks[r - 1];
    a.v_stride_key = vs[r - 2];
    a.v_stride_d = vs[r - 1];
    a.m_stride_key = ms[r - 1];
    a.o_stride_d = os[r - 1];
    a.rows = out.count / plan.value_depth;
    a.keys = plan.keys;
    a.depth = plan.depth;
    a.value_depth = plan.value_depth;
    a.group_size = plan.group_size;
    a.scale = plan.scale;
    a.causal = plan.causal;
    a.causal_offset = plan.causal_offset;
    // 16-bit operands: tensor cores when the layout allows (fastest for
    // decode shapes too); otherwise few query rows over long key ranges
    // split the keys across warps; everything else one warp per row.
    int s = low ? launch_attention_tc(a, stream) : FB_ERR_UNSUPPORTED;
    if (s != FB_ERR_UNSUPPORTED) return launched(s, "attention");
    if (round_low) {  // f32 rows into the scratch copy (same strides, offset 0)
        a.out = static_cast<float*>(res.data);
        a.out_low = 0;
        a.o_offset = 0;
    }
    s = launch_attention_decode(a, stream);
    if (s == FB_ERR_UNSUPPORTED) s = launch_attention_simt(a, stream);
    return finish(launched(s, "attention"));
}

// f64 sum of every element of an f32 view into the device double `partial`
// (zero for an empty view).
int sum_partial_of(const View& in, double* partial, void* stream) {
    if (in.count == 0) {
        if (cudaMemsetAsync(partial, 0, sizeof(double), static_cast<cudaStream_t>(stream)) != cudaSuccess)
            return fail(FB_ERR_DRIVER, "memset failed");
        return FB_OK;
    }
    Rows rows = make_rows(in, all_axes(in.dims.size()));
    return launched(launch_sum_partial(rows, partial, stream), "sum partial");
}

// MatmulPlan::new (tensor-core/src/shape.rs:148-192).
struct MatmulPlanH {
    Dims left, right;      // vector operands promoted to matrices
    Dims matrix_output;    // batch..., M, N
    Dims output;           // promoted axes removed again
    bool left_vector = false, right_vector = false;
};

Error matmul_plan(const Dims& left, const Dims& right, MatmulPlanH* p) {
    if (left.empty() || right.empty())
        return err(FB_ERR_MATMUL_RANK, "matmul operands need rank >= 1 (left rank " + std::to_string(left.size()) +
                                           ", right rank " + std::to_string(right.size()) + ")");
    p->left_vector = left.size() == 1;
    p->right_vector = right.size() == 1;
    p->left = p->left_vector ? Dims{1, left[0]} : left;
    p->right = p->right_vector ? Dims{right[0], 1} : right;
    const Dims& a = p->left;
    const Dims& b = p->right;
    if (a[a.size() - 1] != b[b.size() - 2])
        return err(FB_ERR_MATMUL_INNER_DIMENSION, "matmul inner dimensions differ: " + std::to_string(a[a.size() - 1]) +
                                                      " vs " + std::to_string(b[b.size() - 2]));
    Dims batch;
    Error e = broadcast_dims(Dims(a.begin(), a.end() - 2), Dims(b.begin(), b.end() - 2), &batch);
    if (!ok(e)) return e;
    p->matrix_output = batch;
    p->matrix_output.push_back(a[a.size() - 2]);
    p->matrix_output.push_back(b[b.size() - 1]);
    p->output = p->matrix_output;
    if (p->right_vector) p->output.pop_back();
    if (p->left_vector) p->output.erase(p->output.end() - (p->right_vector ? 1 : 2));
    uint64_t n;
    return numel(p->output, &n);
}

int matmul_impl(const fb_tensor* left, const fb_tensor* right, fb_tensor* output, void* stream, bool round_low) {
    View l, r, out;
    FB_TRY(view_of(left, "left", &l));
    FB_TRY(view_of(right, "right", &r));
    if (!is_low(l.dtype) || !is_low(r.dtype)) return fail(FB_ERR_DTYPE, "low GEMM operands must be f16 or bf16");
    if (l.dtype != r.dtype) return fail(FB_ERR_INVALID_INPUT, "low GEMM inputs must have the same dtype");
    MatmulPlanH plan;
    FB_TRY(matmul_plan(l.dims, r.dims, &plan));
    FB_TRY(check_output(output, "output", plan.output, round_low ? l.dtype : FB_F32, &out));
    if (out.count == 0) return FB_OK;
    // promoted operand strides (a promoted unit axis has stride 0)
    Dims ls = l.strides, rs = r.strides;
    if (plan.left_vector) ls.insert(ls.begin(), 0);
    if (plan.right_vector) rs.push_back(0);
    const Dims& ld = plan.left;
    const Dims& rd = plan.right;
    const size_t nb = plan.matrix_output.size() - 2;
    // output strides in matrix_output form (removed vector axes: stride 0)
    Dims os(plan.matrix_output.size(), 0);
    {
        size_t j = 0;
        for (size_t i = 0; i < nb; ++i) os[i] = out.strides[j++];
        os[nb] = plan.left_vector ? 0 : out.strides[j++];
        os[nb + 1] = plan.right_vector ? 0 : out.strides[j++];
    }
    GemmArgs g;
    g.a = l.data;
    g.b = r.data;
    g.out = out.data;
    g.dtype = l.dtype;
    g.out_low = round_low ? out.dtype : 0;
    g.M = ld[ld.size() - 2];
    g.K = ld[ld.size() - 1];
    g.N = rd[rd.size() - 1];
    g.a_off = l.offset;
    g.b_off = r.offset;
    g.o_off = out.offset;
    g.a_sm = ls[ls.size() - 2];
    g.a_sk = ls[ls.size() - 1];
    g.b_sk = rs[rs.size() - 2];
    g.b_sn = rs[rs.size() - 1];
    g.o_sm = os[nb];
    g.o_sn = os[nb + 1];
    // batch nests over the broadcast batch axes, operands right-aligned
    Dims bdims(plan.matrix_output.begin(), plan.matrix_output.begin() + nb);
    auto batch_strides = [&](const Dims& d, const Dims& st) {
        Dims s(nb, 0);
        const size_t ob = d.size() - 2;
        for (size_t i = 0; i < nb; ++i) {
            if (i + ob < nb) continue;
            const size_t j = i + ob - nb;
            s[i] = d[j] == 1 ? 0 : st[j];
        }
        return s;
    };
    Dims ob(os.begin(), os.begin() + nb);
    g.a_batch = make_nest(bdims, batch_strides(ld, ls), all_axes(nb));
    g.b_batch = make_nest(bdims, batch_strides(rd, rs), all_axes(nb));
    g.o_batch = make_nest(bdims, ob, all_axes(nb));
    FB_TRY(numel(bdims, &g.batch));
    int st = launch_gemm_tc(g, stream);
    if (st == FB_ERR_UNSUPPORTED) st = launch_gemm_simt(g, stream);
    return launched(st, "matmul");
}

}  // namespace

// ------------------------------------------------------------ scratch

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

void count_launch(const char* kernel) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    ++g_thread_launches;
    if (!g_route.empty()) g_route += ';';
    g_route += kernel;
}

std::string kernel_name(const char* base, std::initializer_list<int> params) {
    std::string s(base);
    s += '<';
    bool first = true;
    for (int v : params) {
        if (!first) s += ',';
        s += std::to_string(v);
        first = false;
    }
    s += '>';
    return s;
}

void begin_route() { g_route.clear(); }

uint64_t thread_launch_count() { return g_thread_launches; }

int launch_status(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return FB_OK;
    g_driver_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
    return FB_ERR_DRIVER;
}

void* scratch(void* stream, uint64_t bytes, int slot) {
    int dev = 0;
    cudaGetDevice(&dev);
    // cudaStreamPerThread is one handle value naming a different stream in
    // every host thread: key its scratch by thread so that concurrent threads
    // never share a block.  (The legacy default stream is one stream for all
    // threads; its work is ordered, so sharing its block is safe.)
    static thread_local char per_thread_key;
    void* key = stream == static_cast<void*>(cudaStreamPerThread) ? static_cast<void*>(&per_thread_key) : stream;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    ScratchBlock& b = g_scratch[std::make_tuple(dev, key, slot)];
    if (b.bytes >= bytes) return b.ptr;
    // No allocation while the stream is being captured into a graph (it would
    // invalidate the capture): an eager call on the stream must come first.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &cap) == cudaSuccess &&
        cap != cudaStreamCaptureStatusNone) {
        g_driver_error = "library scratch must be allocated by an eager call on this stream before graph capture";
        return nullptr;
    }
    // Growing: the old block may still be read by enqueued work on this
    // stream, so it is kept (leaked) rather than freed under the stream.
    uint64_t want = std::max<uint64_t>(bytes, b.bytes * 2);
    void* p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) return nullptr;
    if (cudaMemsetAsync(p, 0, want, static_cast<cudaStream_t>(stream)) != cudaSuccess) return nullptr;
    b.ptr = p;
    b.bytes = want;
    return p;
}

}  // namespace fb

using namespace fb;

extern "C" {

int fb_abi_version(void) { return FB_ABI_VERSION; }

const char* fb_status_string(int status) {
    switch (status) {
        case FB_OK: return "ok";
        case FB_ERR_SHAPE_OVERFLOW: return "tensor element count overflows usize";
        case FB_ERR_LAYOUT_OVERFLOW: return "tensor storage address overflows usize";
        case FB_ERR_RANK_MISMATCH: return "rank mismatch";
        case FB_ERR_AXIS_OUT_OF_BOUNDS: return "axis out of bounds";
        case FB_ERR_DUPLICATE_AXIS: return "duplicate axis";
        case FB_ERR_INCOMPATIBLE_BROADCAST: return "incompatible broadcast";
        case FB_ERR_STORAGE_OUT_OF_BOUNDS: return "storage out of bounds";
        case FB_ERR_EMPTY_REDUCTION: return "min, max and mean require a nonempty contraction for each output";
        case FB_ERR_INVALID_EPSILON: return "normalization epsilon must be finite and strictly positive";
        case FB_ERR_INVALID_ATTENTION: return "invalid attention";
        case FB_ERR_INVALID_ATTENTION_SCALE: return "attention scale must be finite";
        case FB_ERR_INVALID_CONVOLUTION: return "invalid convolution";
        case FB_ERR_LOW_DTYPE_MISMATCH: return "low-precision dtypes must match";
        case FB_ERR_INVALID_INPUT: return "invalid input";
        case FB_ERR_MATMUL_RANK: return "matmul operands need rank >= 1";
        case FB_ERR_MATMUL_INNER_DIMENSION: return "matmul inner dimensions differ";
        case FB_ERR_DTYPE: return "tensor dtype mismatch";
        case FB_ERR_DRIVER: return "CUDA driver error";
        case FB_ERR_UNSUPPORTED: return "unsupported";
        case FB_ERR_FOREIGN_RUNTIME: return "tensor belongs to a different device";
        case FB_ERR_MISSING_SYMBOL: return "incompatible library: missing symbol";
        case FB_ERR_GRAPH: return "CUDA graph error";
        case FB_ERR_PROGRAM_POISONED: return "prepared program is poisoned after an execution error";
        default: return "unknown status";
    }
}

const char* fb_last_error(void) { return last_error_cstr(); }

uint64_t fb_launch_count(void) { return g_launches.load(); }

const char* fb_last_route(void) { return g_route.c_str(); }

uint32_t fb_device_status(void) {
    cudaDeviceSynchronize();
    return read_reduce_status() | read_gemm_status() | read_attention_status();
}

int fb_conv_plan(const uint64_t* input_dims, uint32_t input_rank, const uint64_t* weight_dims, uint32_t weight_rank,
                 const fb_conv_options* options, uint64_t* out_dims, uint32_t* out_rank) {
    if (input_rank > FB_MAX_RANK || weight_rank > FB_MAX_RANK || !out_dims || !out_rank)
        return fail(FB_ERR_INVALID_INPUT, "invalid plan arguments");
    ConvPlan plan;
    FB_TRY(conv_plan(Dims(input_dims, input_dims + input_rank), Dims(weight_dims, weight_dims + weight_rank), options,
                     &plan));
    *out_rank = (uint32_t)plan.output.size();
    std::copy(plan.output.begin(), plan.output.end(), out_dims);
    return FB_OK;
}

int fb_matmul_plan(const uint64_t* left_dims, uint32_t left_rank, const uint64_t* right_dims, uint32_t right_rank,
                   uint64_t* out_dims, uint32_t* out_rank) {
    if (left_rank > FB_MAX_RANK || right_rank > FB_MAX_RANK || !out_dims || !out_rank)
        return fail(FB_ERR_INVALID_INPUT, "invalid plan arguments");
    MatmulPlanH plan;
    FB_TRY(matmul_plan(Dims(left_dims, left_dims + left_rank), Dims(right_dims, right_dims + right_rank), &plan));
    if (plan.output.size() > FB_MAX_RANK) return fail(FB_ERR_INVALID_INPUT, "matmul output rank too large");
    *out_rank = (uint32_t)plan.output.size();
    std::copy(plan.output.begin(), plan.output.end(), out_dims);
    return FB_OK;
}

int fb_matmul_low_f32(const fb_tensor* left, const fb_tensor* right, fb_tensor* output, void* stream) {
    begin_route();
    return matmul_impl(left, right, output, stream, false);
}

int fb_matmul_low(const fb_tensor* left, const fb_tensor* right, fb_tensor* output, void* stream) {
    begin_route();
    return matmul_impl(left, right, output, stream, true);
}

int fb_conv(const fb_tensor* input, const fb_tensor* weight, const fb_conv_options* options, fb_tensor* output,
            void* stream) {
    begin_route();
    return conv_impl(input, weight, options, output, stream, false, false);
}

int fb_conv_low_f32(const fb_tensor* input, const fb_tensor* weight, const fb_conv_options* options, fb_tensor* output,
                    void* stream) {
    begin_route();
    return conv_impl(input, weight, options, output, stream, true, false);
}

int fb_conv_low(const fb_tensor* input, const fb_tensor* weight, const fb_conv_options* options, fb_tensor* output,
                void* stream) {
    begin_route();
    return conv_impl(input, weight, options, output, stream, true, true);
}

int fb_conv_low_gelu(const fb_tensor* input, const fb_tensor* weight, const fb_conv_options* options, fb_tensor* output,
                     void* stream) {
    begin_route();
    return conv_impl(input, weight, options, output, stream, true, true, CONV_EPI_GELU);
}

int fb_conv_low_f32_accumulate(const fb_tensor* input, const fb_tensor* weight, const fb_conv_options* options,
                               fb_tensor* output, void* stream) {
    begin_route();
    return conv_impl(input, weight, options, output, stream, true, false, CONV_EPI_ACCUMULATE);
}

int fb_attention_plan(const uint64_t* q_dims, uint32_t q_rank, const uint64_t* k_dims, uint32_t k_rank,
                      const uint64_t* v_dims, uint32_t v_rank, const uint64_t* mask_dims, uint32_t mask_rank,
                      fb_attention_options options, uint64_t* out_dims, uint32_t* out_rank) {
    if (q_rank > FB_MAX_RANK || k_rank > FB_MAX_RANK || v_rank > FB_MAX_RANK || mask_rank > FB_MAX_RANK || !out_dims ||
        !out_rank)
        return fail(FB_ERR_INVALID_INPUT, "invalid plan arguments");
    AttentionPlan plan;
    Dims m;
    if (mask_dims) m.assign(mask_dims, mask_dims + mask_rank);
    FB_TRY(attention_plan(Dims(q_dims, q_dims + q_rank), Dims(k_dims, k_dims + k_rank), Dims(v_dims, v_dims + v_rank),
                          mask_dims ? &m : nullptr, options, &plan));
    if (plan.output.size() > FB_MAX_RANK) return fail(FB_ERR_INVALID_INPUT, "attention output rank too large");
    *out_rank = (uint32_t)plan.output.size();
    std::copy(plan.output.begin(), plan.output.end(), out_dims);
    return FB_OK;
}

int fb_attention(const fb_tensor* query, const fb_tensor* key, const fb_tensor* value, uint32_t mask_kind,
                 const fb_tensor* mask, fb_attention_options options, fb_tensor* output, void* stream) {
    begin_route();
    return attention_impl(query, key, value, mask_kind, mask, options, output, stream, false);
}

int fb_attention_low_f32(const fb_tensor* query, const fb_tensor* key, const fb_tensor* value, uint32_t mask_kind,
                         const fb_tensor* mask, fb_attention_options options, fb_tensor* output, void* stream) {
    begin_route();
    return attention_impl(query, key, value, mask_kind, mask, options, output, stream, true);
}

int fb_attention_low(const fb_tensor* query, const fb_tensor* key, const fb_tensor* value, uint32_t mask_kind,
                     const fb_tensor* mask, fb_attention_options options, fb_tensor* output, void* stream) {
    begin_route();
    return attention_impl(query, key, value, mask_kind, mask, options, output, stream, true, true);
}

int fb_reduce_shape(uint32_t op, const uint64_t* dims, uint32_t rank, const uint32_t* axes, uint32_t n_axes,
                    int32_t keep_dims, int32_t is_mean, uint64_t* out_dims, uint32_t* out_rank) {
    if (rank > FB_MAX_RANK || !out_dims || !out_rank) return fail(FB_ERR_INVALID_INPUT, "invalid shape arguments");
    Dims out;
    FB_TRY(reduction_shape(op, Dims(dims, dims + rank), axes_vec(axes, n_axes), keep_dims != 0, is_mean != 0, &out));
    *out_rank = (uint32_t)out.size();
    std::copy(out.begin(), out.end(), out_dims);
    return FB_OK;
}

int fb_reduce_f32(uint32_t op, const fb_tensor* input, const uint32_t* axes, uint32_t n_axes, int32_t keep_dims,
                  fb_tensor* output, void* stream) {
    begin_route();
    return reduce_impl(op, input, axes, n_axes, keep_dims, output, stream, FB_F32, false);
}

int fb_reduce_u32(uint32_t op, const fb_tensor* input, const uint32_t* axes, uint32_t n_axes, int32_t keep_dims,
                  fb_tensor* output, void* stream) {
    begin_route();
    return reduce_impl(op, input, axes, n_axes, keep_dims, output, stream, FB_U32, false);
}

int fb_mean_axes(const fb_tensor* input, const uint32_t* axes, uint32_t n_axes, int32_t keep_dims, fb_tensor* output,
                 void* stream) {
    begin_route();
    return reduce_impl(FB_REDUCE_SUM, input, axes, n_axes, keep_dims, output, stream, FB_F32, true);
}

int fb_argmax(const fb_tensor* input, uint32_t axis, int32_t keep_dims, fb_tensor* output, void* stream) {
    begin_route();
    View in, out;
    FB_TRY(view_of(input, "input", &in));
    if (in.dtype != FB_F32) return fail(FB_ERR_DTYPE, "argmax input must be f32");
    std::vector<uint32_t> axes{axis};
    Dims shape;
    FB_TRY(reduction_shape(FB_REDUCE_MAX, in.dims, axes, keep_dims != 0, false, &shape));
    FB_TRY(check_output(output, "output", shape, FB_U32, &out));
    if (out.count == 0) return FB_OK;
    if (in.dims[axis] > 0xffffffffull) return fail(FB_ERR_INVALID_INPUT, "argmax axis exceeds u32 indices");
    Rows rows = make_rows(in, axes);
    RowOut ro = make_row_out(out);
    return launched(launch_reduce_rows(ROW_ARGMAX, rows, ro, stream), "argmax");
}

int fb_sum_partial_f64(const fb_tensor* input, double* partial, void* stream) {
    begin_route();
    View in;
    FB_TRY(view_of(input, "input", &in));
    if (in.dtype != FB_F32) return fail(FB_ERR_DTYPE, "global sum input must be f32");
    if (!partial) return fail(FB_ERR_INVALID_INPUT, "null partial pointer");
    return sum_partial_of(in, partial, stream);
}

int fb_global_sum_nccl(const fb_tensor* shard, void* comm, fb_tensor* output, void* stream) {
    begin_route();
    View in, out;
    FB_TRY(view_of(shard, "shard", &in));
    if (in.dtype != FB_F32) return fail(FB_ERR_DTYPE, "global sum input must be f32");
    FB_TRY(view_of(output, "output", &out));
    if (out.dtype != FB_F32 || out.count != 1) return fail(FB_ERR_INVALID_INPUT, "global sum output must be one f32");
    if (!comm) return fail(FB_ERR_INVALID_INPUT, "null communicator");
    double* partial = static_cast<double*>(scratch(stream, 256, SCRATCH_COLLECTIVE));
    if (!partial) return fail(FB_ERR_DRIVER, "scratch allocation failed");
    if (int rc = sum_partial_of(in, partial, stream); rc != FB_OK) return rc;
    if (int rc = nccl_all_reduce_sum_f64(partial, 1, comm, stream); rc != FB_OK) return rc;
    return launched(launch_finish_sum(partial, static_cast<float*>(out.data) + out.offset, stream), "finish sum");
}

int fb_sum_partial_f64_static(const fb_tensor* input, double* partial, void* stream) {
    begin_route();
    View in;
    FB_TRY(view_of(input, "input", &in));
    if (in.dtype != FB_F32) return fail(FB_ERR_DTYPE, "global sum input must be f32");
    if (!partial) return fail(FB_ERR_INVALID_INPUT, "null partial pointer");
    if (in.count > static_sum_max_elements())
        return fail(FB_ERR_INVALID_INPUT, "input has " + std::to_string(in.count) +
                                              " elements; the static-scratch global sum accepts at most " +
                                              std::to_string(static_sum_max_elements()));
    Rows rows = make_rows(in, all_axes(in.dims.size()));
    if (in.count == 0) {
        if (cudaMemsetAsync(partial, 0, sizeof(double), static_cast<cudaStream_t>(stream)) != cudaSuccess)
            return fail(FB_ERR_DRIVER, "memset failed");
        return FB_OK;
    }
    return launched(launch_sum_partial_static(rows, partial, stream), "static-scratch sum partial");
}

uint64_t fb_sum_static_max_elements(void) { return static_sum_max_elements(); }

int fb_selftest_bounded_wait(uint64_t limit_ns, void* stream) {
    begin_route();
    if (limit_ns == 0 || limit_ns > 1000000000ull)
        return fail(FB_ERR_INVALID_INPUT, "self-test wait limit must be in (0, 1e9] nanoseconds");
    return launched(launch_selftest_wait(limit_ns, stream), "self-test wait");
}

int fb_finish_sum_f64(const double* partial, fb_tensor* output, void* stream) {
    begin_route();
    View out;
    FB_TRY(view_of(output, "output", &out));
    if (out.dtype != FB_F32 || out.count != 1) return fail(FB_ERR_INVALID_INPUT, "global sum output must be one f32");
    if (!partial) return fail(FB_ERR_INVALID_INPUT, "null partial pointer");
    return launched(launch_finish_sum(partial, static_cast<float*>(out.data) + out.offset, stream), "finish sum");
}

int fb_softmax(const fb_tensor* input, const uint32_t* axes, uint32_t n_axes, fb_tensor* output, void* stream) {
    begin_route();
    return normalize_impl(STATS_SOFTMAX, input, axes, n_axes, 0.0f, output, stream);
}

int fb_log_softmax(const fb_tensor* input, const uint32_t* axes, uint32_t n_axes, fb_tensor* output, void* stream) {
    begin_route();
    return normalize_impl(STATS_LOG_SOFTMAX, input, axes, n_axes, 0.0f, output, stream);
}

int fb_layer_norm(const fb_tensor* input, const uint32_t* axes, uint32_t n_axes, float epsilon, fb_tensor* output,
                  void* stream) {
    begin_route();
    return normalize_impl(STATS_LAYER_NORM, input, axes, n_axes, epsilon, output, stream);
}

int fb_logsumexp(const fb_tensor* input, const uint32_t* axes, uint32_t n_axes, int32_t keep_dims, fb_tensor* output,
                 void* stream) {
    begin_route();
    return row_stats_impl(STATS_LOGSUMEXP, input, axes, n_axes, keep_dims, output, nullptr, stream);
}

int fb_moments(const fb_tensor* input, const uint32_t* axes, uint32_t n_axes, int32_t keep_dims, fb_tensor* mean,
               fb_tensor* variance, void* stream) {
    begin_route();
    return row_stats_impl(STATS_MOMENTS, input, axes, n_axes, keep_dims, mean, variance, stream);
}

int fb_cast_to_low(const fb_tensor* input, fb_tensor* output, void* stream) {
    begin_route();
    View in, out;
    FB_TRY(view_of(input, "input", &in));
    FB_TRY(view_of(output, "output", &out));
    if (in.dtype != FB_F32 || !is_low(out.dtype)) return fail(FB_ERR_DTYPE, "cast_to_low needs f32 -> f16/bf16");
    if (out.dims != in.dims) return fail(FB_ERR_INVALID_INPUT, "cast output dims differ from input");
    if (!is_contiguous(out)) return fail(FB_ERR_INVALID_INPUT, "cast output must be contiguous");
    Nest n = make_nest(in.dims, in.strides, all_axes(in.dims.size()));
    return launched(launch_cast_to_low(static_cast<const float*>(in.data), in.offset, n,
                                       static_cast<uint16_t*>(out.data) + out.offset, out.dtype, in.count, stream),
                    "cast");
}

int fb_add(const fb_tensor* a, const fb_tensor* b, fb_tensor* output, void* stream) {
    begin_route();
    View x, y, out;
    FB_TRY(view_of(a, "a", &x));
    FB_TRY(view_of(b, "b", &y));
    FB_TRY(view_of(output, "output", &out));
    if (x.dtype != FB_F32 || y.dtype != FB_F32 || out.dtype != FB_F32) return fail(FB_ERR_DTYPE, "add needs f32 operands");
    if (x.dims != out.dims || y.dims != out.dims) return fail(FB_ERR_INVALID_INPUT, "add operand dims differ from output");
    if (out.count == 0) return FB_OK;
    // The output may be any layout that gives every element its own address:
    // non-unit axes sorted by stride, each stride at least the extent of the
    // axes inside it.
    {
        std::vector<std::pair<uint64_t, uint64_t>> ax;
        for (size_t i = 0; i < out.dims.size(); ++i)
            if (out.dims[i] > 1) ax.push_back({out.strides[i], out.dims[i]});
        std::sort(ax.begin(), ax.end());
        uint64_t extent = 1;
        for (auto& e : ax) {
            if (e.first < extent) return fail(FB_ERR_INVALID_INPUT, "add output layout must address each element once");
            extent = e.first * e.second;
        }
    }
    // An operand may share memory with the output only as the identical view.
    auto same_view = [&](const View& v) {
        return v.data == out.data && v.offset == out.offset && v.strides == out.strides;
    };
    auto extent_of = [](const View& v) {
        uint64_t e = 1;
        for (size_t i = 0; i < v.dims.size(); ++i) e += (v.dims[i] - 1) * v.strides[i];
        return e;
    };
    const uint64_t out_lo = out.offset, out_hi = out.offset + extent_of(out);
    auto overlaps = [&](const View& v) {
        if (v.data != out.data || same_view(v)) return false;
        const uint64_t lo = v.offset, hi = v.offset + extent_of(v);
        return lo < out_hi && out_lo < hi;
    };
    if (overlaps(x) || overlaps(y)) return fail(FB_ERR_INVALID_INPUT, "add operand overlaps the output");
    const float* xa = static_cast<const float*>(x.data);
    const float* ya = static_cast<const float*>(y.data);
    float* o = static_cast<float*>(out.data);
    const bool dense = is_contiguous(x) && is_contiguous(y) && is_contiguous(out) && out.count % 4 == 0 &&
                       reinterpret_cast<uintptr_t>(xa + x.offset) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(ya + y.offset) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(o + out.offset) % 16 == 0;
    // One nest over the output's dims for all three views: unit axes
    // dropped, adjacent axes merged only where every view allows it, so the
    // kernel decomposes each index once for all three.
    Nest xn, yn, on;
    for (size_t i = 0; i < out.dims.size(); ++i) {
        if (out.dims[i] == 1) continue;
        const uint32_t r = on.rank;
        auto merges = [&](const Nest& n, uint64_t stride) { return n.strides[r - 1] == stride * out.dims[i]; };
        if (r > 0 && merges(xn, x.strides[i]) && merges(yn, y.strides[i]) && merges(on, out.strides[i])) {
            for (Nest* n : {&xn, &yn, &on}) n->dims[r - 1] *= out.dims[i];
            xn.strides[r - 1] = x.strides[i];
            yn.strides[r - 1] = y.strides[i];
            on.strides[r - 1] = out.strides[i];
        } else {
            for (Nest* n : {&xn, &yn, &on}) {
                n->dims[r] = out.dims[i];
                n->rank = r + 1;
            }
            xn.strides[r] = x.strides[i];
            yn.strides[r] = y.strides[i];
            on.strides[r] = out.strides[i];
        }
    }
    return launched(launch_add(xa, x.offset, xn, ya, y.offset, yn, o, out.offset, on, out.count, dense, stream), "add");
}

int fb_gelu_to_low(const fb_tensor* input, fb_tensor* output, void* stream) {
    begin_route();
    View in, out;
    FB_TRY(view_of(input, "input", &in));
    FB_TRY(view_of(output, "output", &out));
    if (in.dtype != FB_F32 || !is_low(out.dtype)) return fail(FB_ERR_DTYPE, "gelu_to_low needs f32 -> f16/bf16");
    if (out.dims != in.dims) return fail(FB_ERR_INVALID_INPUT, "gelu output dims differ from input");
    if (!is_contiguous(out)) return fail(FB_ERR_INVALID_INPUT, "gelu output must be contiguous");
    Nest n = make_nest(in.dims, in.strides, all_axes(in.dims.size()));
    return launched(launch_gelu_to_low(static_cast<const float*>(in.data), in.offset, n,
                                       static_cast<uint16_t*>(out.data) + out.offset, out.dtype, in.count, stream),
                    "gelu");
}

}  // extern "C"
