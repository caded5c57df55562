// Host validation and plans; see host.h for the reference functions restated.
#include "host.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>

namespace fb {

namespace {
thread_local std::string g_last_error;

bool mul_overflow(uint64_t a, uint64_t b, uint64_t* out) { return __builtin_mul_overflow(a, b, out); }
bool add_overflow(uint64_t a, uint64_t b, uint64_t* out) { return __builtin_add_overflow(a, b, out); }

std::string dims_str(const Dims& d) {
    std::string s = "[";
    for (size_t i = 0; i < d.size(); ++i) {
        if (i) s += ", ";
        s += std::to_string(d[i]);
    }
    return s + "]";
}
}  // namespace

const char* last_error_cstr() { return g_last_error.c_str(); }

int fail(int status, const std::string& detail) {
    g_last_error = detail;
    return status;
}

Error numel(const Dims& dims, uint64_t* out) {
    for (uint64_t d : dims)
        if (d == 0) {
            *out = 0;
            return {};
        }
    uint64_t n = 1;
    for (uint64_t d : dims)
        if (mul_overflow(n, d, &n)) return err(FB_ERR_SHAPE_OVERFLOW, "tensor element count overflows usize");
    *out = n;
    return {};
}

Error validate_axes(const Dims& dims, const std::vector<uint32_t>& axes) {
    std::vector<bool> seen(dims.size(), false);
    for (uint32_t a : axes) {
        if (a >= dims.size())
            return err(FB_ERR_AXIS_OUT_OF_BOUNDS,
                       "axis " + std::to_string(a) + " is outside tensor rank " + std::to_string(dims.size()));
        if (seen[a]) return err(FB_ERR_DUPLICATE_AXIS, "axis " + std::to_string(a) + " occurs more than once");
        seen[a] = true;
    }
    return {};
}

Error reduce_dims(const Dims& dims, const std::vector<uint32_t>& axes, bool keep, Dims* out) {
    Error e = validate_axes(dims, axes);
    if (!ok(e)) return e;
    out->clear();
    for (uint32_t i = 0; i < dims.size(); ++i) {
        bool reduced = false;
        for (uint32_t a : axes) reduced |= (a == i);
        if (reduced) {
            if (keep) out->push_back(1);
        } else {
            out->push_back(dims[i]);
        }
    }
    uint64_t n;
    return numel(*out, &n);
}

Error broadcast_dims(const Dims& left, const Dims& right, Dims* out) {
    size_t rank = std::max(left.size(), right.size());
    Dims result(rank);
    for (size_t axis = 0; axis < rank; ++axis) {
        uint64_t a = axis < rank - left.size() ? 1 : left[axis - (rank - left.size())];
        uint64_t b = axis < rank - right.size() ? 1 : right[axis - (rank - right.size())];
        if (a == b || b == 1)
            result[axis] = a;
        else if (a == 1)
            result[axis] = b;
        else
            return err(FB_ERR_INCOMPATIBLE_BROADCAST,
                       "cannot broadcast shapes " + dims_str(left) + " and " + dims_str(right));
    }
    *out = result;
    return {};
}

uint64_t dtype_size(uint32_t dtype) {
    switch (dtype) {
        case FB_F32:
        case FB_U32: return 4;
        case FB_F16:
        case FB_BF16: return 2;
        default: return 0;
    }
}

bool is_low(uint32_t dtype) { return dtype == FB_F16 || dtype == FB_BF16; }

Error view_of(const fb_tensor* t, const char* name, View* out) {
    if (!t) return err(FB_ERR_INVALID_INPUT, std::string(name) + ": null tensor descriptor");
    if (t->rank > FB_MAX_RANK)
        return err(FB_ERR_INVALID_INPUT, std::string(name) + ": rank exceeds " + std::to_string(FB_MAX_RANK));
    if (dtype_size(t->dtype) == 0) return err(FB_ERR_DTYPE, std::string(name) + ": unknown dtype");
    View v;
    v.dims.assign(t->dims, t->dims + t->rank);
    v.strides.assign(t->strides, t->strides + t->rank);
    v.offset = t->offset;
    v.storage_len = t->storage_len;
    v.dtype = t->dtype;
    v.data = t->data;
    Error e = numel(v.dims, &v.count);
    if (!ok(e)) return e;
    // Layout::required_storage_len: empty views need only `offset` elements.
    uint64_t required = v.offset;
    if (v.count != 0) {
        uint64_t end = v.offset;
        for (size_t i = 0; i < v.dims.size(); ++i) {
            uint64_t delta;
            if (mul_overflow(v.strides[i], v.dims[i] - 1, &delta) || add_overflow(end, delta, &end))
                return err(FB_ERR_LAYOUT_OVERFLOW, "tensor storage address overflows usize");
        }
        if (add_overflow(end, 1, &required)) return err(FB_ERR_LAYOUT_OVERFLOW, "tensor storage address overflows usize");
    }
    if (required > v.storage_len)
        return err(FB_ERR_STORAGE_OUT_OF_BOUNDS, std::string(name) + ": tensor layout needs " +
                                                     std::to_string(required) + " storage elements; available " +
                                                     std::to_string(v.storage_len));
    // validate_logical_size (compute-cuda/src/runtime.rs:354-364).
    uint64_t bytes;
    if (mul_overflow(std::max<uint64_t>(v.count, 1), dtype_size(v.dtype), &bytes))
        return err(FB_ERR_INVALID_INPUT, "CUDA tensor byte count overflows");
    if (v.count != 0 && v.data == nullptr)
        return err(FB_ERR_INVALID_INPUT, std::string(name) + ": null storage for a nonempty tensor");
    *out = v;
    return {};
}

bool is_contiguous(const View& v) {
    if (v.count == 0) return true;
    uint64_t expected = 1;
    for (size_t i = v.dims.size(); i-- > 0;) {
        if (v.dims[i] > 1 && v.strides[i] != expected) return false;
        expected *= v.dims[i];
    }
    return true;
}

Error check_output(const fb_tensor* t, const char* name, const Dims& dims, uint32_t dtype, View* out) {
    Error e = view_of(t, name, out);
    if (!ok(e)) return e;
    if (out->dtype != dtype) return err(FB_ERR_DTYPE, std::string(name) + ": output dtype mismatch");
    if (out->dims != dims)
        return err(FB_ERR_INVALID_INPUT,
                   std::string(name) + ": output dims " + dims_str(out->dims) + " differ from planned " + dims_str(dims));
    if (out->count == 0) return {};
    // Every element must have its own address: sorting the non-unit axes by
    // stride must give a dense nest (a permutation of a contiguous block).
    std::vector<std::pair<uint64_t, uint64_t>> axes;
    for (size_t i = 0; i < dims.size(); ++i)
        if (dims[i] > 1) axes.push_back({out->strides[i], dims[i]});
    std::sort(axes.begin(), axes.end());
    uint64_t expected = 1;
    for (auto& a : axes) {
        if (a.first != expected)
            return err(FB_ERR_INVALID_INPUT, std::string(name) + ": output layout must address each element once");
        expected *= a.second;
    }
    return {};
}

// ------------------------------------------------------------------ conv

Error conv_plan(const Dims& input, const Dims& weight, const fb_conv_options* o, ConvPlan* plan) {
    auto invalid = [](const char* m) { return err(FB_ERR_INVALID_CONVOLUTION, std::string("invalid convolution: ") + m); };
    if (!o) return err(FB_ERR_INVALID_INPUT, "null convolution options");
    if (input.size() < 3 || input.size() > 5 || weight.size() != input.size())
        return invalid("input and weight need equal rank, with one to three spatial axes");
    uint32_t spatial = (uint32_t)input.size() - 2;
    if (o->strides_len != spatial || o->dilations_len != spatial || o->padding_before_len != spatial ||
        o->padding_after_len != spatial)
        return invalid("every option vector must match the spatial rank");
    uint64_t channels = input[1], outputs = weight[0];
    if (o->groups == 0 || channels % o->groups != 0 || outputs % o->groups != 0)
        return invalid("groups must be positive and divide input and output channels");
    ConvPlan p;
    p.input = input;
    p.weight = weight;
    p.spatial_rank = spatial;
    p.groups = o->groups;
    p.channels_per_group = channels / o->groups;
    p.outputs_per_group = outputs / o->groups;
    if (weight[1] != p.channels_per_group)
        return invalid("weight input channels must equal input channels divided by groups");
    p.output = {input[0], outputs};
    for (uint32_t axis = 0; axis < spatial; ++axis) {
        uint64_t kernel = weight[axis + 2], stride = o->strides[axis], dilation = o->dilations[axis];
        if (kernel == 0 || stride == 0 || dilation == 0)
            return invalid("kernel extents, strides and dilations must be positive");
        uint64_t padded, effective;
        if (add_overflow(input[axis + 2], o->padding_before[axis], &padded) ||
            add_overflow(padded, o->padding_after[axis], &padded))
            return err(FB_ERR_SHAPE_OVERFLOW, "tensor element count overflows usize");
        if (mul_overflow(kernel - 1, dilation, &effective) || add_overflow(effective, 1, &effective))
            return err(FB_ERR_SHAPE_OVERFLOW, "tensor element count overflows usize");
        p.output.push_back(padded < effective ? 0 : (padded - effective) / stride + 1);
        p.strides[axis] = stride;
        p.dilations[axis] = dilation;
        p.pad_before[axis] = o->padding_before[axis];
        p.pad_after[axis] = o->padding_after[axis];
    }
    uint64_t n;
    Error e = numel(p.output, &n);
    if (!ok(e)) return e;
    *plan = p;
    return {};
}

// --------------------------------------------------------------- attention

Error attention_plan(const Dims& q0, const Dims& k0, const Dims& v0, const Dims* mask,
                     fb_attention_options options, AttentionPlan* plan) {
    auto invalid = [](const char* m) { return err(FB_ERR_INVALID_ATTENTION, std::string("invalid attention: ") + m); };
    bool matrices = q0.size() == 2 && k0.size() == 2 && v0.size() == 2;
    auto promote = [&](const Dims& d, Dims* out) -> Error {
        if (d.size() < 2) return invalid("operands need rank at least two");
        if (d.size() == 2)
            *out = {1, d[0], d[1]};
        else
            *out = d;
        uint64_t n;
        return numel(*out, &n);
    };
    AttentionPlan p;
    Error e;
    if (!ok(e = promote(q0, &p.query))) return e;
    if (!ok(e = promote(k0, &p.key))) return e;
    if (!ok(e = promote(v0, &p.value))) return e;
    const Dims &q = p.query, &k = p.key, &v = p.value;
    size_t qr = q.size(), kr = k.size(), vr = v.size();
    p.query_heads = q[qr - 3];
    p.queries = q[qr - 2];
    p.depth = q[qr - 1];
    p.key_heads = k[kr - 3];
    p.keys = k[kr - 2];
    uint64_t key_depth = k[kr - 1];
    uint64_t value_heads = v[vr - 3], value_keys = v[vr - 2];
    p.value_depth = v[vr - 1];
    if (p.depth == 0 || p.depth != key_depth) return invalid("query/key depths must be equal and positive");
    if (p.query_heads == 0 || p.key_heads == 0 || value_heads != p.key_heads)
        return invalid("head counts must be positive and key/value heads must match");
    if (p.query_heads % p.key_heads != 0) return invalid("query head count must be a multiple of key/value head count");
    if (p.keys != value_keys) return invalid("key and value sequence lengths must match");
    Dims batch;
    Dims qb(q.begin(), q.end() - 3), kb(k.begin(), k.end() - 3), vb(v.begin(), v.end() - 3);
    if (!ok(e = broadcast_dims(Dims{}, qb, &batch))) return e;
    if (!ok(e = broadcast_dims(batch, kb, &batch))) return e;
    if (!ok(e = broadcast_dims(batch, vb, &batch))) return e;
    uint64_t n;
    if (!ok(e = numel(batch, &n))) return e;
    p.batch = batch;
    p.scores = batch;
    p.scores.insert(p.scores.end(), {p.query_heads, p.queries, p.keys});
    if (!ok(e = numel(p.scores, &n))) return e;
    if (mask) {
        Dims b;
        if (!ok(e = broadcast_dims(*mask, p.scores, &b))) return e;
        if (b != p.scores)
            return err(FB_ERR_INCOMPATIBLE_BROADCAST,
                       "cannot broadcast shapes " + dims_str(*mask) + " and " + dims_str(p.scores));
    }
    p.canonical_output = batch;
    p.canonical_output.insert(p.canonical_output.end(), {p.query_heads, p.queries, p.value_depth});
    if (!ok(e = numel(p.canonical_output, &n))) return e;
    p.output = matrices ? Dims{p.queries, p.value_depth} : p.canonical_output;
    // Default (depth as f32).sqrt().recip(): correctly rounded f32 sqrt, then
    // a correctly rounded f32 reciprocal.
    p.scale = options.has_scale ? options.scale : 1.0f / std::sqrt((float)p.depth);
    if (!std::isfinite(p.scale)) return err(FB_ERR_INVALID_ATTENTION_SCALE, "attention scale must be finite");
    p.group_size = p.query_heads / p.key_heads;
    p.causal = options.has_causal != 0;
    p.causal_offset = options.causal;
    *plan = p;
    return {};
}

// ----------------------------------------------------------- reductions

Error reduction_shape(uint32_t op, const Dims& input, const std::vector<uint32_t>& axes, bool keep, bool is_mean,
                      Dims* out) {
    if (!is_mean && op > FB_REDUCE_MAX) return err(FB_ERR_INVALID_INPUT, "unknown reduction operation");
    Error e = reduce_dims(input, axes, keep, out);
    if (!ok(e)) return e;
    if (is_mean || op == FB_REDUCE_MIN || op == FB_REDUCE_MAX) {
        uint64_t n;
        numel(*out, &n);
        if (n != 0)
            for (uint32_t a : axes)
                if (input[a] == 0)
                    return err(FB_ERR_EMPTY_REDUCTION,
                               "min, max and mean require a nonempty contraction for each output");
    }
    return {};
}

}  // namespace fb
