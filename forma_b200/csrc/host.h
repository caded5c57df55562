// Host-side contracts of the dense-op path: shapes, strided layouts and the
// operation plans that tensor-core validates before any launch.  Each routine
// restates the checks of the cited reference function so that the C ABI
// rejects exactly what the Rust traits reject, with the same error class.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/forma_b200.h"

namespace fb {

using Dims = std::vector<uint64_t>;

// Error carried from a validation routine to the C ABI boundary.
struct Error {
    int status = FB_OK;
    std::string detail;
};

// Records `detail` as this thread's last error and returns `status`.
int fail(int status, const std::string& detail);
inline bool ok(const Error& e) { return e.status == FB_OK; }
inline Error err(int status, std::string detail) { return Error{status, std::move(detail)}; }

// Checked element count (Shape::new, tensor-core/src/shape.rs:11-21): a zero
// dimension makes the shape empty without checking the remaining product.
Error numel(const Dims& dims, uint64_t* out);

// Shape::validate_axes (shape.rs:55-82).
Error validate_axes(const Dims& dims, const std::vector<uint32_t>& axes);

// Shape::reduce (shape.rs:87-100).
Error reduce_dims(const Dims& dims, const std::vector<uint32_t>& axes, bool keep, Dims* out);

// broadcast_dims (shape.rs:115-134).
Error broadcast_dims(const Dims& left, const Dims& right, Dims* out);

// Strided layout of one tensor argument (layout.rs:6-16).
struct View {
    Dims dims;
    Dims strides;
    uint64_t offset = 0;
    uint64_t storage_len = 0;
    uint32_t dtype = FB_F32;
    void* data = nullptr;
    uint64_t count = 0;  // logical element count
};

// Converts a descriptor into a View, checking rank, dtype and that every
// addressed element lies inside the storage (Layout::required_storage_len,
// layout.rs:266-279, and CudaRuntime::check, compute-cuda/src/runtime.rs:217-224).
Error view_of(const fb_tensor* t, const char* name, View* out);

// Layout::is_contiguous (layout.rs:251-265).
bool is_contiguous(const View& v);

// Output descriptors must have the planned dims and a layout that addresses
// every element exactly once within the storage (any permutation of a dense
// block is allowed, so a channels-last conv output can be a permuted view).
Error check_output(const fb_tensor* t, const char* name, const Dims& dims, uint32_t dtype, View* out);

uint64_t dtype_size(uint32_t dtype);
bool is_low(uint32_t dtype);

// ------------------------------------------------------------------ conv
struct ConvPlan {
    Dims input, weight, output;
    uint32_t spatial_rank = 0;
    uint64_t groups = 1;
    uint64_t channels_per_group = 0, outputs_per_group = 0;
    uint64_t strides[3] = {1, 1, 1}, dilations[3] = {1, 1, 1};
    uint64_t pad_before[3] = {0, 0, 0}, pad_after[3] = {0, 0, 0};
};
// ConvPlan::new (tensor-core/src/convolution.rs:43-111).
Error conv_plan(const Dims& input, const Dims& weight, const fb_conv_options* options, ConvPlan* plan);

// --------------------------------------------------------------- attention
struct AttentionPlan {
    Dims query, key, value;  // promoted to rank >= 3
    Dims batch, scores, canonical_output, output;
    uint64_t query_heads = 0, key_heads = 0, queries = 0, keys = 0;
    uint64_t depth = 0, value_depth = 0, group_size = 1;
    float scale = 1.0f;
    bool causal = false;
    int32_t causal_offset = 0;
};
// AttentionPlan::new (tensor-core/src/attention.rs:82-170).
Error attention_plan(const Dims& q, const Dims& k, const Dims& v, const Dims* mask,
                     fb_attention_options options, AttentionPlan* plan);

// ----------------------------------------------------------- reductions
// reduction_shape / mean_shape (tensor-core/src/reduction.rs:44-72).
Error reduction_shape(uint32_t op, const Dims& input, const std::vector<uint32_t>& axes, bool keep,
                      bool is_mean, Dims* out);

}  // namespace fb
