/*
 * oracle.h - CPU restatement of the reference's f64 oracles for the dense-op
 * path.  TEST INFRASTRUCTURE ONLY: used by tests/, by __graft_entry__.smoke()
 * as the checker, and by bench.py's CPU-baseline leg.  Never on the product
 * path.
 *
 * All tensors are logical row-major arrays (the reference oracles work on
 * logical values, not layouts).  Every function cites the reference code it
 * follows (paths relative to the reference repository).
 */
#ifndef FORMA_ORACLE_H
#define FORMA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* conformance data(): ((i*17 + i/19 + seed*7) % 43)/16 - 1.25
 * (crates/tensor-core/src/conformance/attention.rs:26-35). */
void oracle_data(uint64_t n, uint64_t seed, float* out);

/* Output geometry of the independent conv oracle
 * (conformance/convolution.rs:186-199).  Returns output rank. */
int oracle_conv_dims(const uint64_t* in_dims, const uint64_t* w_dims, int rank, const uint64_t* strides,
                     const uint64_t* dilations, const uint64_t* pad_before, const uint64_t* pad_after,
                     uint64_t* out_dims);

/* Dense f64 cross-correlation with signed coordinates
 * (conformance/convolution.rs:180-231).  Output is row-major over
 * oracle_conv_dims.  `threads` >= 1 splits output elements. */
void oracle_conv(const uint64_t* in_dims, const float* in, const uint64_t* w_dims, const float* w, int rank,
                 const uint64_t* strides, const uint64_t* dilations, const uint64_t* pad_before,
                 const uint64_t* pad_after, uint64_t groups, double* out, int threads);

/* The reference CUDA kernel's f32 arithmetic: per output, input channel
 * outer, kernel tap inner, product and sum each rounded to f32, no FMA
 * (crates/compute-cuda/src/convolution.cu:41-63). */
void oracle_conv_f32_seq(const uint64_t* in_dims, const float* in, const uint64_t* w_dims, const float* w, int rank,
                         const uint64_t* strides, const uint64_t* dilations, const uint64_t* pad_before,
                         const uint64_t* pad_after, uint64_t groups, float* out, int threads);

/* Dense f64 attention (conformance/attention.rs:118-252).  Operands have
 * rank >= 2 (rank 2 = one implicit head); batch prefixes broadcast.  `mask`
 * is an additive f64 bias of rank `mask_rank` broadcasting to
 * [batch..., heads, Lq, Lk] (keep masks pass 0 / -inf), or NULL.
 * Output is row-major [batch..., heads, Lq, Dv] (or [Lq, Dv] for three
 * rank-2 operands).  Returns the element count written. */
uint64_t oracle_attention(const uint64_t* q_dims, int q_rank, const float* q, const uint64_t* k_dims, int k_rank,
                          const float* k, const uint64_t* v_dims, int v_rank, const float* v,
                          const uint64_t* mask_dims, int mask_rank, const double* mask, int has_scale, float scale,
                          int has_causal, int32_t causal, double* out, int threads);

/* expected_f32 (conformance/reduction.rs:24-54): f64 fold in element order,
 * rounded to f32.  op: 0 sum, 1 product, 2 min, 3 max. */
void oracle_reduce_f32(const float* x, const uint64_t* dims, int rank, const uint32_t* axes, int n_axes, int op,
                       float* out);
/* expected_u32 (conformance/reduction.rs:56-79): wrapping arithmetic. */
void oracle_reduce_u32(const uint32_t* x, const uint64_t* dims, int rank, const uint32_t* axes, int n_axes, int op,
                       uint32_t* out);

/* Statistics reference (conformance/statistics.rs:267-319): anchor-shifted
 * f64 mean and population variance, max-shifted softmax / log-softmax /
 * logsumexp, layer norm.  Any output pointer may be NULL. */
void oracle_stats(const float* x, const uint64_t* dims, int rank, const uint32_t* axes, int n_axes, float eps,
                  float* mean, float* variance, float* softmax, float* log_softmax, float* logsumexp, float* norm);

/* Same arithmetic for contiguous rows, split over `threads`. */
void oracle_row_stats(const float* x, uint64_t rows, uint64_t cols, float eps, float* mean, float* variance,
                      float* softmax, float* log_softmax, float* logsumexp, float* norm, int threads);

/* Row sums/max in f64 folded in element order, rounded to f32, split over
 * `threads` (the row form of oracle_reduce_f32). */
void oracle_row_reduce(const float* x, uint64_t rows, uint64_t cols, int op, float* out, int threads);

/* Per-row index of the maximum under f32::total_cmp, lowest index on ties
 * (Tensor::topk, crates/tensor-core/src/host_tensor/similarity.rs:52-107). */
void oracle_argmax_rows(const float* x, uint64_t rows, uint64_t cols, uint32_t* out, int threads);

/* f64 sum of n values in element order (the all-axes form of expected_f32). */
double oracle_sum_f64(const float* x, uint64_t n, int threads);

/* Nearest-even f32 -> BF16 / F16 bits (the conformance codec `round`,
 * conformance/low_ops.rs, and encode_low, compute-cuda/src/low_precision.cu:
 * 6-16) and the exact decode. */
uint16_t oracle_round_bf16(float x);
uint16_t oracle_round_f16(float x);
float oracle_decode_bf16(uint16_t b);
float oracle_decode_f16(uint16_t b);

#ifdef __cplusplus
}
#endif

#endif
