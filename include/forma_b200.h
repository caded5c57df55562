/*
 * forma_b200.h - C ABI of the B200 (sm_100a) dense-op backend.
 *
 * This library replaces the kernel launches behind Forma's `compute-cuda`
 * implementations of the tensor-core traits for convolution, scaled
 * dot-product attention, reductions and statistics.  The Rust side keeps its
 * planning, owner checks and output allocation; each trait method ends in one
 * call below with plain descriptors, a caller stream and an int status.
 *
 * Conventions (all mirror the reference runtime):
 *  - A tensor is a strided view into device storage: `dims`, `strides` and
 *    `offset` are in ELEMENTS (crates/tensor-core/src/layout.rs:6-16); stride 0
 *    broadcasts.  `storage_len` is the element count of the backing allocation
 *    and bounds every access (Layout::validate_storage_len, layout.rs:280-289).
 *  - Outputs are caller-allocated, exclusive and sized by the matching
 *    `*_plan` / `*_shape` query; every element of the output is written.
 *  - Validation happens before empty shortcuts (tensor-core/src/convolution.rs:
 *    119-124); a non-zero status leaves outputs untouched and launches nothing.
 *  - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *    stream) and is asynchronous, like the reference's single-stream runtime
 *    (compute-cuda/src/runtime.rs:66-81).
 *  - There is no CPU fallback: a missing device or kernel is FB_ERR_DRIVER.
 *  - Every call runs on the calling thread's current device (cudaSetDevice),
 *    which must own every operand and the stream, as the reference's runtime
 *    owns one device (compute-cuda/src/runtime.rs:66-81).  Library scratch is
 *    kept per (device, stream); host threads that call concurrently must use
 *    different streams or the per-thread default stream (cudaStreamPerThread,
 *    keyed per thread).  Resetting a device (cudaDeviceReset) invalidates
 *    every device address the library has cached for it: make no further
 *    calls on that device in the same process.
 */
#ifndef FORMA_B200_H
#define FORMA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FB_MAX_RANK 8
#define FB_ABI_VERSION 1

/* Element types. F16/BF16 are the reference's LowDtype storage
 * (tensor-core/src/low_precision.rs:7-10): raw 16-bit patterns. */
typedef enum fb_dtype {
    FB_F32 = 0,
    FB_U32 = 1,
    FB_F16 = 2,
    FB_BF16 = 3,
} fb_dtype;

/* Status codes.  1..31 mirror tensor_core::TensorError
 * (tensor-core/src/error.rs:1-56); 32.. mirror compute_cuda::CudaError
 * (compute-cuda/src/error.rs:3-26). */
typedef enum fb_status {
    FB_OK = 0,
    FB_ERR_SHAPE_OVERFLOW = 1,
    FB_ERR_LAYOUT_OVERFLOW = 2,
    FB_ERR_RANK_MISMATCH = 3,
    FB_ERR_AXIS_OUT_OF_BOUNDS = 4,
    FB_ERR_DUPLICATE_AXIS = 5,
    FB_ERR_INCOMPATIBLE_BROADCAST = 6,
    FB_ERR_STORAGE_OUT_OF_BOUNDS = 7,
    FB_ERR_EMPTY_REDUCTION = 8,
    FB_ERR_INVALID_EPSILON = 9,
    FB_ERR_INVALID_ATTENTION = 10,
    FB_ERR_INVALID_ATTENTION_SCALE = 11,
    FB_ERR_INVALID_CONVOLUTION = 12,
    FB_ERR_LOW_DTYPE_MISMATCH = 13,
    FB_ERR_MATMUL_RANK = 14,
    FB_ERR_MATMUL_INNER_DIMENSION = 15,
    FB_ERR_INVALID_INPUT = 32,
    FB_ERR_DTYPE = 33,
    FB_ERR_DRIVER = 34,
    FB_ERR_UNSUPPORTED = 35,
    FB_ERR_FOREIGN_RUNTIME = 36,  /* CudaError::ForeignRuntime: another device's object */
    FB_ERR_MISSING_SYMBOL = 37,   /* CudaError::MissingSymbol (compute-cuda/src/libraries.rs:100-117) */
    FB_ERR_GRAPH = 38,            /* CudaError::Graph: recording or instantiating a program failed */
    FB_ERR_PROGRAM_POISONED = 39, /* CudaError::ProgramPoisoned */
} fb_status;

/* Strided view of device storage (compute-cuda/src/runtime.rs:44-61:
 * CudaTensor = Arc<CudaSlice<T>> + Layout). */
typedef struct fb_tensor {
    void* data;           /* device address of storage element 0 */
    uint64_t storage_len; /* elements in the allocation */
    uint32_t dtype;       /* fb_dtype */
    uint32_t rank;        /* 0..FB_MAX_RANK */
    uint64_t dims[FB_MAX_RANK];
    uint64_t strides[FB_MAX_RANK];
    uint64_t offset;
} fb_tensor;

/* tensor_core::ConvOptions (tensor-core/src/convolution.rs:7-13).  Each vector
 * has its own length so ConvPlan's "every option vector must match the
 * spatial rank" check is preserved. */
typedef struct fb_conv_options {
    const uint64_t* strides;
    uint32_t strides_len;
    const uint64_t* dilations;
    uint32_t dilations_len;
    const uint64_t* padding_before;
    uint32_t padding_before_len;
    const uint64_t* padding_after;
    uint32_t padding_after_len;
    uint64_t groups;
} fb_conv_options;

/* tensor_core::AttentionOptions (tensor-core/src/attention.rs:3-13). */
typedef struct fb_attention_options {
    int32_t has_scale; /* 0 = default 1/sqrt(depth) */
    float scale;
    int32_t has_causal; /* 0 = no causal mask */
    int32_t causal;     /* key j visible to query i iff j <= i + causal */
} fb_attention_options;

/* tensor_core::AttentionMask (tensor-core/src/attention.rs:15-23). */
typedef enum fb_mask_kind {
    FB_MASK_NONE = 0,
    FB_MASK_KEEP = 1,     /* u32 tensor, nonzero keeps the key */
    FB_MASK_ADDITIVE = 2, /* f32 tensor, finite bias or -inf */
} fb_mask_kind;

/* tensor_core::ReduceOp (tensor-core/src/reduction.rs:6-13). */
typedef enum fb_reduce_op {
    FB_REDUCE_SUM = 0,
    FB_REDUCE_PRODUCT = 1,
    FB_REDUCE_MIN = 2,
    FB_REDUCE_MAX = 3,
} fb_reduce_op;

/* ---------------------------------------------------------------- library */

/* FB_ABI_VERSION of the loaded library. */
int fb_abi_version(void);
/* Static description of a status code. */
const char* fb_status_string(int status);
/* Detail of the last non-zero status returned on this host thread. */
const char* fb_last_error(void);
/* Number of kernel launches this library has enqueued (all threads). */
uint64_t fb_launch_count(void);
/* The kernels that the most recent computing call on this host thread
 * enqueued, separated by ';' in launch order, template instantiations
 * spelled out (e.g. "conv_gemm_pair_kernel<192,12>" or
 * "attn_fwd_kernel<128,0,2>;attn_merge_kernel<128>"); "" when that call
 * launched nothing.  Shows which route (tensor cores, CUDA cores, split,
 * scratch + cast) served a call.  No counterpart in the reference, whose
 * kernels are fixed per operation.  Valid until the thread's next call. */
const char* fb_last_route(void);
/* Synchronises the current device and returns (and clears) a bit mask of
 * bounded waits that timed out inside this library's kernels since the last
 * call (0 = none).  A kernel that gives up a wait writes no partial result
 * beyond what it had finished and releases its resources. */
uint32_t fb_device_status(void);

/* ------------------------------------------------------------ convolution */

/* ConvPlan::new (tensor-core/src/convolution.rs:43-111): writes the output
 * dims [N, O, *spatial] and rank.  Host only. */
int fb_conv_plan(const uint64_t* input_dims, uint32_t input_rank,
                 const uint64_t* weight_dims, uint32_t weight_rank,
                 const fb_conv_options* options, uint64_t* out_dims,
                 uint32_t* out_rank);

/* TensorConvBackend::conv (tensor-core/src/convolution.rs:125-132; replaces
 * the conv_f32 launch at compute-cuda/src/convolution.rs:180-212).  f32
 * input/weight/output.  Every output element is accumulated in f32 in the
 * reference's (input channel, kernel tap) order with separately rounded
 * multiply and add, so results are bit-identical to the reference kernel. */
int fb_conv(const fb_tensor* input, const fb_tensor* weight,
            const fb_conv_options* options, fb_tensor* output, void* stream);

/* TensorLowConvBackend::conv_low_f32 (tensor-core/src/low_convolution.rs:
 * 16-33; replaces the conv_low launch at compute-cuda/src/convolution.rs:
 * 226-239).  F16/BF16 input and weight of the same dtype, f32 output.
 * Channels-last input ([N,C,H,W] viewed over NHWC storage) and weights over
 * [O,kh,kw,C] storage run as a tcgen05 implicit GEMM with f32 accumulation;
 * other layouts run a CUDA-core direct kernel with f32 accumulation. */
int fb_conv_low_f32(const fb_tensor* input, const fb_tensor* weight,
                    const fb_conv_options* options, fb_tensor* output,
                    void* stream);

/* TensorLowConvBackend::conv_low (tensor-core/src/low_convolution.rs:35-44):
 * conv_low_f32 followed by one nearest-even rounding to the input dtype.
 * `output` has the input's low dtype. */
int fb_conv_low(const fb_tensor* input, const fb_tensor* weight,
                const fb_conv_options* options, fb_tensor* output,
                void* stream);

/* -------------------------------------------------------------- attention */

/* AttentionPlan::new (tensor-core/src/attention.rs:82-170): output dims and
 * rank.  `mask_dims` may be NULL when there is no mask.  Host only. */
int fb_attention_plan(const uint64_t* q_dims, uint32_t q_rank,
                      const uint64_t* k_dims, uint32_t k_rank,
                      const uint64_t* v_dims, uint32_t v_rank,
                      const uint64_t* mask_dims, uint32_t mask_rank,
                      fb_attention_options options, uint64_t* out_dims,
                      uint32_t* out_rank);

/* TensorAttentionBackend::attention (tensor-core/src/attention.rs:49-58;
 * replaces the attention_f32 launch at compute-cuda/src/attention.rs:20-81).
 * f32 Q/K/V; `mask` is NULL for FB_MASK_NONE. */
int fb_attention(const fb_tensor* query, const fb_tensor* key,
                 const fb_tensor* value, uint32_t mask_kind,
                 const fb_tensor* mask, fb_attention_options options,
                 fb_tensor* output, void* stream);

/* TensorLowAttentionBackend::attention_low_f32 (tensor-core/src/
 * low_attention.rs:28-37; replaces compute-cuda/src/low_attention.rs:4-28).
 * F16/BF16 Q/K/V of one dtype, f32 output.  Heads with unit-stride depth
 * D in {64, 128} and 16-byte aligned rows (keep or additive masks included)
 * run as a fused tcgen05 flash kernel; other geometries run CUDA-core
 * online-softmax kernels. */
int fb_attention_low_f32(const fb_tensor* query, const fb_tensor* key,
                         const fb_tensor* value, uint32_t mask_kind,
                         const fb_tensor* mask, fb_attention_options options,
                         fb_tensor* output, void* stream);

/* TensorLowAttentionBackend::attention_low (tensor-core/src/
 * low_attention.rs:38-47; the CUDA program builder's attention_low,
 * compute-cuda/src/program/builder_attention.rs:29-42): attention_low_f32
 * rounded once, nearest-even, into the operands' 16-bit dtype, which the
 * output must have.  On the tcgen05 path the rounding happens in the
 * kernel's epilogue (no f32 result in memory); otherwise an f32 result in
 * library scratch is cast afterwards. */
int fb_attention_low(const fb_tensor* query, const fb_tensor* key,
                     const fb_tensor* value, uint32_t mask_kind,
                     const fb_tensor* mask, fb_attention_options options,
                     fb_tensor* output, void* stream);

/* -------------------------------------------------------------- reduction */

/* reduction_shape / mean_shape (tensor-core/src/reduction.rs:44-72). */
int fb_reduce_shape(uint32_t op, const uint64_t* dims, uint32_t rank,
                    const uint32_t* axes, uint32_t n_axes, int32_t keep_dims,
                    int32_t is_mean, uint64_t* out_dims, uint32_t* out_rank);

/* TensorReduceBackend::reduce_f32 (tensor-core/src/reduction.rs:20-27;
 * replaces compute-cuda/src/reduction.rs:79-160). */
int fb_reduce_f32(uint32_t op, const fb_tensor* input, const uint32_t* axes,
                  uint32_t n_axes, int32_t keep_dims, fb_tensor* output,
                  void* stream);

/* TensorReduceBackend::reduce_u32 (tensor-core/src/reduction.rs:28-34):
 * wrapping sum/product, exact min/max. */
int fb_reduce_u32(uint32_t op, const fb_tensor* input, const uint32_t* axes,
                  uint32_t n_axes, int32_t keep_dims, fb_tensor* output,
                  void* stream);

/* TensorReduceBackend::mean_axes (tensor-core/src/reduction.rs:35-40;
 * replaces compute-cuda/src/reduction.rs:205-224). */
int fb_mean_axes(const fb_tensor* input, const uint32_t* axes,
                 uint32_t n_axes, int32_t keep_dims, fb_tensor* output,
                 void* stream);

/* Row argmax: index (u32) of the largest element along `axis`, ordered by
 * the IEEE total order (-0 < +0), lowest index on ties.  No trait method in
 * the reference; the rule is Tensor::topk's (tensor-core/src/host_tensor/
 * similarity.rs:82).  Output shape = input with `axis` removed (or kept as
 * 1).  An empty contraction with a nonempty output is FB_ERR_EMPTY_REDUCTION. */
int fb_argmax(const fb_tensor* input, uint32_t axis, int32_t keep_dims,
              fb_tensor* output, void* stream);

/* Sum of every element of an f32 tensor into one f64 on the device
 * (`partial` is a device pointer to one double).  This is the per-shard
 * partial of the global sum; callers combine shards with one all-reduce and
 * finish with fb_finish_sum_f64.  Replaces the multi-pass reduce_all path of
 * compute-cuda/src/reduction.rs:145-160. */
int fb_sum_partial_f64(const fb_tensor* input, double* partial, void* stream);

/* Rounds the device f64 at `partial` into the f32 tensor `output` (one
 * element, any rank with numel 1). */
int fb_finish_sum_f64(const double* partial, fb_tensor* output, void* stream);

/* --------------------------------------------------------- multi-GPU sum */

/* The global sum of rows sharded across GPUs (one process or thread per GPU,
 * or one process driving several): the f64 partial of this shard, ONE
 * in-place NCCL all-reduce of 8 bytes over `comm` on `stream`, and the f32
 * rounding into `output` (one element), all enqueued on the caller's stream.
 * Every rank of the communicator makes the same call.  The reference runtime
 * is single-device per process (gpu-compute/src/cuda.rs:80-86), so the
 * exchange lives in the backend; it replaces the multi-pass reduce_all of
 * compute-cuda/src/reduction.rs:145-160 at the scale of several GPUs.
 * `comm` is an ncclComm_t of the current device (FB_ERR_FOREIGN_RUNTIME
 * otherwise).  NCCL is loaded at run time ($FB_NCCL_LIBRARY, else the copy the
 * process already loaded, else libnccl.so.2); every symbol is checked before
 * the first call and a missing one is FB_ERR_MISSING_SYMBOL. */
int fb_global_sum_nccl(const fb_tensor* shard, void* comm, fb_tensor* output, void* stream);

/* Communicator set-up for fb_global_sum_nccl, so a caller needs no NCCL
 * bindings of its own.  fb_nccl_unique_id writes FB_NCCL_UNIQUE_ID_BYTES
 * bytes (rank 0 creates it and hands it to the other ranks);
 * fb_nccl_comm_init_rank joins rank `rank` of `nranks` on the current
 * device; fb_nccl_comm_init_all creates one communicator per listed device
 * in one process (devices NULL = 0..ndev-1); fb_nccl_comm_destroy releases
 * one (NULL is a no-op). */
#define FB_NCCL_UNIQUE_ID_BYTES 128
int fb_nccl_unique_id(void* id);
int fb_nccl_comm_init_rank(void** comm, int nranks, const void* id, int rank);
int fb_nccl_comm_init_all(void** comms, int ndev, const int* devices);
int fb_nccl_comm_destroy(void* comm);

/* Size of the per-device static scratch array of fb_sum_partial_f64_static. */
#define FB_SUM_STATIC_SCRATCH_BYTES 65536

/* fb_sum_partial_f64 for callers that cannot allocate device memory.  No
 * counterpart in the reference.  Engines that reserve the device's memory up
 * front and route every allocation through their own pool, and latency-
 * critical paths on which cudaMalloc's implicit device-wide synchronisation
 * is not acceptable, cannot let a library call cudaMalloc; this entry point
 * calls no allocating routine.  Its block partials and finishing counter live
 * in a file-scope device array of FB_SUM_STATIC_SCRATCH_BYTES that every GPU
 * loading the library keeps until the process exits.  Limits: each block
 * leaves one partial in the array; a call launches four blocks per SM, or
 * one per 2^18 input elements when that is more, so inputs above
 * fb_sum_static_max_elements() elements (8160 x 2^18, about 2.1e9) are
 * rejected with FB_ERR_INVALID_INPUT before anything is enqueued.  Every call
 * shares the array (the counter is cleared at the start of each call): calls
 * that overlap on the GPU, on any stream, race.  The first call on each
 * device looks up the array's device address (cached afterwards); make that
 * first call before any stream capture.  Output as fb_sum_partial_f64. */
int fb_sum_partial_f64_static(const fb_tensor* input, double* partial, void* stream);
/* Largest input element count fb_sum_partial_f64_static accepts. */
uint64_t fb_sum_static_max_elements(void);

/* ------------------------------------------------------------- statistics */

/* TensorStatsBackend (tensor-core/src/statistics.rs:100-129; replaces
 * compute-cuda/src/statistics.rs:45-252).  Inputs are F32, or F16/BF16 for
 * the *_low_f32 trait methods (tensor-core/src/low_statistics.rs:25-57),
 * selected by the input dtype; outputs are f32.  fb_softmax, fb_log_softmax
 * and fb_layer_norm also take a contiguous output of the input's F16/BF16
 * dtype: the *_low trait methods (low_statistics.rs:59-108, the f32 result
 * rounded once, nearest even), rounded as the rows are stored.  An F32 input
 * with an F16/BF16 output is rounded the same way (no counterpart in the
 * reference trait; for programs that feed a low-precision contraction). */
int fb_softmax(const fb_tensor* input, const uint32_t* axes, uint32_t n_axes,
               fb_tensor* output, void* stream);
int fb_log_softmax(const fb_tensor* input, const uint32_t* axes,
                   uint32_t n_axes, fb_tensor* output, void* stream);
int fb_logsumexp(const fb_tensor* input, const uint32_t* axes, uint32_t n_axes,
                 int32_t keep_dims, fb_tensor* output, void* stream);
int fb_moments(const fb_tensor* input, const uint32_t* axes, uint32_t n_axes,
               int32_t keep_dims, fb_tensor* mean, fb_tensor* variance,
               void* stream);
int fb_layer_norm(const fb_tensor* input, const uint32_t* axes,
                  uint32_t n_axes, float epsilon, fb_tensor* output,
                  void* stream);

/* ----------------------------------------------------------- low storage */

/* TensorLowBackend::cast_to_low (tensor-core/src/low_precision.rs:310-355;
 * encode_low at compute-cuda/src/low_precision.cu:6-16): nearest-even f32 ->
 * F16/BF16 of `output->dtype`; `output` must be contiguous. */
int fb_cast_to_low(const fb_tensor* input, fb_tensor* output, void* stream);

/* ------------------------------------------------------ low-precision GEMM */

/* MatmulPlan::new (tensor-core/src/shape.rs:141-192): vectors are promoted
 * (left [K] -> [1, K], right [K] -> [K, 1]) and removed again from the output,
 * batch axes broadcast.  Writes the output dims. */
int fb_matmul_plan(const uint64_t* left_dims, uint32_t left_rank,
                   const uint64_t* right_dims, uint32_t right_rank,
                   uint64_t* out_dims, uint32_t* out_rank);

/* TensorLowBackend::matmul_low_f32 / matmul_low (tensor-core/src/
 * low_precision.rs:96-106; replaces the cuBLAS GEMM of compute-cuda/src/
 * low_precision.rs:240-270 and matmul.rs:144-162): f16/bf16 operands of one
 * dtype, f32 accumulation; matmul_low_f32 writes f32, matmul_low rounds the
 * f32 result once (nearest even) to the operands' dtype.  Any strides; the
 * tensor cores take rows with a contiguous K axis on the left and either a
 * contiguous N or K axis on the right (K and N multiples of 64). */
int fb_matmul_low_f32(const fb_tensor* left, const fb_tensor* right,
                      fb_tensor* output, void* stream);
int fb_matmul_low(const fb_tensor* left, const fb_tensor* right,
                  fb_tensor* output, void* stream);

/* ------------------------------------------------------- elementwise glue */

/* Glue for composite workloads that chain the operators above (residual
 * additions, the activation between two contractions).  Not part of the
 * reference's conv/attention/reduction path; the arithmetic follows the
 * reference's own elementwise definitions.
 *
 * out = a + b in f32, the `binary` kernel with its add op
 * (compute-cuda/src/kernels.cu:29-58).  `a` and `b` have `output`'s dims and
 * any strides (0 broadcasts); `output` may have any layout that addresses each
 * element once, and an operand may share memory with it only as the
 * identical view (an in-place update). */
int fb_add(const fb_tensor* a, const fb_tensor* b, fb_tensor* output, void* stream);

/* tanh-form GELU (tensor-core/src/host_tensor/activation.rs:9-20) of an f32
 * input, rounded once to `output->dtype` (F16/BF16, nearest even); `output`
 * is contiguous with `input`'s dims. */
int fb_gelu_to_low(const fb_tensor* input, fb_tensor* output, void* stream);

/* Fused forms of the two chains above, for projections written as 1x1 (or
 * any) low convolutions: the tensor-core GEMM applies them to its f32 sums in
 * the epilogue, so the f32 intermediate never reaches memory.  Results are
 * bit-identical to the unfused chains (the same f32 arithmetic, one rounding);
 * layouts the tensor cores refuse compute the same chain through scratch.
 *
 * fb_conv_low_gelu: fb_gelu_to_low(fb_conv_low_f32(input, weight)) into a
 * 16-bit `output` of the operands' dtype (arguments as fb_conv_low). */
int fb_conv_low_gelu(const fb_tensor* input, const fb_tensor* weight, const fb_conv_options* options, fb_tensor* output,
                     void* stream);

/* fb_conv_low_f32_accumulate: output += fb_conv_low_f32(input, weight), the
 * f32 `output` (conv_low_f32's output dims, any layout addressing each
 * element once) read and written in place: a residual connection.  The
 * output may not share memory with the input or the weight
 * (FB_ERR_INVALID_INPUT). */
int fb_conv_low_f32_accumulate(const fb_tensor* input, const fb_tensor* weight, const fb_conv_options* options,
                               fb_tensor* output, void* stream);

/* ------------------------------------------------------ prepared programs */

/* A sequence of the calls above recorded once on a stream and replayed as
 * one CUDA graph launch with the same buffers: the reference's prepared
 * programs with CUDA Graph capture (compute-cuda/src/program.rs:1-60,
 * program/graph.rs, program/execution.rs:20-150), for any sequence of this
 * library's operators, convolution included.  fb_program_begin starts
 * recording on `stream` (a created stream, not a default stream) for this
 * host thread; the fb_* calls that follow on that stream are recorded, not
 * run; fb_program_end stops and instantiates.  Recording allocates nothing:
 * each operator's library scratch must exist already, so run the sequence
 * once eagerly on the same stream first (a call that would need new scratch
 * fails while recording, and the recording then fails as FB_ERR_GRAPH, as
 * does any allocation or synchronising call made while recording).
 * fb_program_launch replays it; a failed launch poisons the program
 * (FB_ERR_PROGRAM_POISONED from then on, like CudaError::ProgramPoisoned).
 * fb_program_stats reports this library's kernels in the recording, the
 * graph's node count and whether the program is poisoned. */
typedef struct fb_program fb_program;
int fb_program_begin(void* stream);
int fb_program_end(void* stream, fb_program** program);
int fb_program_launch(fb_program* program, void* stream);
int fb_program_stats(const fb_program* program, uint64_t* kernel_launches, uint64_t* graph_nodes, int32_t* poisoned);
int fb_program_destroy(fb_program* program);

/* ------------------------------------------------------------ diagnostics */

/* Launches one CTA whose thread waits on an mbarrier that nothing arrives at,
 * through the same bounded wait every kernel here uses, with a limit of
 * `limit_ns` (0 < limit_ns <= 1e9).  The wait gives up, bit 6 is recorded in
 * the word fb_device_status() returns, and the kernel exits normally, so a
 * caller can check - without a hang or a fault - that timed-out waits are
 * reported.  No counterpart in the reference, whose fault injection is on the
 * host (compute-cuda/src/libraries.rs:120-174). */
int fb_selftest_bounded_wait(uint64_t limit_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FORMA_B200_H */
