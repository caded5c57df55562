// Fused flash attention on the 5th-generation tensor cores (tcgen05).
//
// attention_low_f32 for 16-bit Q/K/V, depth D in {64, 128}, keep / additive
// masks, optional causal offset.  One CTA owns 256 query rows (two 128-row Q
// tiles) of one (batch, head) and streams that head's K/V once for both tiles
// (short key ranges at depth 64: one Q tile per CTA, two CTAs per SM).
//   warp 0      TMA producer: both Q tiles once, then K and V tiles of 128
//               keys into rings of 2 (D = 128) or 4 (D = 64) slots with their
//               own full/empty barriers (128B-swizzled boxes of 64 depth
//               columns).  A K slot is released as soon as both tiles' S of
//               that key tile are computed, a key step before its V, so K
//               tiles load two key steps ahead of their use.
//   warp 1      TMEM allocator and MMA issuer (the whole warp runs the issue
//               loop; one elected lane issues).  Per key tile j, per Q tile t:
//                 S_t = Q_t K_j^T  -> TMEM S_t (128 x 128 f32)
//                 O_t += P_t V_j   -> TMEM O_t (128 x D f32), P_t read from
//                                     TMEM where it overwrote S_t (tcgen05.mma
//                                     with the A operand in TMEM)
//               in the order S_0, S_1, then PV_0, S_0', PV_1, S_1', ... so the
//               tensor core computes one tile's products while the other
//               tile's softmax runs (ping-pong).
//   warps 2-5   softmax of Q tile 0, warps 6-9 of Q tile 1, one query row per
//               thread: tcgen05.ld of the S row, row max on raw scores (three-
//               input extremes), one packed FFMA per score pair, exp2 (seven
//               pairs in eight on MUFU ex2, one as a paired polynomial on the
//               FMA pipe), P packed to 16-bit pairs (cvt, nearest even) and
//               written back over S with tcgen05.st.  For BF16 the row sum is
//               taken after P is handed to the MMA warp, from the rounded P
//               values the MMA multiplies (so it is off the S -> P critical
//               path and normalises exactly the weights used).  The running
//               max is only raised (and O rescaled in TMEM) when a row max
//               exceeds it by more than 2^8, so P <= 2^8 and rescales are rare.
//               Finally O / l: staged in the idle K/V ring once both tiles'
//               MMAs are done and written by TMA tensor stores (rows past L
//               clipped by the map), or stored row by row where the output
//               has no tensor map or the key range is split.
// Ordering: a tcgen05.commit completes only after every earlier MMA of the
// issuing thread, so "S_t of tile j+1 ready" also certifies that PV_t of tile
// j has consumed P_t and updated O_t: the softmax needs no other wait.
// Overflow: BF16 P is stored pre-multiplied by 2^-shift (shift = 9 + log2 of
// the key count, an exact power of two), so the unnormalised numerator sum P V
// stays below max|V| and cannot overflow f32 even for V near the format's
// maximum, which the trait contract requires (tensor-core/src/attention.rs:
// 41-48); the final O / l divides the same factor out.  F16 needs no shift.
// Fully masked rows (l == 0) produce zeros.  Every wait is bounded.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>

#include "async.cuh"
#include "device_common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace fb {
namespace {

__device__ uint32_t g_attn_status;

constexpr int TQ = 128, TK = 128;

struct AttnParams {
    uint32_t fmt;           // 0 f16, 1 bf16
    uint32_t L, Lk;         // queries, keys per head
    uint32_t H, Hkv;        // query heads, key/value heads
    uint32_t q_blocks, bh;  // 256-row query blocks per head, batch x heads
    uint32_t kv_tiles;
    float scale_log2;       // scale * log2(e)
    float shift;            // log2 of the numerator pre-scale
    int32_t causal, causal_offset;
    uint32_t k_batch_bcast, v_batch_bcast;  // K / V shared by every batch index (stride 0)
    float* out;             // f32 rows (or 16-bit rows, out_low): depth contiguous, rows at the strides below
    uint32_t out_low;       // 0: f32 output; FB_BF16 / FB_F16: each value rounded once (nearest even)
    uint64_t o_sb, o_sh, o_sl;              // output strides (elements) of batch, head, query
    const void* mask;       // keep (u32) or additive (f32) mask, keys contiguous
    uint64_t m_sb, m_sh, m_sq;              // mask strides (elements; 0 = broadcast) of batch, head, query
    // Key split (few query blocks over many key tiles): each CTA takes
    // `split_tiles` key tiles of its (batch, head, query block) and leaves,
    // per query row, a record {base, l, O[D]} in `part` (O unnormalised,
    // base the log2 reference of its exponentials); attn_merge_kernel
    // combines a row's records.  splits == 1: whole range, final output.
    uint32_t splits, split_tiles;
    uint32_t rec_rows;      // record rows per (batch, head): the query rows L
    uint32_t q_mod;         // a row's query index is row % q_mod (GQA-packed rows; L otherwise)
    float* part;
    uint32_t tma_out;       // 1: output rows staged in the K/V ring and written by TMA tensor stores (splits == 1)
    uint32_t tail_qb;       // causal, splits == 1: the lightest query blocks of every head, run last (0: none)
};

// First element of output row (batch, head, q) when the rows are 16-bit.
__device__ __forceinline__ uint16_t* low_row(const AttnParams& p, uint32_t batch, uint32_t head, uint32_t q) {
    return reinterpret_cast<uint16_t*>(p.out) + (uint64_t)batch * p.o_sb + (uint64_t)head * p.o_sh + (uint64_t)q * p.o_sl;
}

// QT Q tiles of 128 rows per CTA: 2 (the two tiles' softmax and MMA
// ping-pong on one SM) or 1 (short key ranges at D = 64: 256 TMEM columns and
// two K/V stages, so two CTAs share an SM and overlap each other's load and
// epilogue latency).
template <int D, int QT>
struct ACfg {
    static constexpr int THREADS = 64 + QT * 128;
    static constexpr int BOXES = D / 64;               // 64-column swizzle boxes per row
    static constexpr int Q_BYTES = TQ * D * 2;         // one Q tile
    static constexpr int K_BYTES = TK * D * 2;
    static constexpr int V_BYTES = TK * D * 2;
    static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
    static constexpr int STAGES = QT == 1 ? 2 : D == 64 ? 4 : 2;
    static constexpr int SMEM = 1024 + QT * Q_BYTES + STAGES * STAGE_BYTES + 256;
    static constexpr uint32_t TMEM_COLS = QT == 1 ? 256 : 512;
    // TMEM columns: S_t at t*128 (P_t aliases its first 64), O_t at QT*128 + t*128.
    static __device__ __forceinline__ uint32_t s_col(int t) { return (uint32_t)(t * TK); }
    static __device__ __forceinline__ uint32_t o_col(int t) { return (uint32_t)(QT * TK + t * 128); }
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x for a pair of values on the FMA/ALU pipes, for a share of the softmax
// exponentials so that the transcendental unit (MUFU ex2) is not the only
// engine producing them.  Cody-Waite split x = n + f: n is the nearest
// integer, obtained by adding and subtracting 1.5 * 2^23, and |f| <= 1/2; 2^f
// comes from a degree-3 polynomial whose coefficients minimise the maximum
// relative error on [-1/2, 1/2] (a linear program over a dense grid; 7.5e-5,
// below the 2^-11 rounding of an F16 P and the 2^-9 of a BF16 one); n is
// added to the exponent field (the low 9 bits of t's pattern hold n mod 512).
// Inputs are clamped to -127 first; at n = -127 a polynomial value below 1
// carries its exponent field below zero, which the final max with 0 turns
// into exactly 0, so -inf (a masked score) gives 0 and a fully masked row
// keeps a zero sum.  The f32x2 forms process both values in one instruction.
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
    const float2 M = make_float2(12582912.0f, 12582912.0f);
    const float2 xc = make_float2(fmaxf(x.x, -127.0f), fmaxf(x.y, -127.0f));
    const float2 t = __fadd2_rn(xc, M);
    const float2 n = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
    const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), xc);  // exact: xc - n
    float2 q = __ffma2_rn(make_float2(0.0551716685295105f, 0.0551716685295105f), f,
                          make_float2(0.2426111251115799f, 0.2426111251115799f));
    q = __ffma2_rn(q, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
    q = __ffma2_rn(q, f, make_float2(0.9999280571937561f, 0.9999280571937561f));
    const int bx = (int)(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23));
    const int by = (int)(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23));
    return make_float2(__int_as_float(max(bx, 0)), __int_as_float(max(by, 0)));
}

// Three-input extremes.  A NaN score is skipped by the row maximum but its
// exponential is NaN, which makes the row's sum and every output of the row
// NaN, as an elementwise max/exp/sum over the row would (measured: the
// NaN-propagating form costs ~1% of the kernel and changes no result).
__device__ __forceinline__ float max3n(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ float min3n(float a, float b, float c) {
    float d;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, uint32_t fmt) {
    uint32_t r;
    if (fmt)
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    else
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}


// Key tiles visible to the 128 query rows starting at q0 (0 if none exist).
__device__ __forceinline__ uint32_t visible_tiles(const AttnParams& p, uint32_t q0) {
    if (q0 >= p.L) return 0;
    if (!p.causal) return p.kv_tiles;
    int64_t last_q = (int64_t)min(q0 + TQ, p.L) - 1;
    if (p.q_mod < p.L) last_q = min(last_q, (int64_t)p.q_mod - 1);  // packed rows: queries repeat per head
    const int64_t last_key = last_q + (int64_t)p.causal_offset;
    const int64_t need = last_key < 0 ? 0 : last_key / TK + 1;
    return (uint32_t)(need < (int64_t)p.kv_tiles ? need : p.kv_tiles);
}

// MASK: FB_MASK_NONE, FB_MASK_KEEP (u32, nonzero keeps the key) or
// FB_MASK_ADDITIVE (f32 added to the scaled score; -inf excludes the key), as
// the reference applies them (compute-cuda/src/attention.cu:55-80).
template <int D, int MASK, int QT>
__global__ void __launch_bounds__(ACfg<D, QT>::THREADS, QT == 1 ? 2 : 1) attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                              const __grid_constant__ CUtensorMap tmK,
                                                              const __grid_constant__ CUtensorMap tmV,
                                                              const __grid_constant__ CUtensorMap tmO, AttnParams p) {
    using C = ACfg<D, QT>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sQ = smem;                          // QT tiles
    unsigned char* sKV = sQ + QT * C::Q_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + C::STAGES * C::STAGE_BYTES);
    uint64_t* q_full = bars;                           // 1
    uint64_t* k_full = bars + 1;                       // STAGES
    uint64_t* k_empty = k_full + C::STAGES;            // STAGES
    uint64_t* v_full = k_empty + C::STAGES;            // STAGES
    uint64_t* v_empty = v_full + C::STAGES;            // STAGES
    uint64_t* s_full = v_empty + C::STAGES;            // QT
    uint64_t* p_full = s_full + QT;                    // QT
    uint64_t* o_done = p_full + QT;                    // QT
    uint64_t* drain = o_done + QT;                     // 1
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Consecutive CTAs take the query blocks of one (batch, head), heaviest
    // (last, for causal) first, so the CTAs in flight share a few heads' K/V
    // in L2.  Causal launches hold back each head's `tail_qb` lightest query
    // blocks and run them last, heaviest first across heads, so the SMs that
    // finish early pick up short CTAs instead of a late full-length one.
    const uint32_t lead = (p.q_blocks - p.tail_qb) * p.splits * p.bh;
    uint32_t bh, qb;
    if (blockIdx.x < lead) {
        const uint32_t units = (p.q_blocks - p.tail_qb) * p.splits;
        bh = blockIdx.x / units;
        qb = p.q_blocks - 1 - (blockIdx.x % units) / p.splits;
    } else {  // splits == 1
        const uint32_t r = blockIdx.x - lead;
        qb = p.tail_qb - 1 - r / p.bh;
        bh = r % p.bh;
    }
    const uint32_t split = blockIdx.x % p.splits;
    const uint32_t j0 = split * p.split_tiles;  // first key tile of this CTA's range
    const uint32_t q0 = qb * (QT * TQ);
    // key tiles of this CTA's range visible to each Q tile (local indices
    // j = 0 .. n_t - 1 stand for key tiles j0 + j)
    uint32_t n_t[QT];
#pragma unroll
    for (int t = 0; t < QT; ++t) {
        const uint32_t vis_tiles = visible_tiles(p, q0 + t * TQ);
        n_t[t] = vis_tiles > j0 ? min(vis_tiles - j0, p.split_tiles) : 0u;
    }
    uint32_t n_kv = 0;
#pragma unroll
    for (int t = 0; t < QT; ++t) n_kv = max(n_kv, n_t[t]);
    const uint32_t batch = bh / p.H, head = bh % p.H;
    const int32_t kv_head = (int32_t)(head / (p.H / p.Hkv));
    // Tensor maps are 4-D {depth, rows, heads, batch}: rows past L / Lk read
    // as zeros, and any row / head / batch strides are followed.
    const int32_t k_b = p.k_batch_bcast ? 0 : (int32_t)batch, v_b = p.v_batch_bcast ? 0 : (int32_t)batch;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int t = 0; t < QT; ++t) {
            mbar_init(&s_full[t], 1);
            mbar_init(&p_full[t], 128);
            mbar_init(&o_done[t], 1);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        // The producer is this thread: the Q tiles and the first ring's K/V
        // (whose slots are free) load while TMEM is allocated and the block
        // synchronises.
        if (n_kv > 0) {
            mbar_arrive_expect_tx(q_full, QT * C::Q_BYTES);
            for (int t = 0; t < QT; ++t)
                for (int b = 0; b < C::BOXES; ++b)
                    tma_load_4d(sQ + t * C::Q_BYTES + b * (TQ * 128), &tmQ, b * 64, (int32_t)(q0 + t * TQ), (int32_t)head,
                                (int32_t)batch, q_full);
        }
        for (uint32_t j = 0; j < n_kv && j < (uint32_t)C::STAGES; ++j) {
            unsigned char* kd = sKV + j * C::STAGE_BYTES;
            mbar_arrive_expect_tx(&k_full[j], C::K_BYTES);
            for (int b = 0; b < C::BOXES; ++b)
                tma_load_4d(kd + b * (TK * 128), &tmK, b * 64, (int32_t)((j0 + j) * TK), kv_head, k_b, &k_full[j]);
            mbar_arrive_expect_tx(&v_full[j], C::V_BYTES);
            for (int b = 0; b < C::BOXES; ++b)
                tma_load_4d(kd + C::K_BYTES + b * (TK * 128), &tmV, b * 64, (int32_t)((j0 + j) * TK), kv_head, v_b,
                            &v_full[j]);
        }
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------ TMA producer
        // K and V have their own slots and barriers: K(j) is released once
        // both tiles' S(j) are computed, a key step before V(j), so the
        // next K tiles load two key steps ahead of their use.  The first
        // STAGES key tiles were issued before the block barrier.
        const uint32_t pre = n_kv < (uint32_t)C::STAGES ? n_kv : (uint32_t)C::STAGES;
        uint32_t issued_k = pre, issued_v = pre;
        bool failed = false;
        for (uint32_t j = pre; j < n_kv; ++j) {
            const uint32_t s = j % C::STAGES, ph = ((j / C::STAGES) & 1) ^ 1;
            unsigned char* kd = sKV + s * C::STAGE_BYTES;
            unsigned char* vd = kd + C::K_BYTES;
            if (!mbar_wait(&k_empty[s], ph)) {
                failed = true;
                break;
            }
            mbar_arrive_expect_tx(&k_full[s], C::K_BYTES);
            for (int b = 0; b < C::BOXES; ++b)
                tma_load_4d(kd + b * (TK * 128), &tmK, b * 64, (int32_t)((j0 + j) * TK), kv_head, k_b, &k_full[s]);
            ++issued_k;
            if (!mbar_wait(&v_empty[s], ph)) {
                failed = true;
                break;
            }
            mbar_arrive_expect_tx(&v_full[s], C::V_BYTES);
            for (int b = 0; b < C::BOXES; ++b)
                tma_load_4d(vd + b * (TK * 128), &tmV, b * 64, (int32_t)((j0 + j) * TK), kv_head, v_b, &v_full[s]);
            ++issued_v;
        }
        if (failed) {
            // drain the copies still in flight (bounded) before exiting
            atomicOr(&g_attn_status, 1u << DEV_ATTN_TIMEOUT);
            for (uint32_t j = issued_k >= C::STAGES ? issued_k - C::STAGES : 0; j < issued_k; ++j)
                (void)mbar_wait(&k_full[j % C::STAGES], (j / C::STAGES) & 1);
            for (uint32_t j = issued_v >= C::STAGES ? issued_v - C::STAGES : 0; j < issued_v; ++j)
                (void)mbar_wait(&v_full[j % C::STAGES], (j / C::STAGES) & 1);
        }
        if (n_kv > 0) (void)mbar_wait(q_full, 0);
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        // The whole warp runs this loop with warp-uniform operands and waits;
        // one elected lane issues each tcgen05.mma / commit.  Descriptors are
        // built once per group and advanced by constant byte offsets.
        const uint32_t idesc_s = f16_idesc(p.fmt, TQ, TK);
        const uint32_t idesc_o = f16_idesc(p.fmt, TQ, D) | (1u << 16);  // B (V) is MN-major
        auto wait = [](uint64_t* bar, uint32_t parity) { return __all_sync(0xffffffffu, mbar_wait(bar, parity)); };
        bool ok = n_kv == 0 || wait(q_full, 0);
        auto issue_s = [&](int t, uint32_t j) -> bool {
            const uint32_t s = j % C::STAGES;
            if (!wait(&k_full[s], (j / C::STAGES) & 1)) return false;
            tc_fence_after();
            const uint64_t qd = sw128_desc(smem_u32(sQ + t * C::Q_BYTES));
            const uint64_t kd = sw128_desc(smem_u32(sKV + s * C::STAGE_BYTES));
            const uint32_t d = tmem + C::s_col(t);
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
                const uint32_t off = (uint32_t)((k / 4) * (TQ * 128) + (k % 4) * 32);
                umma_f16_ss_warp(d, desc_add(qd, off), desc_add(kd, off), idesc_s, k != 0);
            }
            umma_commit_warp(&s_full[t]);
            return true;
        };
        auto issue_pv = [&](int t, uint32_t j) -> bool {
            const uint32_t s = j % C::STAGES;
            if (!wait(&v_full[s], (j / C::STAGES) & 1)) return false;
            if (!wait(&p_full[t], j & 1)) return false;
            tc_fence_after();
            const uint64_t vd = sw128_mn_desc(smem_u32(sKV + s * C::STAGE_BYTES + C::K_BYTES), TK * 128);
            const uint32_t d = tmem + C::o_col(t), a = tmem + C::s_col(t);
            umma_f16_ts_warp(d, a, vd, idesc_o, j != 0);
#pragma unroll
            for (int k = 1; k < TK / 16; ++k) umma_f16_ts_warp(d, a + k * 8, desc_add(vd, k * 16 * 128), idesc_o, 1u);
            if (j + 1 == n_t[t]) umma_commit_warp(&o_done[t]);
            return true;
        };
        for (int t = 0; t < QT && ok; ++t)
            if (n_t[t] > 0) ok = issue_s(t, 0);
        if (ok && n_kv > 0) umma_commit_warp(&k_empty[0]);  // K(0) consumed by every S(0)
        for (uint32_t j = 0; ok && j < n_kv; ++j) {
            for (int t = 0; t < QT && ok; ++t) {
                if (j >= n_t[t]) continue;
                ok = issue_pv(t, j);
                if (ok && j + 1 < n_t[t]) ok = issue_s(t, j + 1);
            }
            // V(j) is free once every PV(j) has completed, K(j + 1) once
            // every S(j + 1) has
            if (ok) umma_commit_warp(&v_empty[j % C::STAGES]);
            if (ok && j + 1 < n_kv) umma_commit_warp(&k_empty[(j + 1) % C::STAGES]);
        }
        if (!ok && lane == 0) atomicOr(&g_attn_status, 1u << DEV_ATTN_TIMEOUT);
        umma_commit_warp(drain);
        (void)wait(drain, 0);
    } else if (warp >= 2) {
        // ------------------------------------------------ softmax / epilogue
        const int t = (warp - 2) / 4;                  // Q tile of this warpgroup
        const int quarter = warp & 3;
        const uint32_t row = (uint32_t)(quarter * 32 + lane);
        const uint32_t q = q0 + t * TQ + row;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const uint32_t n = n_t[t];
        const int64_t vis = p.causal ? (int64_t)(q % p.q_mod) + (int64_t)p.causal_offset : (int64_t)1 << 40;
        const float NEG = -__int_as_float(0x7f800000);
        const float sl = p.scale_log2;
        float m_used = NEG;  // running max (log2 units)
        float l = 0.0f;
        bool ok = true;
        for (uint32_t j = 0; j < n && ok; ++j) {
            // Wait outcomes are made warp-uniform: tcgen05.ld/st are .sync.aligned.
            if (!__all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float x[TK];
            {
                uint32_t r[TK];
#pragma unroll
                for (int c = 0; c < TK / 32; ++c)
                    tmem_ld32(tmem + lane_base + C::s_col(t) + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < TK; ++i) x[i] = __uint_as_float(r[i]);
            }
            // Keys past the length or the causal edge are masked only in the
            // tiles that reach them; logits are x * sl, so the row maximum of
            // the logits is the maximum of x (sl > 0) or its minimum (sl < 0).
            const int64_t key0 = (int64_t)(j0 + j) * TK;
            const bool edge = MASK != FB_MASK_NONE || key0 + TK > (int64_t)p.Lk || key0 + TK - 1 > vis;
            if (edge || sl == 0.0f) {
                const int64_t lim64 = min((int64_t)p.Lk - key0, vis - key0 + 1);
                const int32_t lim = (int32_t)(lim64 < 0 ? 0 : (lim64 > TK ? TK : lim64));
                if constexpr (MASK == FB_MASK_NONE) {
#pragma unroll
                    for (int i = 0; i < TK; ++i) x[i] = i < lim ? x[i] * sl : NEG;  // logits, masked
                } else {
                    // This row's mask values for the tile's keys, 16 bytes at a
                    // time (keys contiguous; only keys < Lk of rows < L read).
                    const uint64_t mrow = (uint64_t)batch * p.m_sb + (uint64_t)head * p.m_sh + (uint64_t)q * p.m_sq + key0;
                    const bool row_ok = q < p.L;
#pragma unroll
                    for (int c = 0; c < TK / 4; ++c) {
                        uint4 mv = make_uint4(0u, 0u, 0u, 0u);
                        if (row_ok && c * 4 < lim)
                            mv = *reinterpret_cast<const uint4*>(static_cast<const uint32_t*>(p.mask) + mrow + c * 4);
                        const uint32_t mw[4] = {mv.x, mv.y, mv.z, mv.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int i = c * 4 + e;
                            if constexpr (MASK == FB_MASK_KEEP) {
                                x[i] = (i < lim && row_ok && mw[e] != 0u) ? x[i] * sl : NEG;
                            } else {
                                const float bias = __uint_as_float(mw[e]);
                                x[i] = (i < lim && row_ok && bias != NEG) ? fmaf(bias, 1.4426950408889634f, x[i] * sl) : NEG;
                            }
                        }
                    }
                }
            }
            const bool raw = !(edge || sl == 0.0f);
            const bool use_min = raw && sl < 0.0f;
            // Four chains of three-input extremes: 64 instructions per row.
            float mx[4] = {x[0], x[1], x[2], x[3]};
            if (use_min) {
#pragma unroll
                for (int i = 4; i < TK - 4; i += 8)
#pragma unroll
                    for (int a = 0; a < 4; ++a) mx[a] = min3n(mx[a], x[i + 2 * a], x[i + 2 * a + 1]);
                mx[0] = min3n(mx[0], x[TK - 4], x[TK - 3]);
                mx[1] = min3n(mx[1], x[TK - 2], x[TK - 1]);
            } else {
#pragma unroll
                for (int i = 4; i < TK - 4; i += 8)
#pragma unroll
                    for (int a = 0; a < 4; ++a) mx[a] = max3n(mx[a], x[i + 2 * a], x[i + 2 * a + 1]);
                mx[0] = max3n(mx[0], x[TK - 4], x[TK - 3]);
                mx[1] = max3n(mx[1], x[TK - 2], x[TK - 1]);
            }
            float mt = use_min ? min3n(min3n(mx[0], mx[1], mx[2]), mx[3], mx[3])
                               : max3n(max3n(mx[0], mx[1], mx[2]), mx[3], mx[3]);
            if (raw) mt *= sl;  // raw extreme -> logit maximum
            float alpha = 1.0f;
            bool rescale = false;
            if (mt > m_used + 8.0f) {
                alpha = m_used == NEG ? 0.0f : ex2(m_used - mt);
                rescale = j > 0 && l > 0.0f;
                m_used = mt;
            }
            const float base = m_used == NEG ? 0.0f : m_used + p.shift;
            // P = exp2(logit - base): one packed FFMA per score pair on the raw
            // path (the edge path subtracts exactly: z * 1 - base), then ex2 on
            // MUFU for seven pairs in eight and the paired polynomial for the
            // eighth.  (A quarter on the polynomial cut cycles per key step
            // but measured slower in time: more FMA-pipe work under the
            // power cap.)
            float2 lsa[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            // Packed pairs overwrite the scores they came from (element i of
            // a chunk is written after elements 2i and 2i+1 were read), so P
            // needs no registers of its own.
            uint32_t* xb = reinterpret_cast<uint32_t*>(x);
            const float2 sl2 = make_float2(raw ? sl : 1.0f, raw ? sl : 1.0f), nb2 = make_float2(-base, -base);
#pragma unroll
            for (int c = 0; c < TK / 32; ++c) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float2 z = __ffma2_rn(make_float2(x[c * 32 + 2 * i], x[c * 32 + 2 * i + 1]), sl2, nb2);
                    const float2 e = (i & 7) == 7 ? ex2_poly2(z) : make_float2(ex2(z.x), ex2(z.y));
                    if (!p.fmt) lsa[i & 3] = __fadd2_rn(lsa[i & 3], e);
                    xb[c * 32 + i] = pack2(e.x, e.y, p.fmt);
                }
                tmem_st16(tmem + lane_base + C::s_col(t) + c * 16, *reinterpret_cast<const uint32_t(*)[16]>(&xb[c * 32]));
            }
            if (__any_sync(0xffffffffu, rescale)) {
                // After P is out of the score registers: O_t is quiescent (S_t
                // of this tile completed after PV_t of the previous one, and
                // PV_t of this tile waits for the arrival below).  The whole
                // warp takes this branch (tcgen05.ld/st are .sync.aligned);
                // rows that keep their maximum scale by 1.
                const float f = rescale ? alpha : 1.0f;
#pragma unroll 1
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tmem + lane_base + C::o_col(t) + c * 32, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
                    tmem_st32(tmem + lane_base + C::o_col(t) + c * 32, r);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[t]);
            if (p.fmt) {  // BF16 P -> f32 is exact: the high half of the pattern
#pragma unroll
                for (int i = 0; i < TK / 2; ++i) {
                    const uint32_t w = xb[(i / 16) * 32 + (i % 16)];
                    lsa[i & 3] = __fadd2_rn(lsa[i & 3], make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u)));
                }
            }
            const float2 l2 = __fadd2_rn(__fadd2_rn(lsa[0], lsa[1]), __fadd2_rn(lsa[2], lsa[3]));
            const float ls = l2.x + l2.y;
            l = l * alpha + ls;
        }
        // epilogue: O / l, f32 rows
        if (ok && n > 0 && !__all_sync(0xffffffffu, mbar_wait(&o_done[t], 0))) ok = false;
        if (p.tma_out) {
            // Staged epilogue: once every MMA of both tiles has completed, the
            // K/V ring is idle; each thread writes its row of O / l there in
            // the 128-byte-swizzled boxes of the output's tensor map (128 rows
            // x 128 bytes each), and one thread writes the boxes by TMA tensor
            // stores instead of every thread storing its own row.
#pragma unroll
            for (int tt = 0; tt < QT; ++tt)
                if (tt != t && n_t[tt] > 0 && ok && !__all_sync(0xffffffffu, mbar_wait(&o_done[tt], 0))) ok = false;
            if (!ok) atomicOr(&g_attn_status, 1u << DEV_ATTN_TIMEOUT);
            tc_fence_after();
            const bool load = ok && n > 0;
            const float inv = (load && l > 0.0f) ? 1.0f / l : 0.0f;
            const uint32_t esz = p.out_low ? 2u : 4u;
            unsigned char* stage = sKV + (uint32_t)t * (TQ * D * esz);
            const uint32_t swz = row & 7u;
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                uint32_t r[32];
                if (load) {
                    tmem_ld32(tmem + lane_base + C::o_col(t) + c * 32, r);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = 0u;
                }
                if (p.out_low) {  // boxes of 64 16-bit values: chunk c is half of box c / 2
                    unsigned char* dst = stage + (c / 2) * (TQ * 128) + row * 128;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t j = (uint32_t)((c % 2) * 4 + i);
                        *reinterpret_cast<uint4*>(dst + ((j ^ swz) * 16)) = make_uint4(
                            encode_low_pair(__uint_as_float(r[8 * i]) * inv, __uint_as_float(r[8 * i + 1]) * inv, p.out_low),
                            encode_low_pair(__uint_as_float(r[8 * i + 2]) * inv, __uint_as_float(r[8 * i + 3]) * inv, p.out_low),
                            encode_low_pair(__uint_as_float(r[8 * i + 4]) * inv, __uint_as_float(r[8 * i + 5]) * inv, p.out_low),
                            encode_low_pair(__uint_as_float(r[8 * i + 6]) * inv, __uint_as_float(r[8 * i + 7]) * inv, p.out_low));
                    }
                } else {  // boxes of 32 f32 values
                    unsigned char* dst = stage + c * (TQ * 128) + row * 128;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        *reinterpret_cast<float4*>(dst + ((j ^ swz) * 16)) =
                            make_float4(__uint_as_float(r[4 * j]) * inv, __uint_as_float(r[4 * j + 1]) * inv,
                                        __uint_as_float(r[4 * j + 2]) * inv, __uint_as_float(r[4 * j + 3]) * inv);
                }
            }
            tc_fence_before();
            fence_proxy_async_smem();  // the staged rows are visible to the TMA store
            asm volatile("bar.sync 1, %0;" ::"r"(QT * 128) : "memory");  // every softmax warp's rows are staged
            if (warp == 2 && lane == 0) {
                const int boxes = p.out_low ? D / 64 : D / 32;
                for (int tt = 0; tt < QT; ++tt) {
                    if (q0 + tt * TQ >= p.L) continue;
                    for (int bx = 0; bx < boxes; ++bx)
                        tma_store_4d(&tmO, bx * (p.out_low ? 64 : 32), (int32_t)(q0 + tt * TQ), (int32_t)head,
                                     (int32_t)batch, sKV + tt * (TQ * D * esz) + bx * (TQ * 128));
                }
                bulk_commit_group();
                bulk_wait_read_all();  // shared memory stays valid until the stores have read it
            }
        } else {
        if (!ok) atomicOr(&g_attn_status, 1u << DEV_ATTN_TIMEOUT);
        tc_fence_after();
        // `ok` and n are warp-uniform, so the loads are too; only the stores
        // depend on whether this row exists (q < L).
        const bool load = ok && n > 0;
        float* orow = p.out + (uint64_t)batch * p.o_sb + (uint64_t)head * p.o_sh + (uint64_t)q * p.o_sl;
        float inv = (load && l > 0.0f) ? 1.0f / l : 0.0f;
        if (p.splits > 1) {
            // record {base, l, O} of this row and key range (O unnormalised)
            orow = p.part + (((uint64_t)bh * p.rec_rows + q) * p.splits + split) * (D + 2);
            if (q < p.L) {
                orow[0] = m_used == NEG ? 0.0f : m_used + p.shift;
                orow[1] = load ? l : 0.0f;
            }
            orow += 2;
            inv = 1.0f;
        }
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            if (load) {
                tmem_ld32(tmem + lane_base + C::o_col(t) + c * 32, r);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) r[i] = 0u;
            }
            if (q < p.L) {
                if (p.splits > 1) {  // records are 8-byte aligned
#pragma unroll
                    for (int i = 0; i < 32; i += 2)
                        *reinterpret_cast<float2*>(orow + c * 32 + i) =
                            make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1]));
                } else if (p.out_low) {  // 16-bit rows, 16-byte aligned (host)
                    uint4* dst = reinterpret_cast<uint4*>(low_row(p, batch, head, q) + c * 32);
#pragma unroll
                    for (int i = 0; i < 32; i += 8)
                        dst[i / 8] = make_uint4(
                            encode_low_pair(__uint_as_float(r[i]) * inv, __uint_as_float(r[i + 1]) * inv, p.out_low),
                            encode_low_pair(__uint_as_float(r[i + 2]) * inv, __uint_as_float(r[i + 3]) * inv, p.out_low),
                            encode_low_pair(__uint_as_float(r[i + 4]) * inv, __uint_as_float(r[i + 5]) * inv, p.out_low),
                            encode_low_pair(__uint_as_float(r[i + 6]) * inv, __uint_as_float(r[i + 7]) * inv, p.out_low));
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4*>(orow + c * 32 + i) =
                            make_float4(__uint_as_float(r[i]) * inv, __uint_as_float(r[i + 1]) * inv,
                                        __uint_as_float(r[i + 2]) * inv, __uint_as_float(r[i + 3]) * inv);
                }
            }
        }
        tc_fence_before();
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// Combines the key-range records of each query row: with M the largest base
// of the ranges that saw a key, O = sum O_s 2^(base_s - M) / sum l_s
// 2^(base_s - M) (the exponentials' common pre-scale cancels); rows with no
// visible key are 0, as in the unsplit kernel.  One warp per row.
template <int D>
__global__ void attn_merge_kernel(AttnParams p) {
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t total = (uint64_t)p.bh * p.L;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t w = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += warps) {
        const uint64_t bh = w / p.L, q = w % p.L;
        const float* rec = p.part + ((bh * p.rec_rows + q) * p.splits) * (D + 2);
        // the largest base of the ranges that saw a key, lanes over ranges
        float M = -__int_as_float(0x7f800000);
        for (uint32_t s = lane; s < p.splits; s += 32)
            if (rec[s * (D + 2) + 1] > 0.0f) M = fmaxf(M, rec[s * (D + 2)]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float L = 0.0f;
        float o[D / 32];
#pragma unroll
        for (int i = 0; i < D / 32; ++i) o[i] = 0.0f;
        // ranges in index order (four records' loads in flight at once)
#pragma unroll 4
        for (uint32_t s = 0; s < p.splits; ++s) {
            const float* r = rec + s * (D + 2);
            const float l = r[1];
            if (!(l > 0.0f)) continue;
            const float wgt = exp2f(r[0] - M);
            L = fmaf(l, wgt, L);
#pragma unroll
            for (int i = 0; i < D / 32; ++i) o[i] = fmaf(r[2 + i * 32 + lane], wgt, o[i]);
        }
        const uint32_t batch = (uint32_t)(bh / p.H), head = (uint32_t)(bh % p.H);
        const float inv = L > 0.0f ? 1.0f / L : 0.0f;
        if (p.out_low) {
            uint16_t* lrow = low_row(p, batch, head, (uint32_t)q);
#pragma unroll
            for (int i = 0; i < D / 32; ++i)
                lrow[i * 32 + lane] = p.out_low == FB_BF16 ? encode_bf16(o[i] * inv) : encode_f16(o[i] * inv);
        } else {
            float* orow = p.out + (uint64_t)batch * p.o_sb + (uint64_t)head * p.o_sh + q * p.o_sl;
#pragma unroll
            for (int i = 0; i < D / 32; ++i) orow[i * 32 + lane] = o[i] * inv;
        }
    }
}


// Short key ranges (Lk <= 256; the ViT encoder's 197 tokens) at depth 64.  A
// unit is one (batch, head, 128-query tile); CTAs are persistent (192
// threads, 256 TMEM columns, ~81 KB of shared memory, two per SM) and take
// units blockIdx.x, blockIdx.x + gridDim.x, ...
//   warp 0      TMA: per unit the Q tile with every key row of the head (one
//               or two 128-row boxes; rows past Lk read as zeros) as soon as
//               the previous unit's S has read Q and K, and the value rows as
//               soon as the previous unit's output has left the V buffer.
//   warp 1      one S = Q K^T group over all keys (N = Lk rounded up to 16,
//               at most 256) into TMEM columns [0, N), issued once the
//               softmax has read the previous unit's O out of TMEM; after the
//               softmax, one O = P V group (K = N) into columns [128, 128 + D).
//   warps 2-5   the softmax of one query row per thread in two passes over the
//               row in TMEM: the exact row maximum, then exp2 of every score,
//               P packed to 16-bit pairs over the scores already read (P of
//               keys 32c..32c+31 lands in columns 16c..16c+15, which pass 2
//               has read), and the sum of the rounded weights.  With the whole
//               row present there is no running maximum, no rescale and no
//               second S round trip; O overwrites S columns the softmax has
//               consumed.  Then O is read out of TMEM (which lets the next
//               unit's S start), O / l is staged in the V buffer (free once PV
//               is done) and written by TMA tensor stores.
// BF16 weights carry the same 2^-shift pre-scale as attn_fwd_kernel, so the
// numerator cannot overflow f32; fully masked rows (causal) produce zeros.
// SPLIT = 2 (key ranges of 177-208 rounded to 192 or 208 columns, the
// encoder's 197): two softmax warps per TMEM lane quarter (320 threads, 92
// registers), one over keys 0-127 and one over the rest, exchanging the row's
// partial maximum and sum through shared memory behind a 64-thread named
// barrier per quarter, each storing half of O.  The first warp's P goes over
// its own consumed S columns as above; the second's goes to the free columns
// [nkp, 256), so neither overwrites scores the other has still to read, and
// the PV group takes key steps 8.. from there.  Halving each row's softmax
// chain: C5 attention 48.0 -> 41.8 us, C5 forward 2.94 -> 2.86 ms.
constexpr int SD = 64;                          // depth
constexpr int S_Q_BYTES = TQ * SD * 2;          // 16 KB
constexpr int S_KV_BYTES = 2 * TK * SD * 2;     // 32 KB: up to 256 rows
constexpr uint32_t S_TMEM_COLS = 256;
constexpr uint32_t S_O_COL = 128;
template <int SPLIT>
struct SCfg {
    static constexpr int THREADS = 64 + 128 * SPLIT;
    static constexpr int XCH_BYTES = SPLIT == 2 ? 2 * 2 * TQ * 4 : 0;  // partial maxima and sums
    static constexpr int SMEM = 1024 + S_Q_BYTES + 2 * S_KV_BYTES + 128 + XCH_BYTES;
};

// 1 when every calling thread's `v` is true (bar.red over `n` threads of named barrier 1).
__device__ __forceinline__ bool bar_all1(int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred q, a;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred a, 1, %2, q;\n\tselp.u32 %0, 1, 0, a;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(n)
        : "memory");
    return r != 0;
}

// 64-thread named barrier 2 + q (literal ids, so the kernel reserves six barriers, not sixteen).
__device__ __forceinline__ void pair_sync(int id) {
    switch (id) {
        case 2: asm volatile("bar.sync 2, 64;" ::: "memory"); break;
        case 3: asm volatile("bar.sync 3, 64;" ::: "memory"); break;
        case 4: asm volatile("bar.sync 4, 64;" ::: "memory"); break;
        default: asm volatile("bar.sync 5, 64;" ::: "memory"); break;
    }
}

template <int SPLIT>
__global__ void __launch_bounds__(SCfg<SPLIT>::THREADS, 2) attn_short_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                                             const __grid_constant__ CUtensorMap tmK,
                                                                             const __grid_constant__ CUtensorMap tmV,
                                                                             const __grid_constant__ CUtensorMap tmO, AttnParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sQ = smem;
    unsigned char* sK = sQ + S_Q_BYTES;
    unsigned char* sV = sK + S_KV_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sV + S_KV_BYTES);
    uint64_t* qk_full = bars;       // Q and K of the unit landed
    uint64_t* qk_empty = bars + 1;  // S of the unit computed: Q and K may reload
    uint64_t* v_full = bars + 2;
    uint64_t* v_empty = bars + 3;   // the unit's output has left the V buffer
    uint64_t* s_full = bars + 4;
    uint64_t* p_full = bars + 5;    // 128 arrivals
    uint64_t* o_full = bars + 6;
    uint64_t* o_free = bars + 7;    // 128 arrivals: O read out of TMEM
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
    float* xch = reinterpret_cast<float*>(sV + S_KV_BYTES + 128);  // SPLIT 2: [2 halves][TQ] maxima, then sums

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t units = p.q_blocks * p.bh;
    const uint32_t nkb = p.kv_tiles;                      // 128-row key boxes (1 or 2)
    const uint32_t nkp = (p.Lk + 15u) & ~15u;             // keys rounded up to the MMA's N step

    if (threadIdx.x == 0) {
        for (int b = 0; b < 8; ++b) mbar_init(&bars[b], b == 5 || b == 7 ? 128 * SPLIT : 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, S_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            bool failed = false;
            uint32_t k = 0;
            for (uint32_t u = blockIdx.x; u < units; u += gridDim.x, ++k) {
                const uint32_t bh = u / p.q_blocks, qb = u % p.q_blocks;
                const uint32_t batch = bh / p.H, head = bh % p.H;
                const int32_t kv_head = (int32_t)(head / (p.H / p.Hkv));
                const int32_t k_b = p.k_batch_bcast ? 0 : (int32_t)batch, v_b = p.v_batch_bcast ? 0 : (int32_t)batch;
                if (!mbar_wait(qk_empty, (k & 1) ^ 1)) {
                    failed = true;
                    break;
                }
                mbar_arrive_expect_tx(qk_full, (uint32_t)(S_Q_BYTES + nkb * TK * SD * 2));
                tma_load_4d(sQ, &tmQ, 0, (int32_t)(qb * TQ), (int32_t)head, (int32_t)batch, qk_full);
                for (uint32_t b = 0; b < nkb; ++b)
                    tma_load_4d(sK + b * (TK * 128), &tmK, 0, (int32_t)(b * TK), kv_head, k_b, qk_full);
                if (!mbar_wait(v_empty, (k & 1) ^ 1)) {
                    failed = true;
                    break;
                }
                mbar_arrive_expect_tx(v_full, (uint32_t)(nkb * TK * SD * 2));
                for (uint32_t b = 0; b < nkb; ++b)
                    tma_load_4d(sV + b * (TK * 128), &tmV, 0, (int32_t)(b * TK), kv_head, v_b, v_full);
            }
            // every copy this thread issued is consumed before the CTA's
            // final barrier; after a failed wait, drain them (bounded)
            if (failed) {
                atomicOr(&g_attn_status, 1u << DEV_ATTN_TIMEOUT);
                if (k > 0) (void)mbar_wait(v_full, (k - 1) & 1);
                (void)mbar_wait(qk_full, k & 1);
            }
        }
    } else if (warp == 1) {
        auto wait = [](uint64_t* bar, uint32_t parity) { return __all_sync(0xffffffffu, mbar_wait(bar, parity)); };
        const uint32_t idesc_s = f16_idesc(p.fmt, TQ, nkp);
        const uint32_t idesc_o = f16_idesc(p.fmt, TQ, SD) | (1u << 16);  // B (V) is MN-major
        const uint64_t qd = sw128_desc(smem_u32(sQ)), kd = sw128_desc(smem_u32(sK));
        const uint64_t vd = sw128_mn_desc(smem_u32(sV), TK * 128);
        bool ok = true;
        uint32_t k = 0;
        for (uint32_t u = blockIdx.x; ok && u < units; u += gridDim.x, ++k) {
            // S overwrites the previous unit's O columns: wait until they are read
            ok = wait(qk_full, k & 1) && wait(o_free, (k & 1) ^ 1);
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < SD / 16; ++kk)
                umma_f16_ss_warp(tmem, desc_add(qd, (uint32_t)(kk * 32)), desc_add(kd, (uint32_t)(kk * 32)), idesc_s, kk != 0);
            umma_commit_warp(s_full);
            umma_commit_warp(qk_empty);
            ok = wait(v_full, k & 1) && wait(p_full, k & 1);
            if (!ok) break;
            tc_fence_after();
            for (uint32_t kk = 0; kk < nkp / 16; ++kk) {
                const uint32_t pcol = SPLIT == 2 && kk >= 8 ? nkp + (kk - 8) * 8 : kk * 8;
                umma_f16_ts_warp(tmem + S_O_COL, tmem + pcol, desc_add(vd, kk * 16 * 128), idesc_o, kk != 0);
            }
            umma_commit_warp(o_full);
        }
        if (!ok && lane == 0) atomicOr(&g_attn_status, 1u << DEV_ATTN_TIMEOUT);
    } else {
        const int quarter = warp & 3;
        const int half = SPLIT == 2 ? (warp - 2) >> 2 : 0;      // SPLIT 2: keys 0-127 / 128..
        const uint32_t row = (uint32_t)(quarter * 32 + lane);
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const float NEG = -__int_as_float(0x7f800000);
        const float sl = p.scale_log2;
        const uint32_t nch = (nkp + 31u) / 32u;                 // 32-column chunks holding keys
        const uint32_t cb = SPLIT == 2 && half ? 4u : 0u;       // this warp's chunks [cb, ce)
        const uint32_t ce = SPLIT == 2 && !half ? min(nch, 4u) : nch;
        constexpr uint32_t CH1 = SPLIT == 2 ? 2u : 4u;          // chunks per TMEM round trip in pass 1
        constexpr int OC = SD / SPLIT;                          // O columns this warp reads and stores
        const bool neg = sl < 0.0f;                               // logit maximum = min(x) * sl
        const bool storer = warp == 2 && lane == 0;
        const int pair_bar = 2 + quarter;                         // SPLIT 2: the quarter's two warps
        bool ok = true;
        uint32_t k = 0;
        for (uint32_t u = blockIdx.x; ok && u < units; u += gridDim.x, ++k) {
            const uint32_t bh = u / p.q_blocks, qb = u % p.q_blocks;
            const uint32_t q0 = qb * TQ, q = q0 + row;
            const int64_t vis = p.causal ? (int64_t)(q % p.q_mod) + (int64_t)p.causal_offset : (int64_t)1 << 40;
            const int64_t lim64 = min((int64_t)p.Lk, vis + 1);
            const int32_t lim = (int32_t)(lim64 < 0 ? 0 : lim64);   // keys [0, lim) of this row are visible
            float l = 0.0f;
            // A failed wait is warp-uniform but not CTA-uniform: the warp still
            // meets the other softmax warps at every named barrier (zeros for
            // its rows), and all of them leave the loop together after the
            // epilogue's barrier, which ANDs their outcomes.
            bool good = __all_sync(0xffffffffu, mbar_wait(s_full, k & 1));
            float ext = neg ? -NEG : NEG;
            if (good) {
                tc_fence_after();
                // pass 1: the extreme of the visible scores, CH1 chunks per TMEM
                // round trip; only chunks that reach past the row's last visible
                // key are masked element by element
                for (uint32_t c0 = cb; c0 < ce; c0 += CH1) {
                    // chunks past ce are loaded too (every chunk lies inside the
                    // 256 allocated columns) and ignored: loads under a condition
                    // make the compiler keep two copies of the chunk registers
                    uint32_t r[CH1][32];
#pragma unroll
                    for (uint32_t b = 0; b < CH1; ++b)
                        tmem_ld32(tmem + lane_base + (c0 + b) * 32, r[b]);
                    tmem_wait_ld();
#pragma unroll
                    for (uint32_t b = 0; b < CH1; ++b) {
                        if (c0 + b >= ce) break;
                        const int key0 = (int)((c0 + b) * 32);
                        if (key0 + 32 <= lim) {
                            float e0 = ext, e1 = ext;
#pragma unroll
                            for (int i = 0; i < 32; i += 4) {
                                const float a0 = __uint_as_float(r[b][i]), a1 = __uint_as_float(r[b][i + 1]);
                                const float a2 = __uint_as_float(r[b][i + 2]), a3 = __uint_as_float(r[b][i + 3]);
                                e0 = neg ? min3n(e0, a0, a1) : max3n(e0, a0, a1);
                                e1 = neg ? min3n(e1, a2, a3) : max3n(e1, a2, a3);
                            }
                            ext = neg ? fminf(e0, e1) : fmaxf(e0, e1);
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (key0 + i < lim) ext = neg ? fminf(ext, __uint_as_float(r[b][i])) : fmaxf(ext, __uint_as_float(r[b][i]));
                        }
                    }
                }
            }
            if constexpr (SPLIT == 2) {  // the row's extreme from both halves
                xch[half * TQ + row] = ext;
                pair_sync(pair_bar);
                const float other = xch[(half ^ 1) * TQ + row];
                ext = neg ? fminf(ext, other) : fmaxf(ext, other);
            }
            if (good) {
                const float mt = lim == 0 ? NEG : ext * sl;
                const float base = mt == NEG ? 0.0f : mt + p.shift;
                const float2 sl2 = make_float2(sl, sl), nb2 = make_float2(-base, -base);
                // pass 2: P = exp2(x * sl - base) over the visible keys, 0 elsewhere,
                // two chunks per TMEM round trip
                float2 lsa[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                for (uint32_t c0 = cb; c0 < ce; c0 += 2) {
                    uint32_t r[2][32];
#pragma unroll
                    for (int b = 0; b < 2; ++b)
                        tmem_ld32(tmem + lane_base + (c0 + b) * 32, r[b]);
                    tmem_wait_ld();
#pragma unroll
                    for (int b = 0; b < 2; ++b) {
                        if (c0 + b >= ce) break;
                        const int key0 = (int)((c0 + b) * 32);
                        const bool full = key0 + 32 <= lim;
                        uint32_t pk[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            float2 z = __ffma2_rn(make_float2(__uint_as_float(r[b][2 * i]), __uint_as_float(r[b][2 * i + 1])), sl2, nb2);
                            if (!full) {
                                z.x = key0 + 2 * i < lim ? z.x : NEG;
                                z.y = key0 + 2 * i + 1 < lim ? z.y : NEG;
                            }
                            const float2 e = (i & 7) == 7 ? ex2_poly2(z) : make_float2(ex2(z.x), ex2(z.y));
                            pk[i] = pack2(e.x, e.y, p.fmt);
                            lsa[i & 1] = __fadd2_rn(lsa[i & 1], e);
                        }
                        // P of keys 32c..32c+31: columns 16c.. (scores this warp
                        // has read), or for the second half [nkp + 16(c - 4), ..)
                        const uint32_t pc = SPLIT == 2 && half ? nkp + (c0 + b - 4u) * 16u : (c0 + b) * 16u;
                        tmem_st16(tmem + lane_base + pc, pk);
                    }
                }
                tmem_wait_st();
                const float2 l2 = __fadd2_rn(lsa[0], lsa[1]);
                l = l2.x + l2.y;
                tc_fence_before();
                mbar_arrive(p_full);
                good = __all_sync(0xffffffffu, mbar_wait(o_full, k & 1));
            }
            uint32_t o[OC];
            if (good) {
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < OC / 32; ++c)
                    tmem_ld32(tmem + lane_base + S_O_COL + half * OC + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&o[c * 32]));
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(o_free);  // the next unit's S may overwrite O's columns
            } else {
#pragma unroll
                for (int i = 0; i < OC; ++i) o[i] = 0u;
                l = 0.0f;
            }
            if constexpr (SPLIT == 2) {  // the row's sum from both halves
                xch[(2 + half) * TQ + row] = l;
                pair_sync(pair_bar);
                l += xch[(2 + (half ^ 1)) * TQ + row];
            }
            // Epilogue: O / l staged in the V buffer (PV has read it) in the
            // 128-byte-swizzled layout of the output's tensor map, then written
            // by one TMA tensor store per 128-byte-wide box (rows past L are
            // clipped by the map); the V buffer is handed back to the producer
            // once the stores have read it.  Each warp stages its OC columns.
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            const uint32_t swz = row & 7;
            if (p.out_low) {
                unsigned char* dst = sV + row * 128;  // one box: 64 16-bit values per row
#pragma unroll
                for (int j = 0; j < OC / 8; ++j) {
                    const int jj = half * (OC / 8) + j;  // 16-byte unit of the row
                    *reinterpret_cast<uint4*>(dst + ((jj ^ swz) * 16)) = make_uint4(
                        encode_low_pair(__uint_as_float(o[8 * j]) * inv, __uint_as_float(o[8 * j + 1]) * inv, p.out_low),
                        encode_low_pair(__uint_as_float(o[8 * j + 2]) * inv, __uint_as_float(o[8 * j + 3]) * inv, p.out_low),
                        encode_low_pair(__uint_as_float(o[8 * j + 4]) * inv, __uint_as_float(o[8 * j + 5]) * inv, p.out_low),
                        encode_low_pair(__uint_as_float(o[8 * j + 6]) * inv, __uint_as_float(o[8 * j + 7]) * inv, p.out_low));
                }
            } else {
#pragma unroll
                for (int b = 0; b < OC / 32; ++b) {  // boxes of 32 f32 per row
                    unsigned char* dst = sV + (half * (OC / 32) + b) * (TQ * 128) + row * 128;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        *reinterpret_cast<float4*>(dst + ((j ^ swz) * 16)) =
                            make_float4(__uint_as_float(o[32 * b + 4 * j]) * inv, __uint_as_float(o[32 * b + 4 * j + 1]) * inv,
                                        __uint_as_float(o[32 * b + 4 * j + 2]) * inv, __uint_as_float(o[32 * b + 4 * j + 3]) * inv);
                }
            }
            fence_proxy_async_smem();
            // every softmax warp's rows are staged; all of them continue only if all were good
            const bool all_good = bar_all1(128 * SPLIT, good);
            if (storer) {
                const uint32_t batch = bh / p.H, head = bh % p.H;
                const int boxes = p.out_low ? 1 : SD / 32;
                for (int b = 0; b < boxes; ++b)
                    tma_store_4d(&tmO, b * (p.out_low ? 64 : 32), (int32_t)q0, (int32_t)head, (int32_t)batch,
                                 sV + b * (TQ * 128));
                bulk_commit_group();
                bulk_wait_read_all();  // the V buffer stays valid until the stores have read it
                mbar_arrive(v_empty);
            }
            if (!all_good) ok = false;
        }
        if (!ok) atomicOr(&g_attn_status, 1u << DEV_ATTN_TIMEOUT);
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S_TMEM_COLS);
    }
}

// ------------------------------------------------------------------ host

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled_attn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// One operand's rows as a 4-D box source {depth, rows, heads, batch}: element
// strides of the row, head and (merged) batch axes; unit axes may have any
// stride and a stride-0 batch axis (broadcast) becomes a single batch index.
struct RowsLayout {
    uint64_t rows = 0, heads = 1, batch = 1;
    uint64_t s_row = 0, s_head = 0, s_batch = 0;
    bool batch_bcast = false;
};

// Merges the batch axes [0, nb) of the row nest into one (count, stride):
// the non-unit axes must nest row-major (stride[i] = stride[i+1] * dim[i+1])
// or all have stride 0 (broadcast).
bool merge_batch(const AttnArgs& a, const uint64_t* st, int nb, RowsLayout* o) {
    uint64_t count = 1, stride = 0;
    bool any = false, all_zero = true;
    int last = -1;
    for (int i = nb - 1; i >= 0; --i) {
        if (a.row_dims[i] == 1) continue;
        count *= a.row_dims[i];
        if (st[i] != 0) all_zero = false;
        if (!any) {
            stride = st[i];
            any = true;
        } else if (st[i] != st[last] * a.row_dims[last]) {
            if (!(st[i] == 0 && st[last] == 0)) return false;
        }
        last = i;
    }
    if (any && all_zero) {
        o->batch = 1;
        o->s_batch = 0;
        o->batch_bcast = true;
        return true;
    }
    if (any && stride == 0) return false;  // mixed broadcast and strided batch axes
    o->batch = count;
    o->s_batch = stride;
    return true;
}

// [batch, heads, rows, D] 16-bit operand, box {64, box_rows, 1, 1}, 128B swizzle.
bool make_rows_map(CUtensorMap* map, const void* ptr, uint32_t fmt, uint64_t D, const RowsLayout& l, uint32_t box_rows) {
    auto enc = encode_tiled_attn();
    if (!enc) return false;
    cuuint64_t dims[4] = {D, l.rows, l.heads, l.batch};
    // byte strides of dims 1..3; unit dims get any valid stride (16-byte multiple)
    uint64_t sb[3] = {l.s_row * 2, l.s_head * 2, l.s_batch * 2};
    uint64_t filler = (D * 2 + 15) / 16 * 16;
    for (int i = 0; i < 3; ++i) {
        if (dims[i + 1] == 1 && (sb[i] == 0 || sb[i] % 16 != 0 || sb[i] >= (1ull << 40))) sb[i] = filler;
        if (sb[i] == 0 || sb[i] % 16 != 0 || sb[i] >= (1ull << 40)) return false;
        filler = sb[i] * dims[i + 1];
        filler = (filler + 15) / 16 * 16;
        if (filler >= (1ull << 40)) filler = 16;
    }
    cuuint64_t strides[3] = {sb[0], sb[1], sb[2]};
    cuuint32_t box[4] = {64, box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    for (int i = 0; i < 4; ++i)
        if (dims[i] == 0 || dims[i] > (1ull << 31)) return false;
    return enc(map, fmt ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(ptr),
               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_out_map(CUtensorMap* map, void* ptr, uint32_t out_low, uint64_t D, const RowsLayout& l);

// L rows per head over H heads sharing Hkv key/value heads; q_mod < L when
// a GQA group's heads are packed into the rows of one head (row % q_mod is
// the query index).
template <int D, int QT>
int launch_d(const AttnArgs& a, uint32_t fmt, const RowsLayout& ql, const RowsLayout& kl, const RowsLayout& vl,
             const RowsLayout& ol, const RowsLayout& ml, uint64_t L, uint64_t H, uint64_t Hkv, uint64_t q_mod,
             cudaStream_t st) {
    using C = ACfg<D, QT>;
    const uint64_t Lk = a.keys;
    const uint64_t BH = a.rows / L;
    CUtensorMap tq, tk, tv;
    const void* q = static_cast<const uint16_t*>(a.q) + a.q_offset;
    const void* k = static_cast<const uint16_t*>(a.k) + a.k_offset;
    const void* v = static_cast<const uint16_t*>(a.v) + a.v_offset;
    if (!make_rows_map(&tq, q, fmt, D, ql, TQ) || !make_rows_map(&tk, k, fmt, D, kl, TK) ||
        !make_rows_map(&tv, v, fmt, D, vl, TK))
        return FB_ERR_UNSUPPORTED;
    AttnParams p{};
    p.fmt = fmt;
    p.L = (uint32_t)L;
    p.Lk = (uint32_t)Lk;
    p.H = (uint32_t)H;
    p.Hkv = (uint32_t)Hkv;
    p.q_blocks = (uint32_t)((L + QT * TQ - 1) / (QT * TQ));
    p.q_mod = (uint32_t)q_mod;
    p.bh = (uint32_t)BH;
    p.kv_tiles = (uint32_t)((Lk + TK - 1) / TK);
    p.scale_log2 = a.scale * 1.4426950408889634f;
    // P pre-scale for BF16: 2^-(9 + ceil(log2(keys))) keeps sum(P) * max|V|
    // below max|V| (BF16 shares f32's exponent range, so P stays normal).
    // F16 values are bounded by 65504 and the numerator cannot approach the
    // f32 range, while a pre-scale would push P into F16 subnormals: none.
    p.shift = fmt ? 9.0f + std::ceil(std::log2((float)std::max<uint64_t>(Lk, 1))) : 0.0f;
    p.causal = a.causal ? 1 : 0;
    p.causal_offset = a.causal_offset;
    p.k_batch_bcast = kl.batch_bcast ? 1 : 0;
    p.v_batch_bcast = vl.batch_bcast ? 1 : 0;
    p.out = a.out_low ? reinterpret_cast<float*>(reinterpret_cast<uint16_t*>(a.out) + a.o_offset) : a.out + a.o_offset;
    p.out_low = a.out_low;
    p.o_sb = ol.s_batch;
    p.o_sh = ol.s_head;
    p.o_sl = ol.s_row;
    p.mask = a.mask_kind == FB_MASK_NONE ? nullptr : static_cast<const uint32_t*>(a.mask) + a.m_offset;
    p.m_sb = ml.s_batch;
    p.m_sh = ml.s_head;
    p.m_sq = ml.s_row;
    auto kernel = a.mask_kind == FB_MASK_KEEP       ? attn_fwd_kernel<D, FB_MASK_KEEP, QT>
                  : a.mask_kind == FB_MASK_ADDITIVE ? attn_fwd_kernel<D, FB_MASK_ADDITIVE, QT>
                                                    : attn_fwd_kernel<D, FB_MASK_NONE, QT>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
        return launch_status("shared-memory attribute");
    uint64_t grid = (uint64_t)p.q_blocks * BH;
    if (grid == 0) return FB_OK;
    // Fewer CTAs than one wave over long key ranges (decode of a few
    // heads): split each CTA's key tiles so that about four waves of CTAs
    // exist, at least two tiles per range.  A key step costs the same
    // however few query rows are valid, so splitting pays only while SMs
    // would otherwise idle (measured: B=8 x 32 heads x 8192 keys, 256 CTAs,
    // is slower split).
    p.splits = 1;
    p.split_tiles = p.kv_tiles;
    p.rec_rows = (uint32_t)L;  // records exist only for rows q < L
    const uint64_t slots = (uint64_t)sm_count() * (QT == 1 ? 2 : 1);
    if (grid < slots && p.kv_tiles >= 4) {
        uint64_t splits = (4 * slots + grid - 1) / grid;
        if (splits > p.kv_tiles / 2) splits = p.kv_tiles / 2;
        const uint64_t tiles = (p.kv_tiles + splits - 1) / splits;
        splits = (p.kv_tiles + tiles - 1) / tiles;
        const uint64_t bytes = BH * p.rec_rows * splits * (D + 2) * sizeof(float);
        float* part = splits > 1 ? static_cast<float*>(scratch(st, bytes, SCRATCH_ATTN_SPLIT)) : nullptr;
        if (part) {  // none (e.g. first use inside a graph capture): whole ranges
            p.splits = (uint32_t)splits;
            p.split_tiles = (uint32_t)tiles;
            p.part = part;
            grid *= splits;
        } else {
            (void)cudaGetLastError();
        }
    }
    if (grid > 0x7fffffffull) return FB_ERR_UNSUPPORTED;
    // whole ranges: the output through a TMA map where its layout allows one
    CUtensorMap to{};
    p.tma_out = p.splits == 1 && make_out_map(&to, p.out, p.out_low, D, ol) ? 1u : 0u;
    p.tail_qb = 0;
    if (p.causal && p.splits == 1 && p.q_blocks >= 4 && grid > 2 * slots) {
        uint32_t t = (uint32_t)((2 * slots + BH - 1) / BH);
        p.tail_qb = std::min<uint32_t>(t, p.q_blocks / 4);
    }
    kernel<<<(unsigned)grid, C::THREADS, C::SMEM, st>>>(tq, tk, tv, to, p);
    count_launch(kernel_name("attn_fwd_kernel", {D, (int)a.mask_kind, QT}).c_str());
    if (p.splits > 1) {
        if (cudaGetLastError() != cudaSuccess) return launch_status("kernel launch");
        const uint64_t rows = BH * L;
        const unsigned mgrid = (unsigned)std::min<uint64_t>((rows + 7) / 8, (uint64_t)sm_count() * 16);
        attn_merge_kernel<D><<<mgrid, 256, 0, st>>>(p);
        count_launch(kernel_name("attn_merge_kernel", {D}).c_str());
    }
    return launch_status("kernel launch");
}


// ---------------------------------------------------------------- decode
// Decode-shaped 16-bit attention: the G x L query rows that share one key/
// value head (G query heads of a GQA group, L <= 16 / G queries each) form a
// single 16-row block, and every key is read once from HBM for all of them.
// A 128-row tcgen05 tile would carry at most 16 valid rows and its per-key
// softmax cost is that of 128 rows, so this path runs the block on the warp-
// level tensor-core MMA (m16n8k16, f32 accumulation) with the operands loaded
// straight from global memory into registers: the kernel is bound by the
// K/V read (HBM), not by arithmetic.
//   A CTA owns one key range of one (batch, key/value head); each of its four
//   warps walks a quarter of it 16 keys at a time, the keys streamed through
//   its own three-stage cp.async ring in shared memory (two stages in flight
//   while one is consumed): S = Q K^T (two n8 tiles, D/16 k-steps), online
//   softmax on the accumulator fragments (row maxima over the four lanes of a
//   row), P packed to 16-bit pairs in registers as the A operand of O += P V
//   (D/8 n8 tiles).  The four warps combine their partial results through
//   shared memory and the CTA leaves {base, l, O[D]} per query row for
//   attn_merge_kernel, as the key-split tensor-core path does.
//   Depth permutation: the contraction over the depth is order-free, so lane
//   (g, c) (g = lane / 4, c = lane % 4) takes as its k-step s operand words the
//   depth pairs (c*D/4 + 4s, +1) and (c*D/4 + 4s + 2, +3) of Q and K: every
//   lane's Q and K fragments are one contiguous D/4-value run per row (16-byte
//   loads).  Likewise the output columns of PV tile j are permuted so that
//   lane group g supplies V columns g*D/8 .. g*D/8 + D/8 - 1 (contiguous) and
//   lane (g, c) receives O columns [2c*D/8, (2c+2)*D/8) of its rows.
//   BF16 weights carry the 2^-shift pre-scale of attn_fwd_kernel (no f32
//   overflow for V near the format's maximum); the row sum adds the rounded
//   weights the MMA multiplies.
struct Dec16Params {
    const uint16_t* q;
    const uint16_t* k;
    const uint16_t* v;
    uint64_t q_sb, q_sh, q_sl;  // element strides: batch, head, query row (depth contiguous)
    uint64_t k_sb, k_sh, k_sk;  // batch (0: shared), key/value head, key
    uint64_t v_sb, v_sh, v_sk;
    uint32_t H, Hkv, G, L, Lk;
    uint32_t splits, keys_per_split;  // CTAs (key ranges) per (batch, key/value head); keys per warp
    float scale_log2, shift;
    int32_t causal, causal_offset;
    float* part;  // records [((batch * H + head) * L + query) * splits + range] x {base, l, O[D]}
    // cluster != 0: a unit's `splits` CTAs form one thread-block cluster and
    // merge their records through distributed shared memory, each writing some
    // of the output rows (no records in global memory, no merge launch)
    uint32_t cluster;
    void* out;
    uint32_t out_low;           // 0: f32 rows; FB_BF16 / FB_F16: rounded once (nearest even)
    uint64_t o_sb, o_sh, o_sl;  // output strides (elements of the output type)
};

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

template <int FMT>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    if constexpr (FMT == 1)
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int FMT>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
    if constexpr (FMT == 1) return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    else return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

constexpr int DEC_WARPS = 4;
constexpr int DEC_STAGES = 3;  // 16-key stages per warp: two in flight while one is consumed

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Shared-memory positions (16-byte chunks) of a stage's K and V rows: XOR
// swizzles under which every 8-lane phase of the fragment reads below touches
// eight distinct 16-byte bank groups.  K: lane (g, c) reads chunks
// c*D/32 .. of rows g and 8 + g; V: chunk(s) g*D/64 .. of rows 2c, 2c+1,
// 2c+8, 2c+9.
template <int D>
__device__ __forceinline__ uint32_t k_chunk(uint32_t row, uint32_t chunk) {
    if constexpr (D == 128) return chunk ^ (((chunk >> 3) & 1u) | ((row & 1u) << 1));
    else return chunk ^ (row & 1u);
}
__device__ __forceinline__ uint32_t v_chunk(uint32_t row, uint32_t chunk) { return chunk ^ (((row >> 1) & 3u) << 1); }

template <int D, int FMT>
__global__ void __launch_bounds__(32 * DEC_WARPS) attn_decode16_kernel(Dec16Params p) {
    constexpr int QW = D / 8;    // operand words (16-bit pairs) per lane per row: D / 4 values
    constexpr int KS = D / 16;   // k-steps of S
    constexpr int NJ = D / 8;    // n8 tiles of O
    constexpr int CPR = D / 8;   // 16-byte chunks per K / V row
    constexpr int STAGE = 2 * 16 * CPR;  // chunks per stage: 16 K rows then 16 V rows
    extern __shared__ uint4 dsm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    uint4* ring = dsm + (size_t)warp * DEC_STAGES * STAGE;
    const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
    const uint32_t unit = blockIdx.x / p.splits;  // (batch, key/value head)
    const uint32_t split = blockIdx.x % p.splits;  // this CTA's key range; warp w takes its w-th quarter
    const uint32_t b = unit / p.Hkv, hkv = unit % p.Hkv;
    const uint32_t R = p.G * p.L;
    const uint32_t k_begin = min((split * DEC_WARPS + warp) * p.keys_per_split, p.Lk);
    const uint32_t k_end = min(k_begin + p.keys_per_split, p.Lk);  // may be empty: the warp only joins the combine
    const float NEG = -__int_as_float(0x7f800000);

    // Q fragments of rows g and g + 8 (zeros past R)
    uint32_t qa[2][QW];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const uint32_t r = (uint32_t)(g + 8 * rr);
        if (r < R) {
            const uint32_t h = hkv * p.G + r / p.L, l = r % p.L;
            const uint4* src = reinterpret_cast<const uint4*>(p.q + b * p.q_sb + h * p.q_sh + l * p.q_sl + c * (D / 4));
#pragma unroll
            for (int i = 0; i < QW / 4; ++i) {
                const uint4 w = src[i];
                qa[rr][4 * i] = w.x, qa[rr][4 * i + 1] = w.y, qa[rr][4 * i + 2] = w.z, qa[rr][4 * i + 3] = w.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < QW; ++i) qa[rr][i] = 0u;
        }
    }
    // causal visibility of rows g, g + 8: key <= query + offset
    int64_t vis[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const uint32_t r = (uint32_t)(g + 8 * rr);
        vis[rr] = r >= R ? -1 : p.causal ? (int64_t)(r % p.L) + p.causal_offset : (int64_t)1 << 40;
    }
    const uint16_t* kbase = p.k + (uint64_t)b * p.k_sb + (uint64_t)hkv * p.k_sh;
    const uint16_t* vbase = p.v + (uint64_t)b * p.v_sb + (uint64_t)hkv * p.v_sh;
    // One stage: keys k0 .. k0 + 15 of K then V, 16 bytes per copy; keys past
    // the range are zero-filled (source size 0, the address stays in bounds).
    auto issue = [&](uint32_t k0, int slot) {
        const uint32_t dst0 = ring_s + (uint32_t)(slot * STAGE * 16);
#pragma unroll
        for (int n = 0; n < STAGE / 32; ++n) {
            const uint32_t e = (uint32_t)(lane + 32 * n);
            const uint32_t kv = e / (16 * CPR), row = (e / CPR) % 16, chunk = e % CPR;
            const uint32_t key = k0 + row;
            const bool in = key < k_end;
            const uint16_t* src = kv ? vbase + (uint64_t)(in ? key : k_begin) * p.v_sk + chunk * 8
                                     : kbase + (uint64_t)(in ? key : k_begin) * p.k_sk + chunk * 8;
            const uint32_t pc = kv ? v_chunk(row, chunk) : k_chunk<D>(row, chunk);
            cp_async16(dst0 + (kv * 16 * CPR + row * CPR + pc) * 16, src, in ? 16u : 0u);
        }
    };
    float o[NJ][4];
#pragma unroll
    for (int j = 0; j < NJ; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m[2] = {NEG, NEG}, l[2] = {0.0f, 0.0f};
#pragma unroll
    for (int st = 0; st < DEC_STAGES - 1; ++st) {
        if (k_begin + 16 * st < k_end) issue(k_begin + 16 * st, st);
        cp_async_commit();
    }
    int slot = 0;
    for (uint32_t k0 = k_begin; k0 < k_end; k0 += 16) {
        cp_async_wait<DEC_STAGES - 2>();  // this stage's copies (all but the newest group) have landed
        __syncwarp();
        const uint4* kst = ring + slot * STAGE;
        const uint4* vst = kst + 16 * CPR;
        float s[2][4];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            uint32_t kw[QW];
            const uint32_t row = (uint32_t)(8 * t + g);
#pragma unroll
            for (int i = 0; i < QW / 4; ++i) {
                const uint4 w = kst[row * CPR + k_chunk<D>(row, (uint32_t)(c * (QW / 4) + i))];
                kw[4 * i] = w.x, kw[4 * i + 1] = w.y, kw[4 * i + 2] = w.z, kw[4 * i + 3] = w.w;
            }
            s[t][0] = s[t][1] = s[t][2] = s[t][3] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
                mma16816<FMT>(s[t], qa[0][2 * ks], qa[1][2 * ks], qa[0][2 * ks + 1], qa[1][2 * ks + 1], kw[2 * ks],
                              kw[2 * ks + 1]);
        }
        // V words of keys 2c, 2c+1, 2c+8, 2c+9 at columns g*D/8 .. (D = 128:
        // two chunks, read in the order that keeps each 8-lane phase on
        // distinct bank groups)
        uint32_t vw[4][NJ / 2];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint32_t row = (uint32_t)(2 * c + (t & 1) + 8 * (t >> 1));
            if constexpr (NJ / 8 == 2) {
                const uint32_t odd = (uint32_t)(g & 1);
                const uint4 w0 = vst[row * CPR + v_chunk(row, (uint32_t)(2 * g) + odd)];
                const uint4 w1 = vst[row * CPR + v_chunk(row, (uint32_t)(2 * g) + (odd ^ 1u))];
                const uint4 lo = odd ? w1 : w0, hi = odd ? w0 : w1;
                vw[t][0] = lo.x, vw[t][1] = lo.y, vw[t][2] = lo.z, vw[t][3] = lo.w;
                vw[t][4] = hi.x, vw[t][5] = hi.y, vw[t][6] = hi.z, vw[t][7] = hi.w;
            } else {
                const uint4 w = vst[row * CPR + v_chunk(row, (uint32_t)g)];
                vw[t][0] = w.x, vw[t][1] = w.y, vw[t][2] = w.z, vw[t][3] = w.w;
            }
        }
        __syncwarp();  // every lane has read this slot: it may be refilled
        if (k0 + 16 * (DEC_STAGES - 1) < k_end) issue(k0 + 16 * (DEC_STAGES - 1), (slot + DEC_STAGES - 1) % DEC_STAGES);
        cp_async_commit();
        slot = slot + 1 == DEC_STAGES ? 0 : slot + 1;
        // scores in log2 units, masked: s[t][e] is row g + 8 * (e >> 1), key k0 + 8t + 2c + (e & 1)
        float mx[2] = {NEG, NEG};
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int rr = e >> 1;
                const int64_t key = (int64_t)k0 + 8 * t + 2 * c + (e & 1);
                const float x = (key < (int64_t)k_end && key <= vis[rr]) ? s[t][e] * p.scale_log2 : NEG;
                s[t][e] = x;
                mx[rr] = fmaxf(mx[rr], x);
            }
        float alpha[2], base[2];
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
            const float mn = fmaxf(m[rr], mx[rr]);
            alpha[rr] = m[rr] == NEG ? 0.0f : ex2(m[rr] - mn);
            m[rr] = mn;
            base[rr] = mn == NEG ? 0.0f : mn + p.shift;
        }
        // P as the A operand of PV: rows g / g + 8, keys 2c, 2c+1 (tile 0) and 8 + 2c, 9 + 2c (tile 1)
        uint32_t pa[4];
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int rr = 0; rr < 2; ++rr)
                pa[2 * t + rr] = pack2(ex2(s[t][2 * rr] - base[rr]), ex2(s[t][2 * rr + 1] - base[rr]), FMT);
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const float2 w0 = unpack2<FMT>(pa[rr]), w1 = unpack2<FMT>(pa[2 + rr]);
            l[rr] = fmaf(l[rr], alpha[rr], (w0.x + w0.y) + (w1.x + w1.y));
        }
        if (__any_sync(0xffffffffu, alpha[0] != 1.0f || alpha[1] != 1.0f)) {
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                o[j][0] *= alpha[0], o[j][1] *= alpha[0];
                o[j][2] *= alpha[1], o[j][3] *= alpha[1];
            }
        }
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const uint32_t sel = (j & 1) ? 0x7632u : 0x5410u;  // high or low 16-bit halves of the word pair
            const uint32_t b0 = __byte_perm(vw[0][j / 2], vw[1][j / 2], sel);
            const uint32_t b1 = __byte_perm(vw[2][j / 2], vw[3][j / 2], sel);
            mma16816<FMT>(o[j], pa[0], pa[1], pa[2], pa[3], b0, b1);
        }
    }
    cp_async_wait<0>();
    // The CTA's four warps combine their ranges: each leaves {m, l, O} per
    // row in its own (drained) ring, then the CTA writes one record per row,
    // O = sum_w O_w 2^(m_w - M), l = sum_w l_w 2^(m_w - M) with M the largest
    // m of the warps that saw a key.
    float* xs = reinterpret_cast<float*>(ring);  // [16 rows][D + 2]: m, l, O
    __syncwarp();
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 1);
        l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 2);
        float* x = xs + (g + 8 * rr) * (D + 2);
        if (c == 0) {
            x[0] = m[rr];
            x[1] = l[rr];
        }
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            x[2 + 2 * c * NJ + j] = o[j][2 * rr];
            x[2 + (2 * c + 1) * NJ + j] = o[j][2 * rr + 1];
        }
    }
    __syncthreads();
    // the CTA's records: global memory, or (cluster) the upper half of warp
    // 0's ring, clear of every warp's {m, l, O} area
    float* cmb = reinterpret_cast<float*>(dsm) + DEC_STAGES * STAGE * 2;
    for (uint32_t r = 0; r < R; ++r) {
        float mw[DEC_WARPS], lw[DEC_WARPS], M = NEG;
#pragma unroll
        for (int w = 0; w < DEC_WARPS; ++w) {
            const float* x = reinterpret_cast<const float*>(dsm + (size_t)w * DEC_STAGES * STAGE) + r * (D + 2);
            mw[w] = x[0], lw[w] = x[1];
            if (lw[w] > 0.0f) M = fmaxf(M, mw[w]);
        }
        float wt[DEC_WARPS], Lr = 0.0f;
#pragma unroll
        for (int w = 0; w < DEC_WARPS; ++w) {
            wt[w] = lw[w] > 0.0f ? exp2f(mw[w] - M) : 0.0f;
            Lr = fmaf(lw[w], wt[w], Lr);
        }
        const uint32_t h = hkv * p.G + r / p.L, q = r % p.L;
        float* rec = p.cluster ? cmb + r * (D + 2)
                               : p.part + ((((uint64_t)b * p.H + h) * p.L + q) * p.splits + split) * (D + 2);
        if (threadIdx.x == 0) {
            rec[0] = M == NEG ? 0.0f : M + p.shift;
            rec[1] = Lr;
        }
        for (uint32_t d = threadIdx.x; d < (uint32_t)D; d += 32 * DEC_WARPS) {
            float acc = 0.0f;
#pragma unroll
            for (int w = 0; w < DEC_WARPS; ++w)
                if (wt[w] != 0.0f)
                    acc = fmaf(reinterpret_cast<const float*>(dsm + (size_t)w * DEC_STAGES * STAGE)[r * (D + 2) + 2 + d], wt[w], acc);
            rec[2 + d] = acc;
        }
    }
    if (p.cluster) {
        // The cluster's CTAs combine its records as attn_merge_kernel does
        // (ranges in index order, the same arithmetic), CTA t taking rows
        // t, t + splits, ...
        cluster_sync();  // every CTA's records are in its shared memory
        {
            const uint32_t cmb_s = (uint32_t)__cvta_generic_to_shared(cmb);
            for (uint32_t r = split; r < R; r += p.splits) {
                float Mx = NEG;
                for (uint32_t t = 0; t < p.splits; ++t) {
                    const uint32_t rec = mapa_u32(cmb_s + r * (D + 2) * 4, t);
                    if (ld_cluster_f32(rec + 4) > 0.0f) Mx = fmaxf(Mx, ld_cluster_f32(rec));
                }
                float Lr = 0.0f, acc = 0.0f;
                const uint32_t d = threadIdx.x;  // one output column per thread (D <= 128)
                for (uint32_t t = 0; t < p.splits; ++t) {
                    const uint32_t rec = mapa_u32(cmb_s + r * (D + 2) * 4, t);
                    const float lt = ld_cluster_f32(rec + 4);
                    if (!(lt > 0.0f)) continue;
                    const float wgt = exp2f(ld_cluster_f32(rec) - Mx);
                    Lr = fmaf(lt, wgt, Lr);
                    if (d < (uint32_t)D) acc = fmaf(ld_cluster_f32(rec + (2 + d) * 4), wgt, acc);
                }
                const float inv = Lr > 0.0f ? 1.0f / Lr : 0.0f;
                const uint32_t h = hkv * p.G + r / p.L, q = r % p.L;
                const uint64_t off = (uint64_t)b * p.o_sb + (uint64_t)h * p.o_sh + (uint64_t)q * p.o_sl + d;
                if (d < (uint32_t)D) {
                    if (p.out_low)
                        static_cast<uint16_t*>(p.out)[off] = p.out_low == FB_BF16 ? encode_bf16(acc * inv) : encode_f16(acc * inv);
                    else
                        static_cast<float*>(p.out)[off] = acc * inv;
                }
            }
        }
        cluster_sync();  // the records stay in shared memory until every CTA has read them
    }
}

// Decode path for 16-bit Q/K/V: FB_ERR_UNSUPPORTED unless at most 16 query
// rows share a key/value head, keys are many, and every row is 16-byte
// aligned (the merge writes the output rows).
template <int D>
int launch_decode16(const AttnArgs& a, uint32_t fmt, const RowsLayout& ql, const RowsLayout& kl, const RowsLayout& vl,
                    const RowsLayout& ol, uint64_t L, uint64_t H, uint64_t Hkv, cudaStream_t st) {
    const uint64_t Lk = a.keys, G = H / Hkv, R = G * L;
    if (R > 16 || Lk < 1024 || a.mask_kind != FB_MASK_NONE) return FB_ERR_UNSUPPORTED;
    auto rows16 = [](const RowsLayout& rl) { return rl.s_row % 8 == 0 && rl.s_head % 8 == 0 && rl.s_batch % 8 == 0; };
    if (!rows16(ql) || !rows16(kl) || !rows16(vl)) return FB_ERR_UNSUPPORTED;
    if (Lk > 0x7fffffffull || ql.batch * H * L > 0x7fffffffull) return FB_ERR_UNSUPPORTED;
    const uint64_t B = ql.batch, units = B * Hkv;
    // Key ranges: about two CTAs (of four warps) per SM, at least 64 keys per
    // warp (few units, e.g. one batch per GPU, still fill the GPU); `splits`
    // CTAs per (batch, key/value head), each leaving one record per query row.
    const uint64_t target = (uint64_t)sm_count() * 2;
    const uint64_t want = std::max<uint64_t>(1, std::min<uint64_t>(target / units, (Lk + 64 * DEC_WARPS - 1) / (64 * DEC_WARPS)));
    const uint64_t kps = ((Lk + want * DEC_WARPS - 1) / (want * DEC_WARPS) + 15) / 16 * 16;  // keys per warp
    const uint64_t splits = (Lk + kps * DEC_WARPS - 1) / (kps * DEC_WARPS);
    // At most eight ranges: one cluster per unit merges in shared memory.
    const bool cluster = splits <= 8;
    float* part = nullptr;
    if (!cluster) {
        const uint64_t bytes = B * H * L * splits * (D + 2) * sizeof(float);
        part = static_cast<float*>(scratch(st, bytes, SCRATCH_ATTN_SPLIT));
        if (!part) {  // none (e.g. first use inside a graph capture): the tile kernel takes it
            (void)cudaGetLastError();
            return FB_ERR_UNSUPPORTED;
        }
    }
    Dec16Params d{};
    d.q = static_cast<const uint16_t*>(a.q) + a.q_offset;
    d.k = static_cast<const uint16_t*>(a.k) + a.k_offset;
    d.v = static_cast<const uint16_t*>(a.v) + a.v_offset;
    d.q_sb = ql.s_batch, d.q_sh = ql.s_head, d.q_sl = ql.s_row;
    d.k_sb = kl.batch_bcast ? 0 : kl.s_batch, d.k_sh = kl.s_head, d.k_sk = kl.s_row;
    d.v_sb = vl.batch_bcast ? 0 : vl.s_batch, d.v_sh = vl.s_head, d.v_sk = vl.s_row;
    d.H = (uint32_t)H, d.Hkv = (uint32_t)Hkv, d.G = (uint32_t)G, d.L = (uint32_t)L, d.Lk = (uint32_t)Lk;
    d.splits = (uint32_t)splits, d.keys_per_split = (uint32_t)kps;
    d.scale_log2 = a.scale * 1.4426950408889634f;
    d.shift = fmt ? 9.0f + std::ceil(std::log2((float)std::max<uint64_t>(Lk, 1))) : 0.0f;
    d.causal = a.causal ? 1 : 0;
    d.causal_offset = a.causal_offset;
    d.part = part;
    d.cluster = cluster ? 1 : 0;
    d.out = a.out_low ? static_cast<void*>(reinterpret_cast<uint16_t*>(a.out) + a.o_offset)
                      : static_cast<void*>(a.out + a.o_offset);
    d.out_low = a.out_low;
    d.o_sb = ol.s_batch, d.o_sh = ol.s_head, d.o_sl = ol.s_row;
    const uint64_t grid = units * splits;
    if (grid > 0x7fffffffull) return FB_ERR_UNSUPPORTED;
    const int smem = DEC_WARPS * DEC_STAGES * 2 * 16 * D * 2;  // bytes of the per-warp rings
    auto kernel = fmt ? attn_decode16_kernel<D, 1> : attn_decode16_kernel<D, 0>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return launch_status("shared-memory attribute");
    if (cluster) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(32 * DEC_WARPS);
        cfg.dynamicSmemBytes = (size_t)smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)splits;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&cfg, kernel, d) != cudaSuccess) return launch_status("kernel launch");
        count_launch(kernel_name("attn_decode16_kernel", {D, (int)fmt}).c_str());
        return launch_status("kernel launch");
    }
    kernel<<<(unsigned)grid, 32 * DEC_WARPS, smem, st>>>(d);
    count_launch(kernel_name("attn_decode16_kernel", {D, (int)fmt}).c_str());
    if (cudaGetLastError() != cudaSuccess) return launch_status("kernel launch");
    AttnParams m{};
    m.L = (uint32_t)L, m.H = (uint32_t)H, m.bh = (uint32_t)(B * H), m.rec_rows = (uint32_t)L;
    m.splits = (uint32_t)splits, m.part = part;
    m.out = a.out_low ? reinterpret_cast<float*>(reinterpret_cast<uint16_t*>(a.out) + a.o_offset) : a.out + a.o_offset;
    m.out_low = a.out_low;
    m.o_sb = ol.s_batch, m.o_sh = ol.s_head, m.o_sl = ol.s_row;
    const uint64_t rows = B * H * L;
    const unsigned mgrid = (unsigned)std::min<uint64_t>((rows + 7) / 8, (uint64_t)sm_count() * 16);
    attn_merge_kernel<D><<<mgrid, 256, 0, st>>>(m);
    count_launch(kernel_name("attn_merge_kernel", {D}).c_str());
    return launch_status("kernel launch");
}

// Output rows [batch, heads, rows, D] as a 4-D TMA store target: 16-bit
// (out_low = FB_BF16 / FB_F16, boxes of 64 values) or f32 (boxes of 32), 128
// rows per box, 128-byte swizzle.
bool make_out_map(CUtensorMap* map, void* ptr, uint32_t out_low, uint64_t D, const RowsLayout& l) {
    auto enc = encode_tiled_attn();
    if (!enc) return false;
    const uint64_t esz = out_low ? 2 : 4;
    cuuint64_t dims[4] = {D, l.rows, l.heads, l.batch};
    uint64_t sb[3] = {l.s_row * esz, l.s_head * esz, l.s_batch * esz};
    uint64_t filler = (D * esz + 15) / 16 * 16;
    for (int i = 0; i < 3; ++i) {
        if (dims[i + 1] == 1 && (sb[i] == 0 || sb[i] % 16 != 0 || sb[i] >= (1ull << 40))) sb[i] = filler;
        if (sb[i] == 0 || sb[i] % 16 != 0 || sb[i] >= (1ull << 40)) return false;
        filler = sb[i] * dims[i + 1];
        filler = (filler + 15) / 16 * 16;
        if (filler >= (1ull << 40)) filler = 16;
    }
    for (int i = 0; i < 4; ++i)
        if (dims[i] == 0 || dims[i] > (1ull << 31)) return false;
    cuuint64_t strides[3] = {sb[0], sb[1], sb[2]};
    cuuint32_t box[4] = {(cuuint32_t)(128 / esz), TQ, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUtensorMapDataType type = !out_low ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                     : out_low == FB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    return enc(map, type, 4, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The short-range kernel for D = 64, Lk <= 256, no mask: parameters as
// launch_d's, one CTA per (batch, head, 128-row query tile).
int launch_short(const AttnArgs& a, uint32_t fmt, const RowsLayout& ql, const RowsLayout& kl, const RowsLayout& vl,
                 const RowsLayout& ol, uint64_t L, uint64_t H, uint64_t Hkv, uint64_t q_mod, cudaStream_t st) {
    const uint64_t Lk = a.keys;
    const uint64_t BH = a.rows / L;
    CUtensorMap tq, tk, tv;
    const void* q = static_cast<const uint16_t*>(a.q) + a.q_offset;
    const void* k = static_cast<const uint16_t*>(a.k) + a.k_offset;
    const void* v = static_cast<const uint16_t*>(a.v) + a.v_offset;
    if (!make_rows_map(&tq, q, fmt, SD, ql, TQ) || !make_rows_map(&tk, k, fmt, SD, kl, TK) ||
        !make_rows_map(&tv, v, fmt, SD, vl, TK))
        return FB_ERR_UNSUPPORTED;
    AttnParams p{};
    p.fmt = fmt;
    p.L = (uint32_t)L;
    p.Lk = (uint32_t)Lk;
    p.H = (uint32_t)H;
    p.Hkv = (uint32_t)Hkv;
    p.q_blocks = (uint32_t)((L + TQ - 1) / TQ);
    p.q_mod = (uint32_t)q_mod;
    p.bh = (uint32_t)BH;
    p.kv_tiles = (uint32_t)((Lk + TK - 1) / TK);
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.shift = fmt ? 9.0f + std::ceil(std::log2((float)std::max<uint64_t>(Lk, 1))) : 0.0f;
    p.causal = a.causal ? 1 : 0;
    p.causal_offset = a.causal_offset;
    p.k_batch_bcast = kl.batch_bcast ? 1 : 0;
    p.v_batch_bcast = vl.batch_bcast ? 1 : 0;
    p.out = a.out_low ? reinterpret_cast<float*>(reinterpret_cast<uint16_t*>(a.out) + a.o_offset) : a.out + a.o_offset;
    p.out_low = a.out_low;
    p.o_sb = ol.s_batch;
    p.o_sh = ol.s_head;
    p.o_sl = ol.s_row;
    p.splits = 1;
    p.split_tiles = p.kv_tiles;
    p.rec_rows = (uint32_t)L;
    CUtensorMap to;
    if (!make_out_map(&to, p.out, p.out_low, SD, ol)) return FB_ERR_UNSUPPORTED;
    // Two softmax warps per row where the second half's P fits in the
    // columns past the scores and clear of O: 192 or 208 score columns.
    const uint32_t nkp = (uint32_t)((Lk + 15) & ~15ull), nch = (nkp + 31) / 32;
    const bool split = nkp >= 192 && nkp + 16 * (nch - 4) <= S_TMEM_COLS;
    auto kernel = split ? attn_short_kernel<2> : attn_short_kernel<1>;
    const int smem = split ? SCfg<2>::SMEM : SCfg<1>::SMEM;
    const int threads = split ? SCfg<2>::THREADS : SCfg<1>::THREADS;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return launch_status("shared-memory attribute");
    const uint64_t units = (uint64_t)p.q_blocks * BH;
    if (units == 0) return FB_OK;
    if (units > 0xffffffffull) return FB_ERR_UNSUPPORTED;
    const uint64_t grid = std::min<uint64_t>(units, (uint64_t)sm_count() * 2);  // persistent, two CTAs per SM
    kernel<<<(unsigned)grid, threads, smem, st>>>(tq, tk, tv, to, p);
    count_launch(split ? "attn_short_kernel<2>" : "attn_short_kernel");
    return launch_status("kernel launch");
}
}  // namespace

uint32_t read_attention_status() {
    uint32_t v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_attn_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(zero));
    return v;
}

int launch_attention_tc(const AttnArgs& a, void* stream) {
    if (a.dtype != FB_BF16 && a.dtype != FB_F16) return FB_ERR_UNSUPPORTED;
    if (a.depth != a.value_depth || (a.depth != 64 && a.depth != 128)) return FB_ERR_UNSUPPORTED;
    if (a.row_rank < 2 || a.keys == 0 || a.rows == 0) return FB_ERR_UNSUPPORTED;
    const int r = (int)a.row_rank;
    const uint64_t D = a.depth, L = a.row_dims[r - 1], H = a.row_dims[r - 2], Lk = a.keys;
    if (a.q_stride_d != 1 || a.k_stride_d != 1 || a.v_stride_d != 1 || a.o_stride_d != 1) return FB_ERR_UNSUPPORTED;
    if (H % a.group_size != 0) return FB_ERR_UNSUPPORTED;
    const uint64_t Hkv = H / a.group_size;
    if (a.rows / L * L != a.rows || L > (1u << 30) || Lk > (1u << 30)) return FB_ERR_UNSUPPORTED;
    // Row layouts: query/key axis, head axis (K/V heads are query heads /
    // group), batch axes merged; TMA needs 16-byte strides and bases.
    RowsLayout ql, kl, vl, ol;
    ql.rows = L, ql.heads = H, ql.s_row = a.q_row_strides[r - 1], ql.s_head = a.q_row_strides[r - 2];
    kl.rows = Lk, kl.heads = Hkv, kl.s_row = a.k_stride_key, kl.s_head = a.k_row_strides[r - 2];
    vl.rows = Lk, vl.heads = Hkv, vl.s_row = a.v_stride_key, vl.s_head = a.v_row_strides[r - 2];
    ol.rows = L, ol.heads = H, ol.s_row = a.o_row_strides[r - 1], ol.s_head = a.o_row_strides[r - 2];
    if (!merge_batch(a, a.q_row_strides, r - 2, &ql) || !merge_batch(a, a.k_row_strides, r - 2, &kl) ||
        !merge_batch(a, a.v_row_strides, r - 2, &vl) || !merge_batch(a, a.o_row_strides, r - 2, &ol))
        return FB_ERR_UNSUPPORTED;
    if (ql.batch_bcast || ol.batch_bcast) return FB_ERR_UNSUPPORTED;  // distinct query rows per batch index
    if (ql.batch * H * L != a.rows || ol.batch != ql.batch) return FB_ERR_UNSUPPORTED;
    if ((!kl.batch_bcast && kl.batch != ql.batch) || (!vl.batch_bcast && vl.batch != ql.batch)) return FB_ERR_UNSUPPORTED;
    // output rows take 16-byte stores (float4, or eight 16-bit values): 16-byte aligned rows
    const uint64_t o_vec = a.out_low ? 8 : 4;
    auto mult = [o_vec](uint64_t s, uint64_t n) { return n <= 1 || s % o_vec == 0; };
    if (!mult(ol.s_row, L) || !mult(ol.s_head, H) || !mult(ol.s_batch, ol.batch)) return FB_ERR_UNSUPPORTED;
    // Masks (32-bit elements) are read 16 bytes at a time along contiguous
    // keys; rows start 16-byte aligned.  Broadcast axes have stride 0.
    RowsLayout ml;
    if (a.mask_kind != FB_MASK_NONE) {
        if (a.m_stride_key != 1 || Lk % 4 != 0) return FB_ERR_UNSUPPORTED;
        ml.rows = L, ml.heads = H, ml.s_row = a.m_row_strides[r - 1], ml.s_head = a.m_row_strides[r - 2];
        if (!merge_batch(a, a.m_row_strides, r - 2, &ml)) return FB_ERR_UNSUPPORTED;
        if (!ml.batch_bcast && ml.batch != ql.batch) return FB_ERR_UNSUPPORTED;
        if (ml.s_row % 4 != 0 || ml.s_head % 4 != 0 || ml.s_batch % 4 != 0) return FB_ERR_UNSUPPORTED;
        if ((reinterpret_cast<uintptr_t>(a.mask) + a.m_offset * 4) % 16 != 0) return FB_ERR_UNSUPPORTED;
    }
    auto aligned = [](const void* p, uint64_t off, uint64_t esz) {
        return (reinterpret_cast<uintptr_t>(p) + off * esz) % 16 == 0;
    };
    if (!aligned(a.q, a.q_offset, 2) || !aligned(a.k, a.k_offset, 2) || !aligned(a.v, a.v_offset, 2) ||
        !aligned(a.out, a.o_offset, a.out_low ? 2 : 4))
        return FB_ERR_UNSUPPORTED;
    const uint32_t fmt = a.dtype == FB_BF16 ? 1 : 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Decode (at most 16 query rows per key/value head over many keys): one
    // 16-row block per head on the warp-level MMA, K/V read once.
    if (a.mask_kind == FB_MASK_NONE && a.group_size * L <= 16) {
        const int r1 = D == 64 ? launch_decode16<64>(a, fmt, ql, kl, vl, ol, L, H, Hkv, st)
                               : launch_decode16<128>(a, fmt, ql, kl, vl, ol, L, H, Hkv, st);
        if (r1 != FB_ERR_UNSUPPORTED) return r1;
    }
    // Decode of grouped heads (few query rows, no mask): the G query heads of
    // a key/value head share its K/V, so their G x L rows become the rows of
    // one packed head (G times fewer key steps), when each head's rows of Q
    // and of the output are contiguous.
    uint64_t Lp = L, Hp = H, q_mod = L;
    const uint64_t G = a.group_size;
    if (G > 1 && L <= 64 && a.mask_kind == FB_MASK_NONE) {
        auto packable = [&](const RowsLayout& rl) { return L == 1 || rl.s_head == L * rl.s_row; };
        if (packable(ql) && packable(ol)) {
            auto pack = [&](RowsLayout& rl) {
                if (L == 1) rl.s_row = rl.s_head;
                rl.rows = G * L;
                rl.heads = Hkv;
                rl.s_head *= G;
            };
            pack(ql);
            pack(ol);
            Lp = G * L;
            Hp = Hkv;
        }
    }
    // Key ranges that fit one tile row of TMEM at D = 64 (the ViT encoder's
    // 197 tokens): one S group over every key, the exact row maximum, no
    // online rescale, a TMA-store epilogue (attn_short_kernel).  Measured on
    // the encoder's attention (64 x 12 heads x 197 tokens, BF16 out):
    // 55.6 -> 53.7 us; per CTA ~7.8 us of which the softmax passes 3.2 and
    // the epilogue 2.0, two CTAs per SM.
    if (D == 64 && Lk <= 2 * TK && a.mask_kind == FB_MASK_NONE) {
        const int r2 = launch_short(a, fmt, ql, kl, vl, ol, Lp, Hp, Hkv, q_mod, st);
        if (r2 != FB_ERR_UNSUPPORTED) return r2;
    }
    // Short key ranges at D = 64 (the whole K/V loop is a few tiles, so each
    // CTA's fixed load and epilogue latency dominates): one Q tile per CTA,
    // two CTAs per SM.
    if (D == 64) {
        return Lk <= 4 * TK ? launch_d<64, 1>(a, fmt, ql, kl, vl, ol, ml, Lp, Hp, Hkv, q_mod, st)
                            : launch_d<64, 2>(a, fmt, ql, kl, vl, ol, ml, Lp, Hp, Hkv, q_mod, st);
    }
    return launch_d<128, 2>(a, fmt, ql, kl, vl, ol, ml, Lp, Hp, Hkv, q_mod, st);
}

}  // namespace fb
