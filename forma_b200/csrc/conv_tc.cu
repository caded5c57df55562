// Implicit-GEMM convolution on the 5th-generation tensor cores (tcgen05).
//
// conv_low_f32 with 16-bit operands is the GEMM
//     D[m, o] = sum_k A[m, k] * B[o, k]
// over m = (n, p, q) output pixels, o = output channels and k = (r, s, c)
// filter taps x input channels, accumulated in f32.
//   A  channels-last input.  A TMA im2col load gathers 128 output pixels x 64
//      channels of one tap straight from the NHWC tensor, padding with zeros
//      at image borders, into a 128B-swizzled K-major shared tile; 1x1
//      stride-1 convolutions use a plain 2-D [pixels, channels] tiled map.
//   B  weights as [O, R*S*C] (OHWI storage), 2-D tiled TMA.
//   D  128 x BN f32 accumulator in TMEM, double-buffered so the epilogue of
//      one tile overlaps the main loop of the next.
// Warp roles in a 192-thread CTA, persistent over output tiles:
//   warp 0      TMA producer (one lane) into a STAGES-deep smem ring
//   warp 1      TMEM allocator and MMA issuer (the warp runs the issue loop,
//               one elected lane issues each MMA)
//   warps 2-5   epilogue: tcgen05.ld -> f32 stores at the output's strides
// Every wait is bounded (async.cuh); a timeout sets a status bit and the CTA
// drains its copies and MMAs before releasing TMEM and exiting.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "async.cuh"
#include "device_common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace fb {
namespace {

__device__ uint32_t g_gemm_status;

constexpr int BM = 128, BK = 64;
constexpr int THREADS = 192;

struct ConvGemmParams {
    uint32_t mode;  // 0: A = 2-D [M, C] map, 1: A = im2col map
    uint32_t fmt;   // 0 f16, 1 bf16
    uint32_t M, P, Q;
    uint32_t k_blocks, c_blocks, S;
    int32_t pad_h, pad_w, stride_h, stride_w, dil_h, dil_w;
    uint32_t m_tiles, n_tiles;
    uint32_t c_rows;  // 1: channels contiguous (s_c == 1) and aligned rows (16 B for f32, 8 B for 16-bit)
    uint32_t b_mn;    // 0: B map is [N, K] (K contiguous); 1: B map is [K, N] (N contiguous, MN-major operand)
    uint32_t out_low; // 0: f32 output; FB_BF16 / FB_F16: rounded once (nearest even) to that type
    uint32_t act;     // 1: tanh GELU of each f32 sum before the store / rounding
    uint32_t accumulate;  // 1: f32 output += sum (read-modify-write)
    float* out;       // f32 output, or the 16-bit output's storage when out_low != 0
    uint64_t out_offset, s_n, s_c, s_p, s_q;
};

template <int BN>
struct Cfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = BN == 256 ? 4 : BN == 128 ? 6 : 8;
    static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    // Epilogue staging for channels-contiguous outputs: per epilogue warp a
    // 32 x 32 f32 block with rows padded to 36 floats (16-byte aligned rows,
    // conflict-free float4 writes and reads).
    static constexpr int EPI_PITCH = 36;
    static constexpr int EPI_BYTES = 4 * 32 * EPI_PITCH * 4;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + 256;  // align slack + ring + staging + barriers
};

template <int BN>
__global__ void __launch_bounds__(THREADS, 1) conv_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                               const __grid_constant__ CUtensorMap tmB,
                                                               ConvGemmParams p) {
    using C = Cfg<BN>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* ring = smem;
    float* epi = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES + C::EPI_BYTES);
    uint64_t* full = bars;                     // [STAGES]
    uint64_t* empty = bars + C::STAGES;        // [STAGES]
    uint64_t* tfull = bars + 2 * C::STAGES;    // [2]
    uint64_t* tempty = tfull + 2;              // [2]
    uint64_t* drain = tempty + 2;              // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t tiles = p.m_tiles * p.n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4 * 32);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
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
        uint32_t stage = 0, phase = 0;
        uint64_t issued = 0;
        bool failed = false;
        for (uint32_t t = blockIdx.x; t < tiles && !failed; t += gridDim.x) {
            const uint32_t mt = t / p.n_tiles, nt = t % p.n_tiles;
            const uint32_t m0 = mt * BM;
            const uint32_t pq = p.P * p.Q;
            const int32_t n0 = (int32_t)(m0 / pq), rem = (int32_t)(m0 % pq);
            const int32_t w0 = (rem % (int32_t)p.Q) * p.stride_w - p.pad_w;
            const int32_t h0 = (rem / (int32_t)p.Q) * p.stride_h - p.pad_h;
            for (uint32_t kb = 0; kb < p.k_blocks; ++kb) {
                if (!mbar_wait(&empty[stage], phase ^ 1)) {
                    atomicOr(&g_gemm_status, 1u << DEV_GEMM_PRODUCER_TIMEOUT);
                    failed = true;
                    break;
                }
                unsigned char* a_dst = ring + stage * C::STAGE_BYTES;
                unsigned char* b_dst = a_dst + C::A_BYTES;
                mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                const uint32_t cb = kb % p.c_blocks, tap = kb / p.c_blocks;
                if (p.mode == 0) {
                    tma_load_2d(a_dst, &tmA, (int32_t)(cb * BK), (int32_t)m0, &full[stage]);
                } else {
                    const uint32_t r = tap / p.S, s = tap % p.S;
                    tma_load_im2col_4d(a_dst, &tmA, (int32_t)(cb * BK), w0, h0, n0, (uint16_t)(s * p.dil_w),
                                       (uint16_t)(r * p.dil_h), &full[stage]);
                }
                if (p.b_mn) {
                    // [K, N] rows: BN / 64 boxes of 64 k-rows x 64 columns (8 KB each)
#pragma unroll
                    for (int nb = 0; nb < BN / 64; ++nb)
                        tma_load_2d(b_dst + nb * (BK * 128), &tmB, (int32_t)(nt * BN + nb * 64), (int32_t)(kb * BK),
                                    &full[stage]);
                } else {
                    tma_load_2d(b_dst, &tmB, (int32_t)(kb * BK), (int32_t)(nt * BN), &full[stage]);
                }
                ++issued;
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
        if (failed) {
            // Let the loads already issued land before the CTA can exit.
            uint32_t s = stage, ph = phase;
            for (int i = 0; i < C::STAGES && issued > 0; ++i, --issued) {
                if (s == 0) {
                    s = C::STAGES;
                    ph ^= 1;
                }
                --s;
                (void)mbar_wait(&full[s], ph);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        // The whole warp runs the loop with warp-uniform operands and waits;
        // one elected lane issues each tcgen05.mma / commit.
        const uint32_t idesc = f16_idesc(p.fmt, BM, BN);
        const uint32_t idesc_mn = idesc | (1u << 16);  // B MN-major
        auto wait = [](uint64_t* bar, uint32_t parity) { return __all_sync(0xffffffffu, mbar_wait(bar, parity)); };
        uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
        bool failed = false;
        for (uint32_t t = blockIdx.x; t < tiles && !failed; t += gridDim.x) {
            if (!wait(&tempty[acc], acc_phase ^ 1)) {
                failed = true;
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem + acc * BN;
            for (uint32_t kb = 0; kb < p.k_blocks; ++kb) {
                if (!wait(&full[stage], phase)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                const uint64_t ad = sw128_desc(smem_u32(ring + stage * C::STAGE_BYTES));
                if (p.b_mn) {
                    // MN-major B: 64-column blocks BK * 128 bytes apart, 16 k-rows per step
                    const uint64_t bd = sw128_mn_desc(smem_u32(ring + stage * C::STAGE_BYTES + C::A_BYTES), BK * 128);
                    umma_f16_ss_warp(d, ad, bd, idesc_mn, kb != 0);
#pragma unroll
                    for (int k = 1; k < BK / 16; ++k)
                        umma_f16_ss_warp(d, desc_add(ad, k * 32), desc_add(bd, k * 16 * 128), idesc_mn, 1u);
                } else {
                    const uint64_t bd = desc_add(ad, C::A_BYTES);
                    umma_f16_ss_warp(d, ad, bd, idesc, kb != 0);
#pragma unroll
                    for (int k = 1; k < BK / 16; ++k)
                        umma_f16_ss_warp(d, desc_add(ad, k * 32), desc_add(bd, k * 32), idesc, 1u);
                }
                umma_commit_warp(&empty[stage]);  // frees the stage when these MMAs complete
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (failed) break;
            umma_commit_warp(&tfull[acc]);  // accumulator complete
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (failed && lane == 0) atomicOr(&g_gemm_status, 1u << DEV_GEMM_MMA_TIMEOUT);
        // All MMAs issued by this warp have finished once `drain` completes.
        umma_commit_warp(drain);
        (void)wait(drain, 0);
    } else if (warp >= 2) {
        // ------------------------------------------------ epilogue
        const int quarter = warp & 3;  // TMEM lanes [32*quarter, +32)
        const int row = quarter * 32 + lane;
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t t = blockIdx.x; t < tiles; t += gridDim.x) {
            // Warp-uniform outcome: the tcgen05.ld below is .sync.aligned.
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase))) {
                atomicOr(&g_gemm_status, 1u << DEV_GEMM_EPILOGUE_TIMEOUT);
                break;
            }
            tc_fence_after();
            const uint32_t mt = t / p.n_tiles, nt = t % p.n_tiles;
            const uint32_t m = mt * BM + row;
            // element offset of this row's first column in the output (~0: no such row)
            uint64_t base = ~0ull;
            if (m < p.M) {
                const uint32_t pq = p.P * p.Q;
                const uint32_t n = m / pq, r = m % pq;
                base = p.out_offset + (uint64_t)n * p.s_n + (uint64_t)(r / p.Q) * p.s_p + (uint64_t)(r % p.Q) * p.s_q +
                       (uint64_t)(nt * BN) * p.s_c;
            }
            uint16_t* out16 = reinterpret_cast<uint16_t*>(p.out);
            const uint32_t taddr = tmem + acc * BN + ((uint32_t)(quarter * 32) << 16);
            if (p.c_rows) {
                // Channels contiguous: each row's 32-column chunk is 128
                // contiguous bytes.  Stage the warp's 32 x 32 block in shared
                // memory, then store it as float4 so that one instruction
                // writes four whole 128-byte rows (8 lanes per row).
                float* st = epi + quarter * (32 * C::EPI_PITCH);
                const uint64_t my_base = base;
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(taddr + c0, v);
                    tmem_wait_ld();
                    if (p.act) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(gelu_tanh(__uint_as_float(v[j])));
                    }
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        *reinterpret_cast<float4*>(st + lane * C::EPI_PITCH + 4 * q) =
                            make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                        __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
                    __syncwarp();
                    // accumulate: the chunk's eight float4 of the existing
                    // output are loaded before any store (distinct rows, no
                    // aliasing), so their latencies overlap
                    float4 prev[8];
                    if (p.accumulate) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int r = i * 4 + (lane >> 3), cc = lane & 7;
                            const uint64_t rb = __shfl_sync(0xffffffffu, my_base, r);
                            prev[i] = rb != ~0ull ? *reinterpret_cast<const float4*>(p.out + rb + c0 + 4 * cc)
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int r = i * 4 + (lane >> 3), cc = lane & 7;
                        const uint64_t rb = __shfl_sync(0xffffffffu, my_base, r);
                        const float4 val = *reinterpret_cast<const float4*>(st + r * C::EPI_PITCH + 4 * cc);
                        if (rb != ~0ull) {
                            if (p.out_low)
                                *reinterpret_cast<uint2*>(out16 + rb + c0 + 4 * cc) =
                                    make_uint2(encode_low_pair(val.x, val.y, p.out_low),
                                               encode_low_pair(val.z, val.w, p.out_low));
                            else if (p.accumulate)
                                *reinterpret_cast<float4*>(p.out + rb + c0 + 4 * cc) =
                                    make_float4(prev[i].x + val.x, prev[i].y + val.y, prev[i].z + val.z, prev[i].w + val.w);
                            else
                                *reinterpret_cast<float4*>(p.out + rb + c0 + 4 * cc) = val;
                        }
                    }
                    __syncwarp();
                }
            } else {
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(taddr + c0, v);
                    tmem_wait_ld();
                    if (p.act) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(gelu_tanh(__uint_as_float(v[j])));
                    }
                    if (base != ~0ull) {
                        if (p.out_low == FB_BF16) {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                out16[base + (uint64_t)(c0 + j) * p.s_c] = encode_bf16(__uint_as_float(v[j]));
                        } else if (p.out_low) {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                out16[base + (uint64_t)(c0 + j) * p.s_c] = encode_f16(__uint_as_float(v[j]));
                        } else if (p.accumulate) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) p.out[base + (uint64_t)(c0 + j) * p.s_c] += __uint_as_float(v[j]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j) p.out[base + (uint64_t)(c0 + j) * p.s_c] = __uint_as_float(v[j]);
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// The same GEMM on CTA pairs (2-CTA clusters, tcgen05 cta_group::2): a pair
// owns a 256 x 256 output tile; each CTA loads its 128 rows of A and its 128
// of the 256 B rows (half the weight traffic of two independent CTAs, 32 KB
// per stage so six stages fit), and holds its 128 accumulator rows in its own
// TMEM.  The even CTA's MMA warp issues every MMA (M = 256) once both CTAs'
// loads of a stage have landed on the even CTA's `full` barrier, and its
// commits arrive on both CTAs' `empty` / `tfull` barriers; both epilogues
// arrive on the even CTA's `tempty`.
// BN (256 or 192) is the pair tile's N: each CTA loads BN / 2 rows of B, and
// 192 fits tile counts of N = 768 / 2304 / 3072 to 74 pairs better than 256.
// EPW epilogue warps: 4 (one per TMEM lane quarter), or for epilogues with
// per-element work (GELU, 16-bit rounding, the f32 read-modify-write) 8 (two
// per quarter, each taking half of the columns) on 256-wide tiles and 12
// (three per quarter, 64 columns each) on 192-wide ones, at one stage less of
// the ring.  Each epilogue warp's chunk loop is latency-bound (TMEM load,
// rounding, stores held back by the store queue), so more warps per quarter
// drain an accumulator sooner: C5's fc1 + GELU 81.9 -> 68.6 us and the C5
// forward 3.17 -> 2.96 ms going from 8 to 12 (4 warps: fc1 117 us).
template <int BN_, int EPW = 4>
struct PairCfg {
    static constexpr int BN = BN_;
    static constexpr int THREADS = 64 + 32 * EPW;
    static constexpr int A_BYTES = BM * BK * 2;      // 16 KB
    static constexpr int B_BYTES = BN / 2 * BK * 2;  // 16 KB (256) / 12 KB (192)
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (BN == 256 ? 6 : 7) - (EPW >= 8 ? 1 : 0);
    static constexpr int TMEM_COLS = 512;            // two BN-column accumulators
    static constexpr int EPI_PITCH = 36;
    static constexpr int EPI_BYTES = EPW * 32 * EPI_PITCH * 4;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + 256;
    static_assert(SMEM <= 227 * 1024, "pair configuration exceeds shared memory");
    static_assert(EPW == 4 || EPW == 8 || (EPW == 12 && BN == 192), "four, eight or (192 wide) twelve epilogue warps");
};

template <int BN_, int EPW>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfg<BN_, EPW>::THREADS, 1)
    conv_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          ConvGemmParams p) {
    using C = PairCfg<BN_, EPW>;
    constexpr int BN = C::BN;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* ring = smem;
    float* epi = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES + C::EPI_BYTES);
    uint64_t* full = bars;                     // [STAGES] used in the even CTA
    uint64_t* empty = bars + C::STAGES;        // [STAGES]
    uint64_t* tfull = bars + 2 * C::STAGES;    // [2]
    uint64_t* tempty = tfull + 2;              // [2] used in the even CTA
    uint64_t* drain = tempty + 2;              // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const uint32_t pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
    const uint32_t m_pairs = (p.m_tiles + 1) / 2;
    const uint32_t tiles = m_pairs * p.n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 2 * EPW * 32);  // both CTAs' epilogue threads
        }
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool failed = false;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------ TMA producer (both CTAs)
        const uint32_t full0 = mapa_u32(smem_u32(full), 0);
        uint32_t stage = 0, phase = 0;
        uint64_t issued = 0;
        for (uint32_t t = pair; t < tiles && !failed; t += pairs) {
            const uint32_t mt = t / p.n_tiles, nt = t % p.n_tiles;
            const uint32_t m0 = mt * 2 * BM + rank * BM;
            const uint32_t pq = p.P * p.Q;
            const int32_t n0 = (int32_t)(m0 / pq), rem = (int32_t)(m0 % pq);
            const int32_t w0 = (rem % (int32_t)p.Q) * p.stride_w - p.pad_w;
            const int32_t h0 = (rem / (int32_t)p.Q) * p.stride_h - p.pad_h;
            const int32_t b0 = (int32_t)(nt * BN + rank * (BN / 2));
            for (uint32_t kb = 0; kb < p.k_blocks; ++kb) {
                if (!mbar_wait(&empty[stage], phase ^ 1)) {
                    atomicOr(&g_gemm_status, 1u << DEV_GEMM_PRODUCER_TIMEOUT);
                    failed = true;
                    break;
                }
                unsigned char* a_dst = ring + stage * C::STAGE_BYTES;
                unsigned char* b_dst = a_dst + C::A_BYTES;
                const uint32_t bar = full0 + (uint32_t)(stage * sizeof(uint64_t));
                if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);  // both CTAs' bytes
                const uint32_t cb = kb % p.c_blocks, tap = kb / p.c_blocks;
                if (p.mode == 0) {
                    tma_load_2d_pair(a_dst, &tmA, (int32_t)(cb * BK), (int32_t)m0, bar);
                } else {
                    const uint32_t r = tap / p.S, s = tap % p.S;
                    tma_load_im2col_4d_pair(a_dst, &tmA, (int32_t)(cb * BK), w0, h0, n0, (uint16_t)(s * p.dil_w),
                                            (uint16_t)(r * p.dil_h), bar);
                }
                if (BN % 128 == 0 && p.b_mn) {  // MN-major B in 64-column blocks (host: BN = 256 only)
#pragma unroll
                    for (int nb = 0; nb < BN / 2 / 64; ++nb)
                        tma_load_2d_pair(b_dst + nb * (BK * 128), &tmB, b0 + nb * 64, (int32_t)(kb * BK), bar);
                } else {
                    tma_load_2d_pair(b_dst, &tmB, (int32_t)(kb * BK), b0, bar);
                }
                ++issued;
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
        if (failed) {
            // Loads already issued land on the even CTA's barrier; give them
            // time to complete before the CTA can exit (bounded).
            const uint64_t t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < 200000ull) {
            }
        }
    } else if (warp == 1 && leader) {
        // ------------------------------------------------ MMA issuer (even CTA)
        const uint32_t idesc = f16_idesc(p.fmt, 2 * BM, BN);
        const uint32_t idesc_mn = idesc | (1u << 16);
        auto wait = [](uint64_t* bar, uint32_t parity) { return __all_sync(0xffffffffu, mbar_wait(bar, parity)); };
        uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
        for (uint32_t t = pair; t < tiles && !failed; t += pairs) {
            if (!wait(&tempty[acc], acc_phase ^ 1)) {
                failed = true;
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem + acc * BN;
            for (uint32_t kb = 0; kb < p.k_blocks; ++kb) {
                if (!wait(&full[stage], phase)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                const uint64_t ad = sw128_desc(smem_u32(ring + stage * C::STAGE_BYTES));
                if (BN % 128 == 0 && p.b_mn) {
                    const uint64_t bd = sw128_mn_desc(smem_u32(ring + stage * C::STAGE_BYTES + C::A_BYTES), BK * 128);
                    umma_f16_ss_pair_warp(d, ad, bd, idesc_mn, kb != 0);
#pragma unroll
                    for (int k = 1; k < BK / 16; ++k)
                        umma_f16_ss_pair_warp(d, desc_add(ad, k * 32), desc_add(bd, k * 16 * 128), idesc_mn, 1u);
                } else {
                    const uint64_t bd = desc_add(ad, C::A_BYTES);
                    umma_f16_ss_pair_warp(d, ad, bd, idesc, kb != 0);
#pragma unroll
                    for (int k = 1; k < BK / 16; ++k)
                        umma_f16_ss_pair_warp(d, desc_add(ad, k * 32), desc_add(bd, k * 32), idesc, 1u);
                }
                umma_commit_pair_warp(&empty[stage], 0x3);  // frees the stage in both CTAs
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (failed) break;
            umma_commit_pair_warp(&tfull[acc], 0x3);  // accumulator rows complete in both CTAs
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (failed && lane == 0) atomicOr(&g_gemm_status, 1u << DEV_GEMM_MMA_TIMEOUT);
        umma_commit_pair_warp(drain, 0x1);
        (void)wait(drain, 0);
    } else if (warp >= 2) {
        // ------------------------------------------------ epilogue (both CTAs)
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        // columns [c_lo, c_lo + COLS) of the quarter's rows for this warp
        constexpr int COLS = BN / (EPW / 4);
        const int c_lo = ((warp - 2) / 4) * COLS;
        const uint32_t tempty0 = mapa_u32(smem_u32(tempty), 0);
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t t = pair; t < tiles; t += pairs) {
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase))) {
                atomicOr(&g_gemm_status, 1u << DEV_GEMM_EPILOGUE_TIMEOUT);
                break;
            }
            tc_fence_after();
            const uint32_t mt = t / p.n_tiles, nt = t % p.n_tiles;
            const uint32_t m = mt * 2 * BM + rank * BM + row;
            uint64_t base = ~0ull;
            if (m < p.M) {
                const uint32_t pq = p.P * p.Q;
                const uint32_t n = m / pq, r = m % pq;
                base = p.out_offset + (uint64_t)n * p.s_n + (uint64_t)(r / p.Q) * p.s_p + (uint64_t)(r % p.Q) * p.s_q +
                       (uint64_t)(nt * BN) * p.s_c;
            }
            uint16_t* out16 = reinterpret_cast<uint16_t*>(p.out);
            const uint32_t taddr = tmem + acc * BN + ((uint32_t)(quarter * 32) << 16);
            if (p.c_rows && p.out_low) {
                // 16-bit rows straight from registers: each lane writes its
                // own row's 32 columns (64 bytes) as four 16-byte stores, or
                // eight 8-byte ones where the row is only 8-byte aligned.
                // (Staging through shared memory for row-coalesced stores
                // measured slower here: the stores queued behind the ring's
                // TMA and tensor-core traffic.)
#pragma unroll 1
                for (int c0 = c_lo; c0 < c_lo + COLS; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(taddr + c0, v);
                    tmem_wait_ld();
                    if (p.act) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(gelu_tanh(__uint_as_float(v[j])));
                    }
                    if (base != ~0ull) {
                        uint32_t w[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            w[j] = encode_low_pair(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]), p.out_low);
                        uint16_t* dst = out16 + base + c0;
                        if ((reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
                            // 32-byte stores: one full sector per instruction
#pragma unroll
                            for (int q = 0; q < 2; ++q)
                                asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(dst + 16 * q),
                                             "r"(w[8 * q]), "r"(w[8 * q + 1]), "r"(w[8 * q + 2]), "r"(w[8 * q + 3]),
                                             "r"(w[8 * q + 4]), "r"(w[8 * q + 5]), "r"(w[8 * q + 6]), "r"(w[8 * q + 7])
                                             : "memory");
                        } else if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                reinterpret_cast<uint4*>(dst)[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
                        } else {
#pragma unroll
                            for (int q = 0; q < 8; ++q) reinterpret_cast<uint2*>(dst)[q] = make_uint2(w[2 * q], w[2 * q + 1]);
                        }
                    }
                }
            } else if (p.c_rows) {
                float* st = epi + (warp - 2) * (32 * C::EPI_PITCH);
                const uint64_t my_base = base;
#pragma unroll 1
                for (int c0 = c_lo; c0 < c_lo + COLS; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(taddr + c0, v);
                    tmem_wait_ld();
                    if (p.act) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(gelu_tanh(__uint_as_float(v[j])));
                    }
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        *reinterpret_cast<float4*>(st + lane * C::EPI_PITCH + 4 * q) =
                            make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                        __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
                    __syncwarp();
                    // accumulate: the chunk's eight float4 of the existing
                    // output are loaded before any store (distinct rows, no
                    // aliasing), so their latencies overlap
                    float4 prev[8];
                    if (p.accumulate) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int r = i * 4 + (lane >> 3), cc = lane & 7;
                            const uint64_t rb = __shfl_sync(0xffffffffu, my_base, r);
                            prev[i] = rb != ~0ull ? *reinterpret_cast<const float4*>(p.out + rb + c0 + 4 * cc)
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int r = i * 4 + (lane >> 3), cc = lane & 7;
                        const uint64_t rb = __shfl_sync(0xffffffffu, my_base, r);
                        const float4 val = *reinterpret_cast<const float4*>(st + r * C::EPI_PITCH + 4 * cc);
                        if (rb != ~0ull) {
                            if (p.out_low)
                                *reinterpret_cast<uint2*>(out16 + rb + c0 + 4 * cc) =
                                    make_uint2(encode_low_pair(val.x, val.y, p.out_low),
                                               encode_low_pair(val.z, val.w, p.out_low));
                            else if (p.accumulate)
                                *reinterpret_cast<float4*>(p.out + rb + c0 + 4 * cc) =
                                    make_float4(prev[i].x + val.x, prev[i].y + val.y, prev[i].z + val.z, prev[i].w + val.w);
                            else
                                *reinterpret_cast<float4*>(p.out + rb + c0 + 4 * cc) = val;
                        }
                    }
                    __syncwarp();
                }
            } else {
#pragma unroll 1
                for (int c0 = c_lo; c0 < c_lo + COLS; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(taddr + c0, v);
                    tmem_wait_ld();
                    if (p.act) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(gelu_tanh(__uint_as_float(v[j])));
                    }
                    if (base != ~0ull) {
                        if (p.out_low == FB_BF16) {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                out16[base + (uint64_t)(c0 + j) * p.s_c] = encode_bf16(__uint_as_float(v[j]));
                        } else if (p.out_low) {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                out16[base + (uint64_t)(c0 + j) * p.s_c] = encode_f16(__uint_as_float(v[j]));
                        } else if (p.accumulate) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) p.out[base + (uint64_t)(c0 + j) * p.s_c] += __uint_as_float(v[j]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j) p.out[base + (uint64_t)(c0 + j) * p.s_c] = __uint_as_float(v[j]);
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive_cluster(tempty0 + (uint32_t)(acc * sizeof(uint64_t)));  // the even CTA's accumulator slot
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
    }
    // Both CTAs stay until every pair MMA has completed (the even CTA's MMA
    // warp waited on `drain`) and every remote arrive has landed.
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------ host

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
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

PFN_cuTensorMapEncodeIm2col_v12000 encode_im2col() {
    static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(ptr);
    });
    return fn;
}

// 2-D K-major tile map over rows x cols 16-bit elements (cols contiguous,
// row pitch `pitch` elements), box {64, box_rows}, 128B swizzle.
bool make_2d_map(CUtensorMap* map, const void* ptr, uint32_t fmt, uint64_t cols, uint64_t rows, uint64_t pitch,
                 uint32_t box_rows) {
    auto enc = encode_tiled();
    if (!enc) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch * 2};
    cuuint32_t box[2] = {BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, fmt ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr),
               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_im2col_map(CUtensorMap* map, const void* ptr, uint32_t fmt, uint64_t C, uint64_t W, uint64_t H, uint64_t N,
                     int lower_w, int lower_h, int upper_w, int upper_h, uint32_t stride_w, uint32_t stride_h) {
    auto enc = encode_im2col();
    if (!enc) return false;
    cuuint64_t dims[4] = {C, W, H, N};
    cuuint64_t strides[3] = {C * 2, W * C * 2, H * W * C * 2};
    int lower[2] = {lower_w, lower_h};
    int upper[2] = {upper_w, upper_h};
    cuuint32_t estr[4] = {1, stride_w, stride_h, 1};
    return enc(map, fmt ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(ptr),
               dims, strides, lower, upper, BK, BM, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Gathers OIHW-viewed weights into dense [O, R, S, C] rows (K-major B).
template <typename E>
__global__ void weights_to_ohwi_kernel(const E* w, uint64_t off, uint64_t so, uint64_t sc, uint64_t sr, uint64_t ss,
                                       uint32_t O, uint32_t Cc, uint32_t R, uint32_t S, E* out) {
    const uint64_t total = (uint64_t)O * R * S * Cc;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t c = i % Cc;
        uint64_t t = i / Cc;
        const uint32_t s = t % S;
        t /= S;
        const uint32_t r = t % R;
        const uint32_t o = t / R;
        out[i] = w[off + o * so + c * sc + r * sr + s * ss];
    }
}

// Weights into dense [O, C, kh, kw] rows (the K order of gathered patches).
template <typename E>
__global__ void weights_to_oihw_kernel(const E* w, uint64_t off, uint64_t so, uint64_t sc, uint64_t sr, uint64_t ss,
                                       uint32_t O, uint32_t Cc, uint32_t R, uint32_t S, E* out) {
    const uint64_t total = (uint64_t)O * Cc * R * S;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t s = i % S;
        uint64_t t = i / S;
        const uint32_t r = t % R;
        t /= R;
        const uint32_t c = t % Cc;
        const uint32_t o = t / Cc;
        out[i] = w[off + o * so + c * sc + r * sr + s * ss];
    }
}

// Space-to-depth for a convolution whose windows tile the input exactly
// (stride = kernel size, no padding, no dilation): row m = (n, p, q) of the
// GEMM operand holds the window's C * kh * kw inputs in (c, r, s) order, so
// the convolution is one dense [M, K] x [K, O] contraction.  Consecutive
// threads walk s, i.e. consecutive input columns: reads and writes coalesce.
template <typename E>
__global__ void patches_kernel(const E* x, uint64_t off, uint64_t sn, uint64_t sc, uint64_t sh, uint64_t sw, uint32_t Cc,
                               uint32_t R, uint32_t S, uint32_t P, uint32_t Q, uint64_t M, E* out) {
    const uint64_t K = (uint64_t)Cc * R * S;
    const uint64_t total = M * K;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t m = i / K, k = i % K;
        const uint32_t s = (uint32_t)(k % S);
        const uint32_t r = (uint32_t)((k / S) % R);
        const uint32_t c = (uint32_t)(k / ((uint64_t)S * R));
        const uint32_t q = (uint32_t)(m % Q);
        const uint32_t pp = (uint32_t)((m / Q) % P);
        const uint64_t n = m / ((uint64_t)Q * P);
        out[i] = x[off + n * sn + c * sc + ((uint64_t)pp * R + r) * sh + ((uint64_t)q * S + s) * sw];
    }
}

// The same gather eight elements (16 bytes) at a time, for windows whose
// width S is a multiple of eight over a unit-stride width axis with all other
// strides (and the offset) multiples of eight elements, in 32-bit index
// arithmetic: one index decomposition per 16-byte load and store.
__global__ void patches_vec8_kernel(const uint16_t* x, uint64_t off, uint64_t sn, uint64_t sc, uint64_t sh, uint32_t Cc,
                                    uint32_t R, uint32_t S, uint32_t P, uint32_t Q, uint32_t runs, uint16_t* out) {
    const uint32_t K = Cc * R * S;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < runs; t += gridDim.x * blockDim.x) {
        const uint32_t i = t * 8;
        const uint32_t m = i / K, k = i % K;
        const uint32_t s = k % S, r = (k / S) % R, c = k / (S * R);
        const uint32_t q = m % Q, pp = (m / Q) % P, n = m / (Q * P);
        const uint64_t src = off + n * sn + c * sc + ((uint64_t)pp * R + r) * sh + (uint64_t)q * S + s;
        reinterpret_cast<uint4*>(out)[t] = *reinterpret_cast<const uint4*>(x + src);
    }
}

template <int BN>
int launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const ConvGemmParams& p, cudaStream_t st) {
    using C = Cfg<BN>;
    auto kernel = conv_gemm_kernel<BN>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
        return launch_status("shared-memory attribute");
    const uint32_t tiles = p.m_tiles * p.n_tiles;
    const uint32_t grid = tiles < (uint32_t)sm_count() ? tiles : (uint32_t)sm_count();
    kernel<<<grid, THREADS, C::SMEM, st>>>(ta, tb, p);
    count_launch(kernel_name("conv_gemm_kernel", {BN}).c_str());
    return launch_status("kernel launch");
}

// The B operand of a launch: [N, K] rows with K contiguous, or (mn) [K, N]
// rows with N contiguous; `pitch` is the row pitch in elements.
struct BOperand {
    const void* ptr;
    uint32_t fmt;
    uint64_t k, n, pitch;
    bool mn;
};

bool make_b_map(CUtensorMap* m, const BOperand& b, uint32_t box_n) {
    return b.mn ? make_2d_map(m, b.ptr, b.fmt, b.n, b.k, b.pitch, BK) : make_2d_map(m, b.ptr, b.fmt, b.k, b.n, b.pitch, box_n);
}

// 2-CTA clusters of the pair kernel that can be resident at once (0: none).
template <int BN, int EPW>
int pair_clusters() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (cached[dev] == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (unsigned)sm_count());
        cfg.blockDim = dim3(PairCfg<BN, EPW>::THREADS);
        cfg.dynamicSmemBytes = PairCfg<BN, EPW>::SMEM;
        int n = 0;
        if (cudaFuncSetAttribute(conv_gemm_pair_kernel<BN, EPW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 PairCfg<BN, EPW>::SMEM) != cudaSuccess ||
            cudaOccupancyMaxActiveClusters(&n, conv_gemm_pair_kernel<BN, EPW>, &cfg) != cudaSuccess || n < 1) {
            (void)cudaGetLastError();
            n = -1;
        }
        cached[dev] = n;
    }
    return cached[dev] > 0 ? cached[dev] : 0;
}

template <int BN, int EPW>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb_half, const ConvGemmParams& p, int clusters_max,
                cudaStream_t st) {
    using C = PairCfg<BN, EPW>;
    if (cudaFuncSetAttribute(conv_gemm_pair_kernel<BN, EPW>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
        return launch_status("shared-memory attribute");
    const uint32_t tiles = (p.m_tiles + 1) / 2 * p.n_tiles;
    const uint32_t clusters = tiles < (uint32_t)clusters_max ? tiles : (uint32_t)clusters_max;
    conv_gemm_pair_kernel<BN, EPW><<<2 * clusters, C::THREADS, C::SMEM, st>>>(ta, tb_half, p);
    count_launch(kernel_name("conv_gemm_pair_kernel", {BN, EPW}).c_str());
    return launch_status("kernel launch");
}

// Tile shape and kernel for one GEMM launch (p.n_tiles is set here).  CTA
// pairs when N is a multiple of 256 or (K-major B) 192 and there are at least
// two 128-row M tiles: the width with the fewest tile-rounds x width wins
// (ties to 256, fewer re-reads of A).  Otherwise one CTA per 128 x BN tile
// with the widest BN in {256, 128, 64} dividing N.  FB_ERR_UNSUPPORTED when
// N is not a multiple of 64.
int launch_tiles(const CUtensorMap& ta, const BOperand& b, ConvGemmParams p, cudaStream_t st) {
    const uint64_t N = b.n;
    if (p.m_tiles >= 2) {
        const uint64_t m_pairs = (p.m_tiles + 1) / 2;
        // Eight (256 wide) or twelve (192 wide) epilogue warps for the
        // epilogues that do more than store f32 sums: GELU, the
        // read-modify-write add and the 16-bit rounding, each of which
        // otherwise outlasts a short (K = 768) main loop; plain f32 stores
        // keep four and the deeper ring.
        const bool heavy_epilogue = p.act || p.accumulate || p.out_low;
        int best = 0;
        uint64_t best_cost = ~0ull;
        int best_clusters = 0;
        for (int bn : {256, 192}) {
            if (N % bn != 0 || (b.mn && bn != 256)) continue;
            const int cl = bn == 256 ? (heavy_epilogue ? pair_clusters<256, 8>() : pair_clusters<256, 4>())
                                     : (heavy_epilogue ? pair_clusters<192, 12>() : pair_clusters<192, 4>());
            if (cl == 0) continue;
            const uint64_t tiles = m_pairs * (N / bn);
            const uint64_t cost = (tiles + cl - 1) / cl * bn;
            if (cost < best_cost) {
                best_cost = cost;
                best = bn;
                best_clusters = cl;
            }
        }
        // Few tiles with the plain f32 epilogue (a convolution sharded to a
        // few dozen images per GPU): when the pair tiles leave clusters idle,
        // single-CTA tiles of the narrowest width that still fits one wave
        // spread the work over more SMs.  Measured with f32 outputs: C3a at
        // 32 images 24.5 -> 22.5 us (128 wide), at 64 images 26.6 -> 24.5 us
        // (256 wide); C3b at 32 images 18.4 -> 14.3 us.  The heavy epilogues
        // keep their pairs (C5 projections at 8 images were no faster on
        // single CTAs).
        if (best && !heavy_epilogue && m_pairs * (N / best) < (uint64_t)best_clusters) {
            int single = 0;
            for (int bn : {256, 128})
                if (N % bn == 0 && (uint64_t)p.m_tiles * (N / bn) <= (uint64_t)sm_count()) single = bn;
            if (single) {
                CUtensorMap tb;
                if (!make_b_map(&tb, b, (uint32_t)single)) return FB_ERR_UNSUPPORTED;
                p.n_tiles = (uint32_t)(N / single);
                return single == 256 ? launch_bn<256>(ta, tb, p, st) : launch_bn<128>(ta, tb, p, st);
            }
        }
        if (best) {
            CUtensorMap tb;
            if (!make_b_map(&tb, b, (uint32_t)best / 2)) return FB_ERR_UNSUPPORTED;
            p.n_tiles = (uint32_t)(N / best);
            if (heavy_epilogue)
                return best == 256 ? launch_pair<256, 8>(ta, tb, p, best_clusters, st)
                                   : launch_pair<192, 12>(ta, tb, p, best_clusters, st);
            return best == 256 ? launch_pair<256, 4>(ta, tb, p, best_clusters, st)
                               : launch_pair<192, 4>(ta, tb, p, best_clusters, st);
        }
    }
    const int BN = N % 256 == 0 ? 256 : N % 128 == 0 ? 128 : N % 64 == 0 ? 64 : 0;
    if (BN == 0) return FB_ERR_UNSUPPORTED;
    CUtensorMap tb;
    if (!make_b_map(&tb, b, (uint32_t)BN)) return FB_ERR_UNSUPPORTED;
    p.n_tiles = (uint32_t)(N / BN);
    switch (BN) {
        case 256: return launch_bn<256>(ta, tb, p, st);
        case 128: return launch_bn<128>(ta, tb, p, st);
        default: return launch_bn<64>(ta, tb, p, st);
    }
}

}  // namespace

uint32_t read_gemm_status() {
    uint32_t v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(zero));
    return v;
}

// Channels-contiguous output whose rows start on 16-byte (f32) or 8-byte
// (16-bit) boundaries: the epilogue may store each row's 32-column chunks as
// float4 / four packed 16-bit values.
bool c_rows_ok(const ConvArgs& a) {
    if (a.out_stride_c != 1) return false;
    const uint64_t strides[3] = {a.out_stride_n, a.out_strides[0], a.out_strides[1]};
    for (uint64_t st : strides)
        if (st % 4 != 0) return false;
    const uint64_t esz = a.out_low ? 2 : 4;
    return (reinterpret_cast<uintptr_t>(a.output) + a.out_offset * esz) % (4 * esz) == 0;
}

// Element offset of a batch index in a batch nest (row-major).
uint64_t host_nest_offset(const Nest& n, uint64_t linear) {
    uint64_t off = 0;
    for (int d = (int)n.rank - 1; d >= 0; --d) {
        off += (linear % n.dims[d]) * n.strides[d];
        linear /= n.dims[d];
    }
    return off;
}

// Low-precision GEMM on the implicit-GEMM kernel: A = left rows [M, K] (K
// contiguous), B = right as [K, N] rows (N contiguous: MN-major operand) or
// [N, K] rows (K contiguous), one launch per batch index.
int launch_gemm_tc(const GemmArgs& g, void* stream) {
    if (g.dtype != FB_BF16 && g.dtype != FB_F16) return FB_ERR_UNSUPPORTED;
    if (g.M == 0 || g.N == 0 || g.K == 0 || g.K % BK != 0 || g.M > 0x7fffffffull) return FB_ERR_UNSUPPORTED;
    const int BN = g.N % 256 == 0 ? 256 : g.N % 128 == 0 ? 128 : g.N % 64 == 0 ? 64 : 0;
    if (BN == 0) return FB_ERR_UNSUPPORTED;
    if (g.a_sk != 1 || g.a_sm % 8 != 0 || g.a_sm < g.K) return FB_ERR_UNSUPPORTED;
    const bool b_mn = g.b_sn == 1 && g.b_sk % 8 == 0 && g.b_sk >= g.N;
    const bool b_k = !b_mn && g.b_sk == 1 && g.b_sn % 8 == 0 && g.b_sn >= g.K;
    if (!b_mn && !b_k) return FB_ERR_UNSUPPORTED;
    const uint64_t esz_out = g.out_low ? 2 : 4;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint32_t fmt = g.dtype == FB_BF16 ? 1 : 0;
    for (uint64_t bi = 0; bi < g.batch; ++bi) {
        const uint16_t* a = static_cast<const uint16_t*>(g.a) + g.a_off + host_nest_offset(g.a_batch, bi);
        const uint16_t* b = static_cast<const uint16_t*>(g.b) + g.b_off + host_nest_offset(g.b_batch, bi);
        const uint64_t o_off = g.o_off + host_nest_offset(g.o_batch, bi);
        if (reinterpret_cast<uintptr_t>(a) % 16 != 0 || reinterpret_cast<uintptr_t>(b) % 16 != 0) return FB_ERR_UNSUPPORTED;
        CUtensorMap ta;
        if (!make_2d_map(&ta, a, fmt, g.K, g.M, g.a_sm, BM)) return FB_ERR_UNSUPPORTED;
        const BOperand bop{b, fmt, g.K, g.N, b_mn ? g.b_sk : g.b_sn, b_mn};
        ConvGemmParams p{};
        p.mode = 0;
        p.fmt = fmt;
        p.M = (uint32_t)g.M;
        p.P = 1;
        p.Q = (uint32_t)g.M;
        p.c_blocks = p.k_blocks = (uint32_t)(g.K / BK);
        p.S = 1;
        p.stride_h = p.stride_w = p.dil_h = p.dil_w = 1;
        p.m_tiles = (uint32_t)((g.M + BM - 1) / BM);
        p.out = static_cast<float*>(g.out);
        p.out_offset = o_off;
        p.s_n = 0;
        p.s_p = 0;
        p.s_q = g.o_sm;
        p.s_c = g.o_sn;
        p.out_low = g.out_low;
        p.b_mn = b_mn ? 1 : 0;
        p.c_rows = g.o_sn == 1 && g.o_sm % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(g.out) + o_off * esz_out) % (4 * esz_out) == 0;
        const int r = launch_tiles(ta, bop, p, st);
        if (r != FB_OK) return r;
    }
    return FB_OK;
}

int launch_patches(const ConvArgs& a, void* stream) {
    const uint64_t C = a.channels_per_group, R = a.k_dims[0], S = a.k_dims[1], O = a.out_channels;
    const uint64_t P = a.out_dims[0], Q = a.out_dims[1], N = a.batch;
    const uint64_t K = C * R * S, M = N * P * Q;
    if (K % BK != 0 || M == 0 || M > 0x7fffffffull || M * K > (1ull << 40)) return FB_ERR_UNSUPPORTED;
    const int BN = O % 256 == 0 ? 256 : O % 128 == 0 ? 128 : O % 64 == 0 ? 64 : 0;
    if (BN == 0) return FB_ERR_UNSUPPORTED;
    const uint32_t fmt = a.dtype == FB_BF16 ? 1 : 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // A operand: gathered windows.
    void* pa = scratch(stream, M * K * 2 + 256, SCRATCH_CONV_PATCH);
    if (!pa) return FB_ERR_DRIVER;
    {
        const uint64_t total = M * K;
        const bool vec8 = S % 8 == 0 && a.in_strides[1] == 1 && a.in_offset % 8 == 0 && a.in_stride_n % 8 == 0 &&
                          a.in_stride_c % 8 == 0 && a.in_strides[0] % 8 == 0 && total < (1ull << 32) &&
                          reinterpret_cast<uintptr_t>(a.input) % 16 == 0 && reinterpret_cast<uintptr_t>(pa) % 16 == 0;
        if (vec8) {
            const uint64_t runs = total / 8;
            const unsigned grid = (unsigned)std::min<uint64_t>((runs + 255) / 256, (uint64_t)sm_count() * 16);
            patches_vec8_kernel<<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(a.input), a.in_offset, a.in_stride_n,
                                                      a.in_stride_c, a.in_strides[0], (uint32_t)C, (uint32_t)R,
                                                      (uint32_t)S, (uint32_t)P, (uint32_t)Q, (uint32_t)runs,
                                                      static_cast<uint16_t*>(pa));
        } else {
            const unsigned grid = (unsigned)std::min<uint64_t>((total + 255) / 256, (uint64_t)sm_count() * 16);
            patches_kernel<uint16_t><<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(a.input), a.in_offset,
                                                            a.in_stride_n, a.in_stride_c, a.in_strides[0],
                                                            a.in_strides[1], (uint32_t)C, (uint32_t)R, (uint32_t)S,
                                                            (uint32_t)P, (uint32_t)Q, M, static_cast<uint16_t*>(pa));
        }
        count_launch(vec8 ? "patches_vec8_kernel" : "patches_kernel");
        if (cudaGetLastError() != cudaSuccess) return launch_status("patch gather");
    }
    // B operand: [O, C, kh, kw] rows, in place when the weights are stored so.
    const void* wptr = static_cast<const uint16_t*>(a.weight) + a.w_offset;
    const bool oihw = a.w_stride_o == K && a.w_stride_c == R * S && a.w_strides[0] == S && a.w_strides[1] == 1 &&
                      reinterpret_cast<uintptr_t>(wptr) % 16 == 0;
    if (!oihw) {
        void* tmp = scratch(stream, O * K * 2 + 256, SCRATCH_CONV_WEIGHT);
        if (!tmp) return FB_ERR_DRIVER;
        const uint64_t total = O * K;
        const unsigned grid = (unsigned)std::min<uint64_t>((total + 255) / 256, (uint64_t)sm_count() * 8);
        weights_to_oihw_kernel<uint16_t><<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(a.weight), a.w_offset,
                                                               a.w_stride_o, a.w_stride_c, a.w_strides[0], a.w_strides[1],
                                                               (uint32_t)O, (uint32_t)C, (uint32_t)R, (uint32_t)S,
                                                               static_cast<uint16_t*>(tmp));
        count_launch("weights_to_oihw_kernel");
        if (cudaGetLastError() != cudaSuccess) return launch_status("weight gather");
        wptr = tmp;
    }
    CUtensorMap ta;
    if (!make_2d_map(&ta, pa, fmt, K, M, K, BM)) return FB_ERR_UNSUPPORTED;
    const BOperand bop{wptr, fmt, K, O, K, false};
    ConvGemmParams p{};
    p.mode = 0;
    p.fmt = fmt;
    p.M = (uint32_t)M;
    p.P = (uint32_t)P;
    p.Q = (uint32_t)Q;
    p.c_blocks = (uint32_t)(K / BK);
    p.k_blocks = (uint32_t)(K / BK);
    p.S = 1;
    p.stride_h = p.stride_w = p.dil_h = p.dil_w = 1;
    p.m_tiles = (uint32_t)((M + BM - 1) / BM);
    p.out = a.output;
    p.out_offset = a.out_offset;
    p.s_n = a.out_stride_n;
    p.s_c = a.out_stride_c;
    p.s_p = a.out_strides[0];
    p.s_q = a.out_strides[1];
    p.c_rows = c_rows_ok(a) ? 1 : 0;
    p.out_low = a.out_low;
    p.act = a.act;
    p.accumulate = a.accumulate;
    return launch_tiles(ta, bop, p, st);
}

int launch_conv_tc(const ConvArgs& a, void* stream) {
    if (a.dtype != FB_BF16 && a.dtype != FB_F16) return FB_ERR_UNSUPPORTED;
    if (a.spatial != 2 || a.outputs_per_group != a.out_channels) return FB_ERR_UNSUPPORTED;  // 2-D, one group
    const uint64_t C = a.channels_per_group, H = a.in_dims[0], W = a.in_dims[1];
    const uint64_t R = a.k_dims[0], S = a.k_dims[1], O = a.out_channels;
    const uint64_t P = a.out_dims[0], Q = a.out_dims[1], N = a.batch;
    if (O % 16 != 0 || O == 0) return FB_ERR_UNSUPPORTED;
    // Windows that tile the input exactly (a ViT patch embedding) go through
    // a space-to-depth gather and one dense GEMM, whatever the channel count.
    // (trailing padding is never reached when P * R == H and Q * S == W)
    const bool patches = a.stride[0] == R && a.stride[1] == S && a.pad[0] == 0 && a.pad[1] == 0 &&
                         a.dilation[0] == 1 && a.dilation[1] == 1 && (R > 1 || S > 1) && P * R == H && Q * S == W;
    if (patches) return launch_patches(a, stream);
    if (C % BK != 0) return FB_ERR_UNSUPPORTED;
    // Channels-last input: c stride 1, w stride C, h stride W*C, n stride H*W*C.
    if (a.in_stride_c != 1 || a.in_strides[1] != C || a.in_strides[0] != W * C || a.in_stride_n != H * W * C)
        return FB_ERR_UNSUPPORTED;
    const uintptr_t in_addr = reinterpret_cast<uintptr_t>(a.input) + a.in_offset * 2;
    if (in_addr % 16 != 0) return FB_ERR_UNSUPPORTED;
    const uint64_t M = N * P * Q;
    if (M == 0 || M > 0x7fffffffull || N * H * W * C > (1ull << 40)) return FB_ERR_UNSUPPORTED;
    const uint32_t fmt = a.dtype == FB_BF16 ? 1 : 0;
    const bool one_by_one = R == 1 && S == 1 && a.stride[0] == 1 && a.stride[1] == 1 && a.pad[0] == 0 && a.pad[1] == 0 &&
                            P == H && Q == W;
    // im2col corners: lower = -pad_before, upper = pad_after - (k - 1) * dilation,
    // each within [-128, 127] for two spatial dimensions; traversal stride <= 8.
    const int64_t pa_h = (int64_t)((P - 1) * a.stride[0] + (R - 1) * a.dilation[0] + 1) - (int64_t)(H + a.pad[0]);
    const int64_t pa_w = (int64_t)((Q - 1) * a.stride[1] + (S - 1) * a.dilation[1] + 1) - (int64_t)(W + a.pad[1]);
    const int64_t lower_h = -(int64_t)a.pad[0], lower_w = -(int64_t)a.pad[1];
    const int64_t upper_h = pa_h - (int64_t)((R - 1) * a.dilation[0]);
    const int64_t upper_w = pa_w - (int64_t)((S - 1) * a.dilation[1]);
    auto corner_ok = [](int64_t v) { return v >= -128 && v <= 127; };
    const bool im2col_ok = corner_ok(lower_h) && corner_ok(lower_w) && corner_ok(upper_h) && corner_ok(upper_w) &&
                           a.stride[0] <= 8 && a.stride[1] <= 8 && (R - 1) * a.dilation[0] < 65536 &&
                           (S - 1) * a.dilation[1] < 65536 && N * H * W * C * 2 >= (128u << 10);
    if (!one_by_one && !im2col_ok) return FB_ERR_UNSUPPORTED;
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    // B operand: dense [O, R*S*C] rows; gather when the weights are not OHWI.
    const uint64_t K = R * S * C;
    const void* wptr = static_cast<const uint16_t*>(a.weight) + a.w_offset;
    // (strides of unit kernel dimensions do not matter: [O, C, 1, 1] weights are dense rows)
    const bool ohwi = a.w_stride_c == 1 && (S == 1 || a.w_strides[1] == C) && (R == 1 || a.w_strides[0] == S * C) &&
                      a.w_stride_o == K && reinterpret_cast<uintptr_t>(wptr) % 16 == 0;
    if (!ohwi) {
        void* tmp = scratch(stream, O * K * 2 + 256, SCRATCH_CONV_WEIGHT);
        if (!tmp) return FB_ERR_DRIVER;
        const uint64_t total = O * K;
        const unsigned grid = (unsigned)std::min<uint64_t>((total + 255) / 256, (uint64_t)sm_count() * 8);
        weights_to_ohwi_kernel<uint16_t><<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(a.weight), a.w_offset,
                                                               a.w_stride_o, a.w_stride_c, a.w_strides[0], a.w_strides[1],
                                                               (uint32_t)O, (uint32_t)C, (uint32_t)R, (uint32_t)S,
                                                               static_cast<uint16_t*>(tmp));
        count_launch("weights_to_ohwi_kernel");
        if (cudaGetLastError() != cudaSuccess) return FB_ERR_DRIVER;
        wptr = tmp;
    }
    const int BN = O % 256 == 0 ? 256 : O % 128 == 0 ? 128 : O % 64 == 0 ? 64 : 0;
    if (BN == 0) return FB_ERR_UNSUPPORTED;

    CUtensorMap ta;
    const void* in_ptr = static_cast<const uint16_t*>(a.input) + a.in_offset;
    const BOperand bop{wptr, fmt, K, O, K, false};
    ConvGemmParams p{};
    if (one_by_one) {
        if (!make_2d_map(&ta, in_ptr, fmt, C, M, C, BM)) return FB_ERR_UNSUPPORTED;
        p.mode = 0;
    } else {
        if (!make_im2col_map(&ta, in_ptr, fmt, C, W, H, N, (int)lower_w, (int)lower_h, (int)upper_w, (int)upper_h,
                             (uint32_t)a.stride[1], (uint32_t)a.stride[0]))
            return FB_ERR_UNSUPPORTED;
        p.mode = 1;
    }
    p.fmt = fmt;
    p.M = (uint32_t)M;
    p.P = (uint32_t)P;
    p.Q = (uint32_t)Q;
    p.c_blocks = (uint32_t)(C / BK);
    p.k_blocks = (uint32_t)(K / BK);
    p.S = (uint32_t)S;
    p.pad_h = (int32_t)a.pad[0];
    p.pad_w = (int32_t)a.pad[1];
    p.stride_h = (int32_t)a.stride[0];
    p.stride_w = (int32_t)a.stride[1];
    p.dil_h = (int32_t)a.dilation[0];
    p.dil_w = (int32_t)a.dilation[1];
    p.m_tiles = (uint32_t)((M + BM - 1) / BM);
    p.out = a.output;
    p.out_offset = a.out_offset;
    p.s_n = a.out_stride_n;
    p.s_c = a.out_stride_c;
    p.s_p = a.out_strides[0];
    p.s_q = a.out_strides[1];
    p.c_rows = c_rows_ok(a) ? 1 : 0;
    p.out_low = a.out_low;
    p.act = a.act;
    p.accumulate = a.accumulate;
    return launch_tiles(ta, bop, p, st);
}

}  // namespace fb
