// tcgen05.mma issue-pattern rates on one B200 (measurement tool, not part of
// the library).  One CTA per SM allocates all 512 TMEM columns, fills 128 KiB
// of shared memory with small BF16 values, and one thread issues REPS groups
// of an MMA pattern (eight K=16 steps per chain); the CTA's clock64 span gives
// flop/clk/SM against the 8192 of a full-rate M=128 pipe.  Operands never
// leave shared memory / TMEM, so only the tensor pipe and its operand path
// are measured.  Every wait is bounded (2 s), all addresses stay inside the
// buffers laid out below.
//
// Build and run:
//   nvcc -O3 -std=c++17 -gencode arch=compute_100a,code=sm_100a -I include \
//        forma_b200/microbench/umma_issue.cu -o forma_b200/microbench/umma_issue -lcuda
//   ./forma_b200/microbench/umma_issue
#include <cuda.h>

#include <cstdint>
#include <cstdio>

#include "../csrc/async.cuh"
#include "../csrc/tc.cuh"

using namespace fb;

namespace {

// Shared memory (1024-aligned base):
//   Q  [128 rows x 128 k] K-major            0 ..  32 KiB
//   K  [up to 256 rows x 128 k] K-major      32 ..  96 KiB   (P for SS PV lives at 64 KiB)
//   V  [128 k x 128 n] MN-major              96 .. 128 KiB
// TMEM: accumulators at columns 0..511.  The attention order mirrors the
// kernel's plan: S_0 at 0, S_1 at 128, O_0 at 256, O_1 at 384, and each PV
// reads its A operand (P) from its own tile's S columns.
constexpr uint32_t SMEM = 129 * 1024;
constexpr int REPS = 4000;

enum Pattern : int {
    SS_N64, SS_N128, SS_N256,  // one accumulator chain
    SS_N256_X2,                // two N=256 chains interleaved per instruction
    SS_N128_X4,                // four N=128 chains, same operands
    S_PV_SS,                   // S (K-major B) / PV (MN-major B, A = P in SMEM) interleaved
    S_PV_TS,                   // S / PV with A from TMEM, interleaved
    ATTN_ORDER,                // groups PV_0 (TS), S_0, PV_1 (TS), S_1
    ATTN_ORDER_TMEM_BUSY,      // the same while three warps stream tcgen05.ld/st like a softmax
    RT_ONE_LANE,               // N=256 chain chosen by a runtime argument, issued from one lane
    RT_WARP,                   // the same issued by the whole warp with elect.sync
    N_PATTERNS
};
const char* kNames[N_PATTERNS] = {"SS N=64, one chain",  "SS N=128, one chain", "SS N=256, one chain",
                                  "SS N=256, 2 chains",  "SS N=128, 4 chains",  "S + PV both SS, interleaved",
                                  "S (SS) + PV (TS), interleaved", "PV_0 TS, S_0, PV_1 TS, S_1 groups",
                                  "  the same, TMEM ld/st traffic", "runtime-selected N=256, one lane",
                                  "runtime-selected N=256, warp + elect"};
// output columns computed per group of eight K steps (flop = 2 * 128 * cols * 128)
const int kCols[N_PATTERNS] = {64, 128, 256, 512, 512, 256, 256, 512, 512, 256, 256};

__device__ __forceinline__ uint64_t mn_desc(uint32_t addr, uint32_t lbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

template <int PATTERN>
__global__ void __launch_bounds__(128, 1) umma_issue_kernel(unsigned long long* out, int sel) {
    extern __shared__ unsigned char raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint32_t tmem_base;
    __shared__ __align__(8) uint64_t bar;
    const int warp = threadIdx.x / 32;
    uint16_t* h = reinterpret_cast<uint16_t*>(sm);
    for (uint32_t i = threadIdx.x; i < 128u * 1024u / 2u; i += blockDim.x) {
        uint32_t x = i * 2654435761u + blockIdx.x;
        x ^= x >> 15;
        h[i] = (uint16_t)(0x3c00u | (x & 0x7fu) | ((x & 0x100u) << 7));  // BF16 in +-[2^-7, 2^-6)
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base, 512);
        tmem_relinquish();
    }
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    __shared__ volatile int done;
    if (threadIdx.x == 0) done = 0;
    __syncthreads();
    if (PATTERN == ATTN_ORDER_TMEM_BUSY && warp >= 1) {
        // tcgen05.ld of 64 columns at a time from O_1's columns (448..511;
        // the values are discarded, only the traffic matters: reads race
        // harmlessly with the MMAs' writes) until the issuing thread ends.
        // The loop condition is warp-uniform (tcgen05.ld is .sync.aligned)
        // and bounded by ~1 s of clocks.
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        const long long limit = clock64() + 2000000000ll;
        uint32_t v[32], sink = 0;
        while (__all_sync(0xffffffffu, !done && clock64() < limit)) {
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                tmem_ld32(tmem + lane_base + 448 + c * 32, v);
                tmem_wait_ld();
                sink ^= v[c];
            }
        }
        if (sink == 0x9e3779b9u) out[2 * gridDim.x] = sink;  // keeps the loads; practically never true
    }
    if (PATTERN == RT_ONE_LANE || PATTERN == RT_WARP) {
        // `sel` (2 at run time) picks N=256 among runtime branches, as an issue
        // loop with runtime tile parameters would.
        const uint32_t q = smem_u32(sm), kk = smem_u32(sm + 32 * 1024);
        const uint32_t i128 = f16_idesc(1, 128, 128), i256 = f16_idesc(1, 128, 256);
        const bool issuer = PATTERN == RT_WARP ? warp == 0 : threadIdx.x == 0;
        if (issuer) {
            const long long t0 = clock64();
            for (int r = 0; r < REPS; ++r)
                for (int k = 0; k < 8; ++k) {
                    const uint32_t qo = (uint32_t)((k / 4) * (128 * 128) + (k % 4) * 32);
                    const uint32_t k256 = (uint32_t)((k / 4) * (256 * 128) + (k % 4) * 32);
                    const uint32_t acc = (r | k) != 0;
                    if (PATTERN == RT_WARP) {
                        if (sel == 1) umma_f16_ss_warp(tmem, sw128_desc(q + qo), sw128_desc(kk + qo), i128, acc);
                        else if (sel == 2) umma_f16_ss_warp(tmem, sw128_desc(q + qo), sw128_desc(kk + k256), i256, acc);
                    } else {
                        if (sel == 1) umma_f16_ss(tmem, sw128_desc(q + qo), sw128_desc(kk + qo), i128, acc);
                        else if (sel == 2) umma_f16_ss(tmem, sw128_desc(q + qo), sw128_desc(kk + k256), i256, acc);
                    }
                }
            if (PATTERN == RT_WARP) umma_commit_warp(&bar);
            else umma_commit(&bar);
            const bool ok = __all_sync(PATTERN == RT_WARP ? 0xffffffffu : 1u, mbar_wait(&bar, 0));
            const long long t1 = clock64();
            if (threadIdx.x == 0) {
                out[blockIdx.x * 2] = (unsigned long long)(t1 - t0);
                out[blockIdx.x * 2 + 1] = ok ? 1 : 0;
            }
        }
    } else if (threadIdx.x == 0) {
        const uint32_t q = smem_u32(sm), kk = smem_u32(sm + 32 * 1024), p = smem_u32(sm + 64 * 1024),
                       v = smem_u32(sm + 96 * 1024);
        const uint32_t i64 = f16_idesc(1, 128, 64), i128 = f16_idesc(1, 128, 128), i256 = f16_idesc(1, 128, 256);
        const uint32_t i128mn = i128 | (1u << 16);
        const long long t0 = clock64();
        for (int r = 0; r < REPS; ++r) {
            if (PATTERN == ATTN_ORDER || PATTERN == ATTN_ORDER_TMEM_BUSY) {
                // four groups per iteration, each eight K steps, fully unrolled
#pragma unroll
                for (int g = 0; g < 4; ++g)
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const uint32_t qo = (uint32_t)((k / 4) * (128 * 128) + (k % 4) * 32);
                        const uint64_t vd = mn_desc(v + k * 16 * 128, 128 * 128);
                        if (g == 0) umma_f16_ts(tmem + 256, tmem + 0 + k * 8, vd, i128mn, 1u);
                        else if (g == 1) umma_f16_ss(tmem, sw128_desc(q + qo), sw128_desc(kk + qo), i128, k != 0);
                        else if (g == 2) umma_f16_ts(tmem + 384, tmem + 128 + k * 8, vd, i128mn, 1u);
                        else umma_f16_ss(tmem + 128, sw128_desc(q + qo), sw128_desc(kk + qo), i128, k != 0);
                    }
                continue;
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t acc = (r | k) != 0;
                const uint32_t qo = (uint32_t)((k / 4) * (128 * 128) + (k % 4) * 32);
                const uint32_t k64 = (uint32_t)((k / 4) * (64 * 128) + (k % 4) * 32);
                const uint32_t k256 = (uint32_t)((k / 4) * (256 * 128) + (k % 4) * 32);
                const uint64_t vd = mn_desc(v + k * 16 * 128, 128 * 128);
                switch (PATTERN) {
                    case SS_N64: umma_f16_ss(tmem, sw128_desc(q + qo), sw128_desc(kk + k64), i64, acc); break;
                    case SS_N128: umma_f16_ss(tmem, sw128_desc(q + qo), sw128_desc(kk + qo), i128, acc); break;
                    case SS_N256: umma_f16_ss(tmem, sw128_desc(q + qo), sw128_desc(kk + k256), i256, acc); break;
                    case SS_N256_X2:
                        umma_f16_ss(tmem, sw128_desc(q + qo), sw128_desc(kk + k256), i256, acc);
                        umma_f16_ss(tmem + 256, sw128_desc(q + qo), sw128_desc(kk + k256), i256, acc);
                        break;
                    case SS_N128_X4:
                        for (int c = 0; c < 4; ++c)
                            umma_f16_ss(tmem + 128 * c, sw128_desc(q + qo), sw128_desc(kk + qo), i128, acc);
                        break;
                    case S_PV_SS:
                        umma_f16_ss(tmem, sw128_desc(q + qo), sw128_desc(kk + qo), i128, acc);
                        umma_f16_ss(tmem + 128, sw128_desc(p + qo), vd, i128mn, acc);
                        break;
                    case S_PV_TS:  // S_0 at 0; PV_1 into O_1 at 384 with P from S_1's columns
                        umma_f16_ss(tmem, sw128_desc(q + qo), sw128_desc(kk + qo), i128, acc);
                        umma_f16_ts(tmem + 384, tmem + 128 + k * 8, vd, i128mn, acc);
                        break;
                    default:
                        break;
                }
            }
        }
        umma_commit(&bar);
        const bool ok = mbar_wait(&bar, 0);
        const long long t1 = clock64();
        out[blockIdx.x * 2] = (unsigned long long)(t1 - t0);
        out[blockIdx.x * 2 + 1] = ok ? 1 : 0;
        done = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace

int main() {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    unsigned long long* d = nullptr;
    if (cudaMalloc(&d, ((size_t)sms * 2 + 1) * 8) != cudaSuccess) return 1;  // + the sink slot
    void (*kernels[N_PATTERNS])(unsigned long long*, int) = {
        umma_issue_kernel<SS_N64>,  umma_issue_kernel<SS_N128>,    umma_issue_kernel<SS_N256>,
        umma_issue_kernel<SS_N256_X2>, umma_issue_kernel<SS_N128_X4>, umma_issue_kernel<S_PV_SS>,
        umma_issue_kernel<S_PV_TS>, umma_issue_kernel<ATTN_ORDER>, umma_issue_kernel<ATTN_ORDER_TMEM_BUSY>,
        umma_issue_kernel<RT_ONE_LANE>, umma_issue_kernel<RT_WARP>};
    for (auto k : kernels) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    printf("%-36s %14s %14s\n", "pattern", "cycles/group", "flop/clk/SM");
    for (int pat = 0; pat < N_PATTERNS; ++pat) {
        for (int rep = 0; rep < 2; ++rep) {  // first launch warms up
            kernels[pat]<<<sms, 128, SMEM>>>(d, 2);
            const cudaError_t e = cudaDeviceSynchronize();
            if (e != cudaSuccess) {
                printf("error: %s\n", cudaGetErrorString(e));
                return 1;
            }
        }
        unsigned long long hbuf[2 * 256];
        cudaMemcpy(hbuf, d, (size_t)sms * 2 * 8, cudaMemcpyDeviceToHost);
        double cyc = 0;
        int ok = 0;
        for (int i = 0; i < sms; ++i) {
            cyc += (double)hbuf[2 * i];
            ok += (int)hbuf[2 * i + 1];
        }
        cyc /= sms;
        const double flop = 2.0 * 128 * kCols[pat] * 128 * REPS;
        printf("%-36s %14.1f %14.1f%s\n", kNames[pat], cyc / REPS, flop / cyc, ok == sms ? "" : "  (a wait timed out)");
    }
    cudaFree(d);
    return 0;
}
