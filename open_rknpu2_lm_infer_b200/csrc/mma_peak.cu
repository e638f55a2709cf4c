// tcgen05 tensor-core rate and exactness probes (measurement tool, not part of
// the MoE operator; built into libmoe_b200_peak.so and run by
// open_rknpu2_lm_infer_b200/mma_peak.py).
//
// mma_peak_rate: one CTA per SM; `issuers` threads (lane 0 of warps
// 0..issuers-1) each issue `iters` MMAs of M = 128 x N x K (K = 32 int8 or 16
// fp16 per instruction) back to back into their own accumulator columns (one
// accumulator, or `rot` of them in turn so that consecutive MMAs do not
// depend on each other), then commit and wait. Operands sit in shared memory in the 128-byte-swizzle
// K-major layout (A may instead come from tensor memory, the `ts` form the
// expert GEMMs use). Reports the median issuer cycles per MMA and the grid's
// wall time (CUDA events), from which ops/s follow. At N = 256 this is the
// dense int8 (or fp16) tensor-core peak of the part as this pool runs it.
//
// mma_peak_exact: kind::f16 with integer-valued fp16 operands (A in [-8, 7],
// B in [-127, 127]) accumulating K = 32 into fp32: every partial sum is an
// integer below 2^24, so an exact accumulation reproduces the int32 dot. The
// kernel compares each accumulator with the integer dot it computes itself and
// counts mismatches. All accesses are in bounds; no wait is unbounded.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <vector>

#include "common.cuh"

namespace {

using namespace moe;

constexpr int kThreads = 128;  // four warps: one per TMEM lane quadrant

__host__ __device__ constexpr uint32_t idesc_f16_(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                           uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_f16_ts_(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

// byte offset of (row, byte) in a rows x 128-byte operand stored with the
// 128-byte swizzle (8-row atoms of 1024 bytes, 16-byte chunk ^ row % 8)
__device__ __forceinline__ int sw128(int row, int byte) {
    return (row >> 3) * 1024 + (row & 7) * 128 + ((((byte >> 4) ^ (row & 7)) << 4) | (byte & 15));
}

__device__ __forceinline__ uint32_t lcg(uint32_t x) { return x * 1664525u + 1013904223u; }

// the bounded spin of a wait, kept out of line so that the issuing loop holds
// only the first try_wait and a branch
__device__ __noinline__ bool wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                       uint32_t* err) {
    return mbar_wait(bar, parity, abort_flag, err);
}

// KIND 0: int8, 1: fp16. A: 128 rows, B: N rows, one 128-byte k-block each.
template <int KIND, int N, bool TS>
__global__ void __launch_bounds__(kThreads, 1)
rate_kernel(int iters, int issuers, int rot, int gap, int waits, int mode,
            unsigned long long* cycles) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* As = smem;
    uint8_t* Bs = smem + 128 * 128;
    __shared__ uint64_t bar[4];
    __shared__ uint32_t tmem_s;
    __shared__ uint32_t err_s;  // bounded waits record a timeout here
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) err_s = 0;
    // operand bytes: small pseudo-random integers (int8 codes or fp16 ints)
    for (int i = threadIdx.x; i < (128 + N) * 128 / 4; i += kThreads) {
        const uint32_t r = lcg(i * 2654435761u + blockIdx.x);
        uint32_t v;
        if (KIND == 0) {
            v = r & 0x0F0F0F0Fu;
        } else {
            const __half2 h = __floats2half2_rn((float)((int)(r & 15) - 8), (float)((int)((r >> 8) & 127) - 64));
            v = *reinterpret_cast<const uint32_t*>(&h);
        }
        reinterpret_cast<uint32_t*>(smem)[i] = v;
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < 4; ++i) mbar_init(&bar[i], 1);
        fence_barrier_init();
        mbar_arrive(&bar[3]);  // completes phase 0 of bar[3]: a wait on parity 0 returns at once
    }
    if (warp == 0) {
        tmem_alloc(&tmem_s, 512);
        tmem_relinquish();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_s;
    constexpr int kACols = 32;  // A operand region (one 128-byte k-block per lane)
    if (TS) {
        // lane quadrant of this warp: row = 32 * warp + lane; column c = bytes 4c..4c+3
        // of the row's k-block (k-major, no swizzle in tensor memory)
        uint32_t o[32];
        const int row = 32 * warp + lane;
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = *reinterpret_cast<const uint32_t*>(As + sw128(row, 4 * c));
        tmem_st32(tmem + ((uint32_t)(32 * warp) << 16), o);
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Loop variants (mode >> 2): 0 bare MMA loop; 1 + a spin of `gap` cycles
    // after each MMA; 2 + `waits` try_waits on a completed phase; 3 + `waits`
    // bounded waits (the GEMM's mbar_wait). Lane 0 of each issuing warp runs it.
    const int variant = mode >> 2;
    if (warp < issuers && lane == 0) {
        constexpr uint32_t idesc = KIND == 0 ? idesc_i8(128, N) : idesc_f16_(128, N);
        // rot > 1: the MMAs rotate over rot accumulators (independent
        // instructions); rot = 1: every MMA accumulates into the previous one's
        const uint32_t dbase = tmem + kACols + warp * rot * N;
        const uint32_t a0 = smem_u32(As), b0 = smem_u32(Bs);
        unsigned long long t0 = 0, t1 = 0;
        bool ok = true;
        auto issue = [&](int i, int ri) {
            const int j = i & 3;  // the four 32-byte K steps of the k-block
            const uint64_t bd = smem_desc_k_sw128(b0 + 32 * j);
            const uint32_t d = dbase + ri * N;
            const uint32_t acc = i >= rot ? 1u : 0u;
            if (KIND == 0) {
                if (TS) mma_i8_ts(d, tmem + 8 * j, bd, idesc, acc);
                else mma_i8(d, smem_desc_k_sw128(a0 + 32 * j), bd, idesc, acc);
            } else {
                if (TS) mma_f16_ts_(d, tmem + 8 * j, bd, idesc, acc);
                else mma_f16_ss(d, smem_desc_k_sw128(a0 + 32 * j), bd, idesc, acc);
            }
        };
        int never = 0;
        t0 = clock64();
        if (variant == 0) {
            int ri = 0;
            for (int i = 0; i < iters; ++i) {
                issue(i, ri);
                if (++ri == rot) ri = 0;
            }
        } else if (variant == 1) {
            int ri = 0;
            for (int i = 0; i < iters; ++i) {
                issue(i, ri);
                if (++ri == rot) ri = 0;
                if (gap > 0) {
                    const unsigned long long g0 = clock64();
                    while (clock64() - g0 < (unsigned long long)gap) {
                    }
                }
            }
        } else if (variant == 2) {
            int ri = 0;
            for (int i = 0; i < iters; ++i) {
                issue(i, ri);
                if (++ri == rot) ri = 0;
                for (int w = 0; w < waits; ++w) mbar_try_wait(&bar[3], 0);
            }
        } else if (variant == 3) {
            int ri = 0;
            for (int i = 0; i < iters; ++i) {
                issue(i, ri);
                if (++ri == rot) ri = 0;
                for (int w = 0; w < waits; ++w) mbar_wait(&bar[3], 0, &never, &err_s);
            }
        } else if (variant == 4) {
            // waits as an inline try_wait with the bounded spin out of line, unrolled
            int ri = 0;
            for (int i = 0; i < iters; ++i) {
                issue(i, ri);
                if (++ri == rot) ri = 0;
                if (waits > 0 && !mbar_try_wait(&bar[3], 0)) wait_slow(&bar[3], 0, &never, &err_s);
                if (waits > 1 && !mbar_try_wait(&bar[3], 0)) wait_slow(&bar[3], 0, &never, &err_s);
            }
        } else if (variant == 5) {
            // a commit to an mbarrier after every `gap`-th MMA (gap >= 1)
            int ri = 0;
            for (int i = 0; i < iters; ++i) {
                issue(i, ri);
                if (++ri == rot) ri = 0;
                if (gap > 0 && (i % gap) == gap - 1) mma_commit(&bar[2]);
            }
        } else {
            // four MMAs unrolled per iteration, then one wait (inline fast path)
            for (int i = 0; i < iters; i += 4) {
                issue(i, 0);
                issue(i + 1, 1 % rot);
                issue(i + 2, 2 % rot);
                issue(i + 3, 3 % rot);
                if (waits > 0 && !mbar_try_wait(&bar[3], 0)) wait_slow(&bar[3], 0, &never, &err_s);
                if (waits > 1) mma_commit(&bar[2]);
            }
        }
        mma_commit(&bar[warp]);
        ok = mbar_wait(&bar[warp], 0, &never, &err_s);
        t1 = clock64();
        cycles[blockIdx.x * 4 + warp] = ok ? t1 - t0 : ~0ull;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// kind::f16, integer-valued operands, M = 128, N = 32, K = 32 (two MMAs):
// every accumulator against the integer dot. pattern 0: pseudo-random codes,
// 1: the extremes (-8 x -127 everywhere, the largest sum), 2: mixed signs.
__global__ void __launch_bounds__(kThreads, 1) exact_kernel(int pattern, uint32_t seed,
                                                            unsigned int* mismatches,
                                                            float* sample) {
    constexpr int N = 32;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* As = smem;             // 128 rows x 64 bytes used (32 fp16)
    uint8_t* Bs = smem + 128 * 128;  // 32 rows
    __shared__ int a_int[128][32];
    __shared__ int b_int[N][32];
    __shared__ uint64_t bar;
    __shared__ uint32_t tmem_s;
    __shared__ uint32_t err_s;  // bounded waits record a timeout here
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) err_s = 0;
    for (int i = threadIdx.x; i < (128 + N) * 32; i += kThreads) {
        const int row = i / 32, k = i % 32;
        const uint32_t r = lcg(lcg(seed ^ (uint32_t)(i * 2654435761u)));
        int v;
        if (row < 128) {
            v = pattern == 1 ? -8 : pattern == 2 ? ((k & 1) ? 7 : -8) : (int)(r >> 28) - 8;
            a_int[row][k] = v;
        } else {
            v = pattern == 1 ? -127 : pattern == 2 ? ((row & 1) ? 127 : -127)
                                                   : (int)((r >> 16) % 255u) - 127;
            b_int[row - 128][k] = v;
        }
        const __half h = __float2half_rn((float)v);
        uint8_t* base = row < 128 ? As : Bs;
        const int rr = row < 128 ? row : row - 128;
        *reinterpret_cast<__half*>(base + sw128(rr, 2 * k)) = h;
    }
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_s, 32);
        tmem_relinquish();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_s;
    if (threadIdx.x == 0) {
        constexpr uint32_t idesc = idesc_f16_(128, N);
        for (int j = 0; j < 2; ++j)
            mma_f16_ss(tmem, smem_desc_k_sw128(smem_u32(As) + 32 * j),
                       smem_desc_k_sw128(smem_u32(Bs) + 32 * j), idesc, j > 0 ? 1u : 0u);
        mma_commit(&bar);
    }
    int never = 0;
    if (!mbar_wait(&bar, 0, &never, &err_s)) {
        if (threadIdx.x == 0) atomicAdd(mismatches, 1u << 30);
    } else {
        tc_fence_after();
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16), v);
        tmem_wait_ld();
        tmem_ld_pin(v);
        const int row = 32 * warp + lane;
        unsigned int bad = 0;
        for (int c = 0; c < N; ++c) {
            int dot = 0;
            for (int k = 0; k < 32; ++k) dot += a_int[row][k] * b_int[c][k];
            const float got = __uint_as_float(v[c]);
            if (got != (float)dot) ++bad;
            if (row == 0 && c < 4) sample[2 * c] = got, sample[2 * c + 1] = (float)dot;
        }
        if (bad) atomicAdd(mismatches, bad);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 32);
    }
}

// Wake-up latency: warp 1 waits on an mbarrier phase that warp 0 completes
// after a delay; both read the SM clock (same SM). mode 0: try_wait with a
// 1 ms suspend hint, 1: try_wait without a hint, 2: test_wait spin. Each of
// `reps` rounds records (wake clock - arrive clock); the median is returned.
__global__ void __launch_bounds__(64, 1) wake_kernel(int mode, int reps, int delay,
                                                     long long* lat) {
    __shared__ uint64_t bar;
    __shared__ long long t_arrive;
    __shared__ uint32_t err_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        err_s = 0;
    }
    __syncthreads();
    for (int i = 0; i < reps; ++i) {
        const uint32_t parity = i & 1;
        if (warp == 0 && lane == 0) {
            const long long t0 = clock64();
            while (clock64() - t0 < delay) {
            }
            t_arrive = clock64();
            mbar_arrive(&bar);
        } else if (warp == 1 && lane == 0) {
            const unsigned long long g0 = global_timer_ns();
            bool done = false;
            while (!done) {
                if (mode == 0) {
                    done = mbar_try_wait(&bar, parity);
                } else if (mode == 1) {
                    done = mbar_poll(&bar, parity);
                } else {
                    uint32_t ok;
                    asm volatile(
                        "{\n\t.reg .pred p;\n\t"
                        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                        "selp.u32 %0, 1, 0, p;\n\t}"
                        : "=r"(ok)
                        : "r"(smem_u32(&bar)), "r"(parity)
                        : "memory");
                    done = ok != 0;
                }
                if (global_timer_ns() - g0 > 100000000ull) break;  // 0.1 s bound
            }
            const long long t1 = clock64();
            __threadfence_block();
            lat[i] = done ? t1 : -1;
        }
        __syncthreads();
        if (warp == 1 && lane == 0 && lat[i] >= 0) lat[i] -= t_arrive;
        __syncthreads();
    }
}

// TMEM bandwidth: `warps` warps (a multiple of 4, each in its lane quadrant)
// repeat tcgen05.ld (mode 0) or tcgen05.st (mode 1) of 32 lanes x `cols`
// 32-bit columns, `batch` instructions per wait. Returns cycles per round of
// every warp in *cycles (median over CTAs).
template <int COLS>
__global__ void __launch_bounds__(512, 1) tmem_bw_kernel(int mode, int iters, int batch, int warps,
                                                         unsigned long long* cycles) {
    __shared__ uint32_t tmem_s;
    const int warp = threadIdx.x >> 5;
    if (warp == 0) {
        tmem_alloc(&tmem_s, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t base = tmem_s + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((warp >> 2) * 64 % 512);
    uint32_t acc = 0;
    const unsigned long long t0 = clock64();
    if (warp < warps) {
        for (int i = 0; i < iters; ++i) {
            if (mode == 0) {
                uint32_t v[COLS];
                for (int b = 0; b < batch; ++b) {
                    tmem_ld<COLS>(base + (uint32_t)((b * COLS) % 256), v);
                }
                tmem_wait_ld();
                tmem_ld_pin(v);
                acc += v[0];
            } else {
                for (int b = 0; b < batch; ++b) tmem_fill<COLS>(base + (uint32_t)((b * COLS) % 256), (uint32_t)i);
                tmem_wait_st();
            }
        }
    }
    __syncthreads();
    const unsigned long long t1 = clock64();
    if (threadIdx.x == 0) cycles[blockIdx.x] = t1 - t0 + (acc == 12345678u ? 1 : 0);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_s, 512);
    }
}

template <int KIND, int N, bool TS>
int launch_rate(int grid, int iters, int issuers, int rot, int gap, int waits, int mode,
                unsigned long long* d_cycles, cudaStream_t s) {
    // at least 120 KB of shared memory keeps one CTA per SM (each allocates
    // all 512 TMEM columns)
    const int smem = std::max(1024 + 128 * 128 + N * 128, 120 * 1024);
    auto k = rate_kernel<KIND, N, TS>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return -1;
    k<<<grid, kThreads, smem, s>>>(iters, issuers, rot, gap, waits, mode, d_cycles);
    return 0;
}

template <int KIND, bool TS>
int launch_rate_n(int n, int grid, int iters, int issuers, int rot, int gap, int waits, int mode,
                  unsigned long long* c, cudaStream_t s) {
    switch (n) {
        case 16: return launch_rate<KIND, 16, TS>(grid, iters, issuers, rot, gap, waits, mode, c, s);
        case 32: return launch_rate<KIND, 32, TS>(grid, iters, issuers, rot, gap, waits, mode, c, s);
        case 64: return launch_rate<KIND, 64, TS>(grid, iters, issuers, rot, gap, waits, mode, c, s);
        case 128: return launch_rate<KIND, 128, TS>(grid, iters, issuers, rot, gap, waits, mode, c, s);
        case 256: return launch_rate<KIND, 256, TS>(grid, iters, issuers, rot, gap, waits, mode, c, s);
        default: return -1;
    }
}

}  // namespace

extern "C" {

// kind: 0 int8, 1 fp16. Returns 0 and fills median cycles per MMA (over the
// issuers of all CTAs) and the grid's wall time in ms, or a negative code.
int mma_peak_rate(int kind, int n, int ts, int issuers, int rot, int gap, int waits, int mode,
                  int iters, int grid, double* cycles_per_mma, double* ms) {
    const int acc_cols = 32 + issuers * rot * n;
    if (issuers < 1 || issuers > 3 || rot < 1 || acc_cols > 512 || iters < 1 || grid < 1 ||
        gap < 0 || gap > 100000 || waits < 0 || waits > 64 || mode < 0 || mode > 31)
        return -2;
    unsigned long long* d = nullptr;
    if (cudaMalloc(&d, sizeof(unsigned long long) * 4 * grid) != cudaSuccess) return -3;
    cudaMemset(d, 0, sizeof(unsigned long long) * 4 * grid);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    auto run = [&]() -> int {
        if (kind == 0)
            return ts ? launch_rate_n<0, true>(n, grid, iters, issuers, rot, gap, waits, mode, d, 0)
                      : launch_rate_n<0, false>(n, grid, iters, issuers, rot, gap, waits, mode, d, 0);
        return ts ? launch_rate_n<1, true>(n, grid, iters, issuers, rot, gap, waits, mode, d, 0)
                  : launch_rate_n<1, false>(n, grid, iters, issuers, rot, gap, waits, mode, d, 0);
    };
    int rc = run();  // warm-up
    if (rc == 0) {
        cudaEventRecord(e0);
        rc = run();
        cudaEventRecord(e1);
    }
    cudaError_t err = cudaDeviceSynchronize();
    if (rc == 0 && err == cudaSuccess) {
        float f = 0.0f;
        cudaEventElapsedTime(&f, e0, e1);
        *ms = f;
        std::vector<unsigned long long> h(4 * (size_t)grid);
        cudaMemcpy(h.data(), d, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
        std::vector<double> per;
        for (int b = 0; b < grid; ++b)
            for (int w = 0; w < issuers; ++w) per.push_back((double)h[4 * b + w] / iters);
        std::sort(per.begin(), per.end());
        *cycles_per_mma = per[per.size() / 2];
    } else if (rc == 0) {
        rc = -4;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(d);
    return rc;
}

// Median wake-up latency (SM cycles) of a waiter on an mbarrier (see
// wake_kernel), or a negative code.
double mma_peak_wake(int mode, int reps, int delay) {
    long long* d = nullptr;
    if (reps < 1 || reps > 4096 || mode < 0 || mode > 2 || delay < 0 || delay > 1000000) return -2;
    if (cudaMalloc(&d, sizeof(long long) * reps) != cudaSuccess) return -3;
    wake_kernel<<<1, 64>>>(mode, reps, delay, d);
    double r = -4;
    if (cudaDeviceSynchronize() == cudaSuccess) {
        std::vector<long long> h(reps);
        cudaMemcpy(h.data(), d, sizeof(long long) * reps, cudaMemcpyDeviceToHost);
        std::sort(h.begin(), h.end());
        r = (double)h[reps / 2];
    }
    cudaFree(d);
    return r;
}

// TMEM bytes per SM cycle of tcgen05.ld (mode 0) / tcgen05.st (mode 1) by
// `warps` warps, 32 x cols per instruction, `batch` per wait; or < 0.
double mma_peak_tmem_bw(int mode, int cols, int batch, int warps, int iters, int grid) {
    if ((cols != 8 && cols != 16 && cols != 32) || batch < 1 || batch > 8 || warps < 4 ||
        warps > 16 || (warps & 3) || iters < 1 || grid < 1 || mode < 0 || mode > 1)
        return -2;
    unsigned long long* d = nullptr;
    if (cudaMalloc(&d, sizeof(unsigned long long) * grid) != cudaSuccess) return -3;
    const int smem = 120 * 1024;  // one CTA per SM (it allocates all 512 columns)
    auto go = [&]() {
        if (cols == 8) {
            cudaFuncSetAttribute(tmem_bw_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            tmem_bw_kernel<8><<<grid, 512, smem>>>(mode, iters, batch, warps, d);
        } else if (cols == 16) {
            cudaFuncSetAttribute(tmem_bw_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            tmem_bw_kernel<16><<<grid, 512, smem>>>(mode, iters, batch, warps, d);
        } else {
            cudaFuncSetAttribute(tmem_bw_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            tmem_bw_kernel<32><<<grid, 512, smem>>>(mode, iters, batch, warps, d);
        }
    };
    go();
    go();
    double r = -4;
    if (cudaDeviceSynchronize() == cudaSuccess) {
        std::vector<unsigned long long> h(grid);
        cudaMemcpy(h.data(), d, sizeof(unsigned long long) * grid, cudaMemcpyDeviceToHost);
        std::sort(h.begin(), h.end());
        const double cyc = (double)h[grid / 2];
        r = (double)warps * 32.0 * cols * 4.0 * batch * iters / cyc;
    }
    cudaFree(d);
    return r;
}

// Returns the number of fp32 accumulators that differ from the integer dot
// (0 = exact), or a negative code; sample[8] gets (got, want) of 4 values.
int mma_peak_exact(int pattern, unsigned int seed, float* sample) {
    unsigned int* d = nullptr;
    float* ds = nullptr;
    if (cudaMalloc(&d, sizeof(unsigned int)) != cudaSuccess) return -3;
    if (cudaMalloc(&ds, 8 * sizeof(float)) != cudaSuccess) {
        cudaFree(d);
        return -3;
    }
    cudaMemset(d, 0, sizeof(unsigned int));
    const int smem = 1024 + 128 * 128 + 32 * 128;
    cudaFuncSetAttribute(exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    exact_kernel<<<1, kThreads, smem>>>(pattern, seed, d, ds);
    int rc;
    if (cudaDeviceSynchronize() != cudaSuccess) {
        rc = -4;
    } else {
        unsigned int h = 0;
        cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost);
        cudaMemcpy(sample, ds, 8 * sizeof(float), cudaMemcpyDeviceToHost);
        rc = (int)h;
    }
    cudaFree(d);
    cudaFree(ds);
    return rc;
}

}  // extern "C"
