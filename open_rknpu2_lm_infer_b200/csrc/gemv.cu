// Small-batch (decode) path of group-32 int4 banks: grouped GEMVs on the CUDA
// cores, HBM-bound by design.
//
// At a few tokens per layer each routed expert row is used by one token, so
// the tensor-core GEMM's per-k-block TMEM round trip of the exact group path
// is pure latency. Here every CTA streams whole 18 KB weight stages (the
// bank's own packed layout: 128 rows x 256 codes + 128 x 8 fp16 group scales)
// with one bulk copy each, all stages in flight at once, and reduces them with
// dp4a: a group's int32 sum is exact (sum over its 32 codes of code * q_x),
// then f = fma((float)acc_g, s_g, f) over ascending groups and * s_x, the
// restatement's order — the same values as the exact tensor-core path.
//
//   gemv_gateup_kernel : grid (T*k assignments, I/64 tiles). One CTA = one
//     128-row gate|up tile (64 gate + 64 up channels) of one assignment ->
//     SwiGLU middle values; the last CTA of an assignment requantises its
//     middle row (A8, the MoE rule) for the down projection.
//   gemv_down_kernel   : grid (T*k assignments, H/128 tiles) -> expert rows
//     y; the last CTA of a (token, tile) combines the token's kept ranks in
//     rank order (fma), adds the residual and writes the output tile.
//
// The "last CTA" hand-offs are counter increments after a __threadfence: no
// CTA ever waits for another, so nothing can hang. Reference semantics: the
// expert FFN of src/npu/moe.rs:324-333 (native), the SwiGLU of
// native/cpu_kernels/swiglu.cpp:23-25, the combine of
// src/model/experts/paged.rs:495-506 and the residual of
// src/model/qwen35/decoder.rs:215-217.
#include <float.h>

#include "kernels.cuh"

namespace moe {

namespace {

constexpr int kGvThreads = 128;
constexpr int kGvStage = 128 * 128 + 128 * 16;  // bytes of one packed group-32 stage
constexpr int kGvStageW = 128 * 128;

// dp4a with unsigned bytes in a (the offset-binary nibbles 0..15) and signed
// bytes in b (the int8 activation codes).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Activation row -> shared memory in the packed word order: a weight word
// holds (low nibbles) codes j = 0,4,1,5 and (high nibbles) j = 2,6,3,7 of its
// 8 k, so the activations of each 8-k word are stored as x0 x4 x1 x5 | x2 x6
// x3 x7. Also the per-group sums of the codes (for the offset-binary
// correction: sum((b - 8) * x) = sum(b * x) - 8 * sum(x)).
__device__ __forceinline__ void stage_activation(const int8_t* __restrict__ q, int K,
                                                 uint32_t* xp, int* gsum) {
    for (int wd = threadIdx.x; wd < K / 8; wd += blockDim.x) {
        const uint2 v = reinterpret_cast<const uint2*>(q)[wd];
        const uint32_t lo = v.x, hi = v.y;  // bytes x0..x3, x4..x7
        // A = x0 x4 x1 x5, B = x2 x6 x3 x7
        xp[2 * wd] = __byte_perm(lo, hi, 0x5140);
        xp[2 * wd + 1] = __byte_perm(lo, hi, 0x7362);
    }
    for (int g = threadIdx.x; g < K / 32; g += blockDim.x) {
        const int8_t* p = q + g * 32;
        int s = 0;
        for (int i = 0; i < 32; ++i) s += p[i];
        gsum[g] = s;
    }
}

// One step: 4 rows x 8 groups of one stage, lane = (row rs = lane >> 3,
// logical group gl = lane & 7). Returns this lane's exact group sum.
__device__ __forceinline__ int group_dot(const uint8_t* stg, int lr, int gl, const uint32_t (&A)[4],
                                         const uint32_t (&B)[4], int gs) {
    const uint4 wv = *reinterpret_cast<const uint4*>(stg + lr * 128 + ((gl ^ (lr & 7)) * 16));
    const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
    int acc = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc = dp4a_us(wd[i] & 0x0F0F0F0Fu, A[i], acc);
        acc = dp4a_us((wd[i] >> 4) & 0x0F0F0F0Fu, B[i], acc);
    }
    return acc - 8 * gs;
}

// The row leader (gl == 0) folds the 8 group sums of its row in ascending
// group order: f = fma((float)acc_g, s_g, f).
__device__ __forceinline__ float fold_groups(float f, int acc, const uint8_t* stg, int lr, int lane) {
    const __half* sc = reinterpret_cast<const __half*>(stg + kGvStageW + lr * 16);
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const int a = __shfl_sync(0xffffffffu, acc, (lane & ~7) | g);
        f = __fmaf_rn((float)a, __half2float(sc[g]), f);
    }
    return f;
}

__device__ __forceinline__ void load_stage_regs(const uint32_t* xp, const int* gsum, int s, int gl,
                                                uint32_t (&A)[4], uint32_t (&B)[4], int& gs) {
    const uint4* p = reinterpret_cast<const uint4*>(xp + (s * 8 + gl) * 8);
    const uint4 u0 = p[0], u1 = p[1];
    A[0] = u0.x; B[0] = u0.y; A[1] = u0.z; B[1] = u0.w;
    A[2] = u1.x; B[2] = u1.y; A[3] = u1.z; B[3] = u1.w;
    gs = gsum[s * 8 + gl];
}

// Issue every stage of one packed tile: one bulk copy and one barrier each.
__device__ __forceinline__ void issue_stages(uint8_t* st, uint64_t* bars, const uint8_t* tile,
                                             size_t stage_stride, int S) {
    for (int s = 0; s < S; ++s) {
        mbar_arrive_expect_tx(&bars[s], kGvStage);
        bulk_g2s(st + (size_t)s * kGvStage, tile + (size_t)s * stage_stride, kGvStage, &bars[s]);
    }
}

__device__ __forceinline__ bool last_arrival(int* counter, int expected) {
    __shared__ int is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(counter, 1);
        is_last = (prev == expected - 1);
        if (is_last) *counter = 0;  // ready for the next call
    }
    __syncthreads();
    if (is_last) __threadfence();
    return is_last;
}

}  // namespace

__global__ void __launch_bounds__(kGvThreads) gemv_gateup_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int S = a.gu_stages, Kp = S * 256;
    uint8_t* st = sm;
    uint32_t* xp = reinterpret_cast<uint32_t*>(sm + (size_t)S * kGvStage);
    int* gsum = reinterpret_cast<int*>(xp + Kp / 4);
    uint64_t* bars = reinterpret_cast<uint64_t*>(gsum + Kp / 32);
    __shared__ int abort_flag;
    const int asg = blockIdx.x, rt = blockIdx.y, t = asg / a.k;
    const float w = a.routes[asg];
    const int e = a.ids[asg];
    if (!(w >= 0.0f) && rt == 0 && threadIdx.x == 0) atomicOr(a.err, kErrBadRoute);  // < 0 or NaN
    if (!(w > 0.0f)) return;  // skipped route: its middle row is never read
    if (e < 0 || e >= a.E) {
        if (threadIdx.x == 0) atomicOr(a.err, kErrBadExpert);
        return;
    }
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0)
        issue_stages(st, bars, a.gu_w + (size_t)e * a.gu_expert_stride + (size_t)rt * a.gu_tile_stride,
                     a.gu_stage_stride, S);
    stage_activation(a.q_x + (size_t)t * a.ld_qx, Kp, xp, gsum);
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gl = lane & 7, rs = lane >> 3;
    // warp w: gate channels 16w + 4j + rs (rows), up rows 64 + the same
    float f[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = 0.0f;
    bool ok = true;
    for (int s = 0; s < S && ok; ++s) {
        // every lane waits (acquire), the warp decides together (shuffles follow)
        ok = __all_sync(0xffffffffu, mbar_wait(&bars[s], 0, &abort_flag, a.err));
        if (!ok) break;
        const uint8_t* stg = st + (size_t)s * kGvStage;
        uint32_t A[4], B[4];
        int gs;
        load_stage_regs(xp, gsum, s, gl, A, B, gs);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int lr = (j < 4 ? 0 : 64) + 16 * warp + 4 * (j & 3) + rs;
            const int acc = group_dot(stg, lr, gl, A, B, gs);
            f[j] = fold_groups(f[j], acc, stg, lr, lane);
        }
    }
    // a stalled copy (flagged above) still arrives, so the counters stay consistent
    if (ok && gl == 0) {
        const float sx = a.s_x[t];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = rt * 64 + 16 * warp + 4 * j + rs;
            if (c < a.I) {
                const float g = __fmul_rn(f[j], sx), u = __fmul_rn(f[4 + j], sx);
                const float d = __fadd_rn(1.0f, expf(-g));
                a.middle[(size_t)asg * a.I + c] = __fmul_rn(__fdiv_rn(g, d), u);
            }
        }
    }
    if (!last_arrival(&a.counters[asg], gridDim.y)) return;
    // requantise the assignment's middle row (MoE A8: s = max|x| / 127, q = rne(x / s))
    __shared__ float red[kGvThreads / 32];
    const float* mrow = a.middle + (size_t)asg * a.I;
    float m = 0.0f;
    for (int c = threadIdx.x; c < a.I; c += blockDim.x) m = fmaxf(m, fabsf(__ldcg(mrow + c)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int i = 1; i < kGvThreads / 32; ++i) m = fmaxf(m, red[i]);
    const float sc = m == 0.0f ? 1.0f : __fdiv_rn(m, 127.0f);
    if (threadIdx.x == 0) a.s_m[asg] = sc;
    int8_t* qrow = a.q_m + (size_t)asg * a.ld_qm;
    for (int c = threadIdx.x; c < a.ld_qm; c += blockDim.x) {
        int q = 0;
        if (c < a.I) {
            q = __float2int_rn(__fdiv_rn(__ldcg(mrow + c), sc));
            q = q > 127 ? 127 : (q < -127 ? -127 : q);
        }
        qrow[c] = (int8_t)q;
    }
}

__global__ void __launch_bounds__(kGvThreads) gemv_down_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int S = a.dn_stages, Kp = S * 256;
    uint8_t* st = sm;
    uint32_t* xp = reinterpret_cast<uint32_t*>(sm + (size_t)S * kGvStage);
    int* gsum = reinterpret_cast<int*>(xp + Kp / 4);
    uint64_t* bars = reinterpret_cast<uint64_t*>(gsum + Kp / 32);
    __shared__ int abort_flag;
    const int asg = blockIdx.x, dt = blockIdx.y, t = asg / a.k;
    const float w = a.routes[asg];
    const int e = a.ids[asg];
    const bool valid = e >= 0 && e < a.E;
    const bool kept = w > 0.0f && valid;
    if (w > 0.0f && !valid && threadIdx.x == 0) atomicOr(a.err, kErrBadExpert);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gl = lane & 7, rs = lane >> 3;
    if (kept) {
        if (threadIdx.x == 0) {
            abort_flag = 0;
            for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
            fence_barrier_init();
        }
        __syncthreads();
        if (threadIdx.x == 0)
            issue_stages(st, bars,
                         a.dn_w + (size_t)e * a.dn_expert_stride + (size_t)dt * a.dn_tile_stride,
                         a.dn_stage_stride, S);
        stage_activation(a.q_m + (size_t)asg * a.ld_qm, Kp, xp, gsum);
        __syncthreads();
        // warp w: output rows 32w + 4j + rs of the tile
        float f[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = 0.0f;
        bool ok = true;
        for (int s = 0; s < S && ok; ++s) {
            ok = __all_sync(0xffffffffu, mbar_wait(&bars[s], 0, &abort_flag, a.err));
            if (!ok) break;
            const uint8_t* stg = st + (size_t)s * kGvStage;
            uint32_t A[4], B[4];
            int gs;
            load_stage_regs(xp, gsum, s, gl, A, B, gs);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int lr = 32 * warp + 4 * j + rs;
                const int acc = group_dot(stg, lr, gl, A, B, gs);
                f[j] = fold_groups(f[j], acc, stg, lr, lane);
            }
        }
        if (ok && gl == 0) {
            const float sm_ = a.s_m[asg];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = dt * 128 + 32 * warp + 4 * j + rs;
                if (c < a.H) a.y[(size_t)asg * a.H + c] = __fmul_rn(f[j], sm_);
            }
        }
    }
    if (!last_arrival(&a.counters[a.dn_counter_base + t * gridDim.y + dt], a.k)) return;
    // combine the token's kept ranks in rank order, then the residual
    for (int c = dt * 128 + threadIdx.x; c < min(a.H, dt * 128 + 128); c += blockDim.x) {
        float acc = 0.0f;
        for (int r = 0; r < a.k; ++r) {
            const int as = t * a.k + r;
            const float wr = a.routes[as];
            const int er = a.ids[as];
            if (!(wr > 0.0f) || er < 0 || er >= a.E) continue;
            acc = __fmaf_rn(__ldcg(a.y + (size_t)as * a.H + c), wr, acc);
        }
        if (a.residual) acc = __fadd_rn(a.residual[(size_t)t * a.H + c], acc);
        a.out[(size_t)t * a.H + c] = acc;
    }
}

size_t gemv_smem_bytes(int S) {
    const size_t Kp = (size_t)S * 256;
    return (size_t)S * kGvStage + Kp + (Kp / 32) * 4 + (size_t)S * 8;
}

int launch_gemv(const GemvArgs& a, int part, cudaStream_t s) {
    const int n = a.T * a.k;
    if (part == 0) {
        const size_t smg = gemv_smem_bytes(a.gu_stages);
        if (smg > kGemvMaxSmem) return -1;
        cudaFuncSetAttribute(gemv_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smg);
        gemv_gateup_kernel<<<dim3(n, (a.I + 63) / 64), kGvThreads, smg, s>>>(a);
    } else {
        const size_t smd = gemv_smem_bytes(a.dn_stages);
        if (smd > kGemvMaxSmem) return -1;
        cudaFuncSetAttribute(gemv_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smd);
        gemv_down_kernel<<<dim3(n, (a.H + 127) / 128), kGvThreads, smd, s>>>(a);
    }
    return 0;
}

}  // namespace moe
