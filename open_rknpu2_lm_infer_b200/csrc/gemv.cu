// Small-batch (decode) path of group-32 int4 banks: grouped GEMVs on the CUDA
// cores, HBM-bound by design.
//
// At a few tokens per layer each routed expert row is used by one token, so
// the tensor-core GEMM's per-k-block TMEM round trip of the exact group path
// is pure latency. Here every CTA streams one 128-row tile of one assignment
// as whole 18 KB stages (the bank's own packed layout: 128 rows x 256 codes +
// 128 x 8 fp16 group scales), one bulk copy each, all stages in flight at
// once. Sixteen warps split the (stage, 4-row) items and write every group's
// exact int32 sum (sum over its 32 codes of code * activation code) to shared
// memory; then one thread per row folds them in ascending group order,
// f = fma((float)acc_g, s_g, f), and scales by the activation scale: the
// restatement's order, the same values as the exact tensor-core path.
//
//   gemv_gateup_kernel : grid (T*k assignments, I/64 tiles). Quantises its
//     token's activation row itself (the MoE A8 rule), computes the 64 gate and
//     64 up channels of its tile -> SwiGLU middle values; the last CTA of an
//     assignment requantises the middle row (A8) for the down projection.
//   gemv_down_kernel   : grid (T*k assignments, H/128 tiles) -> expert rows
//     y; the last CTA of a (token, tile) combines the token's kept ranks in
//     rank order (fma), adds the residual and writes the output tile.
//
// The "last CTA" hand-offs are counter increments after a __threadfence: no
// CTA ever waits for another, so nothing can hang. Reference semantics: the
// expert FFN of src/npu/moe.rs:324-333 (native), the activation quantiser of
// llm_generated_docs/MOE_CPU_FUSION_20261023.md:13, the SwiGLU of
// native/cpu_kernels/swiglu.cpp:23-25, the combine of
// src/model/experts/paged.rs:495-506 and the residual of
// src/model/qwen35/decoder.rs:215-217.
#include <float.h>

#include <mutex>

#include "kernels.cuh"
#include "route.cuh"

namespace moe {

namespace {

constexpr int kGvThreads = 512;
constexpr int kGvWarps = kGvThreads / 32;
constexpr int kGvStage = 128 * 128 + 128 * 16;  // bytes of one packed group-32 stage
constexpr int kGvStageW = 128 * 128;

// dp4a with unsigned bytes in a (the offset-binary nibbles 0..15) and signed
// bytes in b (the int8 activation codes).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ int byte_sum(uint32_t w) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(w), "r"(0x01010101), "r"(0));
    return d;
}

// Shared-memory layout of both kernels (S stages, Kp = 256 S activation codes,
// G = 8 S groups per row).
struct GvSmem {
    uint8_t* st;     // [S][kGvStage]
    uint32_t* xp;    // [Kp / 4] activation codes in the packed word order
    int* gsum;       // [G] per-group sums of the activation codes
    int* acc;        // [128][G + 8] exact group sums
    float* val;      // [128] dequantised row values
    uint64_t* bars;  // [S]
    int G, ld;
};

__device__ __forceinline__ GvSmem gv_smem(uint8_t* sm, int S) {
    GvSmem m;
    const int Kp = S * 256;
    m.G = S * 8;
    m.ld = m.G + 8;  // rows 8 banks apart: the 4 rows of a step store conflict-free
    m.st = sm;
    m.xp = reinterpret_cast<uint32_t*>(sm + (size_t)S * kGvStage);
    m.gsum = reinterpret_cast<int*>(m.xp + Kp / 4);
    m.acc = m.gsum + m.G;
    m.val = reinterpret_cast<float*>(m.acc + 128 * m.ld);
    m.bars = reinterpret_cast<uint64_t*>(m.val + 128);
    return m;
}

// The 8 codes of one 8-k word -> the packed word order: a weight word holds
// (low nibbles) codes j = 0,4,1,5 and (high nibbles) j = 2,6,3,7, so the
// activations are stored as x0 x4 x1 x5 | x2 x6 x3 x7. The group sums feed
// the offset-binary correction sum((b - 8) x) = sum(b x) - 8 sum(x). Called
// by whole warps with wd = thread index (4 consecutive words = one group).
__device__ __forceinline__ void put_word(const GvSmem& m, int wd, uint32_t lo, uint32_t hi) {
    m.xp[2 * wd] = __byte_perm(lo, hi, 0x5140);
    m.xp[2 * wd + 1] = __byte_perm(lo, hi, 0x7362);
    int s = byte_sum(lo) + byte_sum(hi);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if ((wd & 3) == 0) m.gsum[wd >> 2] = s;
}

// Every stage of one packed tile: one bulk copy and one barrier each.
__device__ __forceinline__ void issue_stages(const GvSmem& m, const uint8_t* tile,
                                             size_t stage_stride, int S) {
    for (int s = 0; s < S; ++s) {
        mbar_arrive_expect_tx(&m.bars[s], kGvStage);
        bulk_g2s(m.st + (size_t)s * kGvStage, tile + (size_t)s * stage_stride, kGvStage,
                 &m.bars[s]);
    }
}

// Phase A: items (stage s, rows 4q..4q+3), lane = (row rs = lane >> 3, logical
// group gl = lane & 7); every group's exact sum goes to acc[row][8 s + gl].
// A warp's items run in stage order and it waits (acquire, the whole warp
// deciding together) for a stage when it reaches the stage's first item, so
// the sums of the stages that landed overlap the copies of the rest. Returns
// false when a stage never arrived (flagged). Bit s of `phases` is the phase
// parity stage s's barrier is in (a CTA that reuses its barriers passes the
// parities; one use per barrier: 0).
__device__ __forceinline__ bool group_sums_p(const GvSmem& m, int S, uint32_t phases,
                                             int* abort_flag, uint32_t* err) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gl = lane & 7, rs = lane >> 3;
    int landed = -1;  // stages 0..landed have been waited for
#pragma unroll 4
    for (int it = warp; it < S * 32; it += kGvWarps) {
        const int s = it >> 5, lr = (it & 31) * 4 + rs;
        if (s > landed) {  // warp-uniform
            bool arrived = true;
            for (int w = landed + 1; w <= s; ++w)
                arrived = mbar_wait(&m.bars[w], (phases >> w) & 1u, abort_flag, err) && arrived;
            if (!__all_sync(0xffffffffu, arrived)) return false;
            landed = s;
        }
        const uint4* xq = reinterpret_cast<const uint4*>(m.xp + (s * 8 + gl) * 8);
        const uint4 u0 = xq[0], u1 = xq[1];
        const uint32_t A[4] = {u0.x, u0.z, u1.x, u1.z}, B[4] = {u0.y, u0.w, u1.y, u1.w};
        const uint8_t* stg = m.st + (size_t)s * kGvStage;
        const uint4 wv = *reinterpret_cast<const uint4*>(stg + lr * 128 + ((gl ^ (lr & 7)) * 16));
        const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
        int acc = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            acc = dp4a_us(wd[i] & 0x0F0F0F0Fu, A[i], acc);
            acc = dp4a_us((wd[i] >> 4) & 0x0F0F0F0Fu, B[i], acc);
        }
        m.acc[lr * m.ld + s * 8 + gl] = acc - 8 * m.gsum[s * 8 + gl];
    }
    return true;
}

__device__ __forceinline__ bool group_sums(const GvSmem& m, int S, int* abort_flag,
                                           uint32_t* err) {
    return group_sums_p(m, S, 0u, abort_flag, err);
}

// Phase B (one thread per row): f = fma((float)acc_g, s_g, f) over ascending
// groups.
__device__ __forceinline__ float fold_row(const GvSmem& m, int S, int r) {
    float f = 0.0f;
    for (int s = 0; s < S; ++s) {
        const uint4 hs =
            *reinterpret_cast<const uint4*>(m.st + (size_t)s * kGvStage + kGvStageW + r * 16);
        const int4 a0 = *reinterpret_cast<const int4*>(m.acc + r * m.ld + s * 8);
        const int4 a1 = *reinterpret_cast<const int4*>(m.acc + r * m.ld + s * 8 + 4);
        const __half2* h = reinterpret_cast<const __half2*>(&hs);
        const int av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const __half hg = (g & 1) ? __high2half(h[g >> 1]) : __low2half(h[g >> 1]);
            f = __fmaf_rn((float)av[g], __half2float(hg), f);
        }
    }
    return f;
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

// Block-wide max of non-negative values.
__device__ __forceinline__ float gv_block_max(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = red[0];
    for (int i = 1; i < kGvWarps; ++i) r = fmaxf(r, red[i]);
    __syncthreads();
    return r;
}

__device__ __forceinline__ int quant_moe(float x, float s) {
    const int q = __float2int_rn(__fdiv_rn(x, s));
    return q > 127 ? 127 : (q < -127 ? -127 : q);
}

}  // namespace

__global__ void __launch_bounds__(kGvThreads) gemv_gateup_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ int abort_flag;
    __shared__ float red[kGvWarps];
    const int S = a.gu_stages, Kp = S * 256;
    const GvSmem m = gv_smem(sm, S);
    const int asg = blockIdx.x, rt = blockIdx.y, t = asg / a.k;
    // prologue, independent of the routing: barriers and the activation codes
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; ++s) mbar_init(&m.bars[s], 1);
        fence_barrier_init();
    }
    // the token's activation row -> MoE A8 codes (s = max|x| / 127, 0 -> 1,
    // q = rne(x / s)), computed by every CTA of the token from the f32 row
    const float* xr = a.x + (size_t)t * a.H;
    float mx = 0.0f;
    for (int i = threadIdx.x; i < a.H; i += kGvThreads) mx = fmaxf(mx, fabsf(xr[i]));
    mx = gv_block_max(mx, red);
    const float sx = mx == 0.0f ? 1.0f : __fdiv_rn(mx, 127.0f);
    if (!isfinite(sx) && rt == 0 && threadIdx.x == 0) atomicOr(a.err, kErrNonFinite);
    // Kp / 8 is a multiple of 32: whole warps take words or stop together
    for (int wd = threadIdx.x; wd < Kp / 8; wd += kGvThreads) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = wd * 8 + j;
            const uint32_t q = k < a.H ? (uint32_t)(quant_moe(xr[k], sx) & 0xFF) : 0u;
            if (j < 4) lo |= q << (8 * j);
            else hi |= q << (8 * (j - 4));
        }
        put_word(m, wd, lo, hi);
    }
    // the routing comes from the preceding grid (the router, when this kernel
    // is its programmatic dependent); once it is visible, the down kernel may
    // launch and read it too
    pdl_wait();
    pdl_trigger();
    const float w = a.routes[asg];
    const int e = a.ids[asg];
    if (!(w >= 0.0f) && rt == 0 && threadIdx.x == 0) atomicOr(a.err, kErrBadRoute);  // < 0 or NaN
    if (!(w > 0.0f)) return;  // skipped route: its middle row is never read
    if (e < 0 || e >= a.E) {
        if (threadIdx.x == 0) atomicOr(a.err, kErrBadExpert);
        return;
    }
    __syncthreads();  // barriers initialised, activation codes staged
    if (threadIdx.x == 0)
        issue_stages(m, a.gu_w + (size_t)e * a.gu_expert_stride + (size_t)rt * a.gu_tile_stride,
                     a.gu_stage_stride, S);
    const bool ok = group_sums(m, S, &abort_flag, a.err);
    __syncthreads();
    if (threadIdx.x < 128) m.val[threadIdx.x] = __fmul_rn(fold_row(m, S, threadIdx.x), sx);
    __syncthreads();
    // a stalled copy (flagged above) still arrives, so the counters stay consistent
    if (ok && threadIdx.x < 64) {
        const int c = rt * 64 + threadIdx.x;
        if (c < a.I) {
            const float g = m.val[threadIdx.x], u = m.val[64 + threadIdx.x];
            const float d = __fadd_rn(1.0f, expf(-g));
            a.middle[(size_t)asg * a.I + c] = __fmul_rn(__fdiv_rn(g, d), u);
        }
    }
    if (!last_arrival(&a.counters[asg], gridDim.y)) return;
    // requantise the assignment's middle row (MoE A8)
    const float* mrow = a.middle + (size_t)asg * a.I;
    float mm = 0.0f;
    for (int c = threadIdx.x; c < a.I; c += kGvThreads) mm = fmaxf(mm, fabsf(__ldcg(mrow + c)));
    mm = gv_block_max(mm, red);
    const float sc = mm == 0.0f ? 1.0f : __fdiv_rn(mm, 127.0f);
    if (threadIdx.x == 0) a.s_m[asg] = sc;
    int8_t* qrow = a.q_m + (size_t)asg * a.ld_qm;
    for (int c = threadIdx.x; c < a.ld_qm; c += kGvThreads)
        qrow[c] = (int8_t)(c < a.I ? quant_moe(__ldcg(mrow + c), sc) : 0);
}

__global__ void __launch_bounds__(kGvThreads) gemv_down_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ int abort_flag;
    const int S = a.dn_stages, Kp = S * 256;
    const GvSmem m = gv_smem(sm, S);
    const int asg = blockIdx.x, dt = blockIdx.y, t = asg / a.k;
    const float w = a.routes[asg];
    const int e = a.ids[asg];
    const bool valid = e >= 0 && e < a.E;
    const bool kept = w > 0.0f && valid;
    if (w > 0.0f && !valid && threadIdx.x == 0) atomicOr(a.err, kErrBadExpert);
    // the routing was visible before the gate/up grid let this grid launch, so
    // the weights stream in while the gate/up kernel still runs; its outputs
    // (middle codes and scales) are read only after pdl_wait
    if (kept && threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; ++s) mbar_init(&m.bars[s], 1);
        fence_barrier_init();
        issue_stages(m, a.dn_w + (size_t)e * a.dn_expert_stride + (size_t)dt * a.dn_tile_stride,
                     a.dn_stage_stride, S);
    }
    pdl_wait();
    if (kept) {
        __syncthreads();
        const uint2* qr = reinterpret_cast<const uint2*>(a.q_m + (size_t)asg * a.ld_qm);
        for (int wd = threadIdx.x; wd < Kp / 8; wd += kGvThreads) {
            const uint2 v = __ldcg(qr + wd);
            put_word(m, wd, v.x, v.y);
        }
        __syncthreads();
        const bool ok = group_sums(m, S, &abort_flag, a.err);
        __syncthreads();
        if (ok && threadIdx.x < 128) {
            const int c = dt * 128 + threadIdx.x;
            const float f = fold_row(m, S, threadIdx.x);
            if (c < a.H) a.y[(size_t)asg * a.H + c] = __fmul_rn(f, a.s_m[asg]);
        }
    }
    if (!last_arrival(&a.counters[a.dn_counter_base + t * gridDim.y + dt], a.k)) return;
    // combine the token's kept ranks in rank order, then the shared expert's
    // row (scaled by the sigmoid of its gate logit, if gated), then the
    // residual: combine_kernel's order and roundings
    float gs = 1.0f;
    if (a.shared && a.gate)
        gs = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f32(-a.gate[(size_t)t * a.gate_ld])));
    for (int c = dt * 128 + threadIdx.x; c < min(a.H, dt * 128 + 128); c += kGvThreads) {
        float acc = 0.0f;
        for (int r = 0; r < a.k; ++r) {
            const int as = t * a.k + r;
            const float wr = a.routes[as];
            const int er = a.ids[as];
            if (!(wr > 0.0f) || er < 0 || er >= a.E) continue;
            acc = __fmaf_rn(__ldcg(a.y + (size_t)as * a.H + c), wr, acc);
        }
        if (a.shared) {
            float sv = __ldcg(a.shared + (size_t)t * a.H + c);
            if (a.gate) sv = __fmul_rn(gs, sv);
            acc = __fadd_rn(acc, sv);
        }
        if (a.residual) acc = __fadd_rn(a.residual[(size_t)t * a.H + c], acc);
        a.out[(size_t)t * a.H + c] = acc;
    }
}

size_t gemv_smem_bytes(int S) {
    const size_t Kp = (size_t)S * 256, G = (size_t)S * 8;
    return (size_t)S * kGvStage + Kp + G * 4 + 128 * (G + 8) * 4 + 128 * 4 + (size_t)S * 8;
}

// Both kernels launch as programmatic dependents of the kernel before them
// (their prologues overlap its tail); each waits (pdl_wait) before reading
// what that kernel wrote.
int launch_gemv(const GemvArgs& a, int part, cudaStream_t s) {
    const int n = a.T * a.k;
    const size_t smem = gemv_smem_bytes(part == 0 ? a.gu_stages : a.dn_stages);
    if (smem > kGemvMaxSmem) return -1;
    void (*kern)(const GemvArgs) = part == 0 ? gemv_gateup_kernel : gemv_down_kernel;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = part == 0 ? dim3(n, (a.I + 63) / 64) : dim3(n, (a.H + 127) / 128);
    cfg.blockDim = dim3(kGvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? 0 : -1;
}

// ===================================================================== fused
// The small-batch layer as one cooperative launch, one CTA per SM. Phases:
//   R  router logits, item = (token, weight row) spread over all CTAs (the
//      CTA's rows and the token rows staged in shared memory, the NEON16 /
//      TF32 dot of the decode router, on warps 0-1), and at the same time the
//      tokens' activation codes (MoE A8, warps 2-15).
//   -- grid barrier --
//   T  every CTA routes every token itself (the softmax top-k by the whole
//      block, the grouped rule by one warp per token) from the logits; CTA 0
//      writes ids and weights out.
//   G  gate/up items = (assignment, 64-channel tile) as gemv_gateup_kernel,
//      then SwiGLU -> middle values and each middle
//      row's max |value| (atomic max of the float bits); each item then
//      counts itself done for its assignment (release). Then the CTA's first
//      down item's weights are requested, so they stream in while it waits.
//   D  down items = (assignment, 128-row tile) as gemv_down_kernel, each
//      waiting (acquire, bounded) only for its own assignment's gate/up items
//      before requantising the middle row itself; the last item of a (token,
//      tile) combines the kept ranks in rank order and adds the residual.
// Every value is computed by the same functions in the same order as the
// three-kernel path, so results are bit-identical to it.
namespace {

__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier (every CTA is resident: cooperative launch) over
// kGridBarLanes counters 128 bytes apart that only grow: CTA b arrives on
// counter b % kGridBarLanes (n_j CTAs share counter j), so the atomics of one
// barrier spread over eight lines instead of queueing on one; between barriers
// counter j rests on a multiple of n_j (every launch has the same grid), so an
// arrival's count before it tells the barrier's number m, and the barrier
// completes when every counter j reaches (m + 1) n_j (lanes 0..7 of warp 0
// poll one counter each). Waits at most kWaitLimitNs, then kErrWaitTimeout
// and false (the caller gives up; the host rearms the counters).
constexpr int kGridBarLanes = 8, kGridBarStride = 16;  // u64 counters, 128 bytes apart

__device__ bool grid_sync(unsigned long long* bar, uint32_t* err) {
    __shared__ int ok_s;
    __syncthreads();
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x, nb = gridDim.x, j0 = blockIdx.x % kGridBarLanes;
        unsigned long long m = 0;
        if (lane == 0) {
            __threadfence();
            const unsigned long long nj = (nb - j0 + kGridBarLanes - 1) / kGridBarLanes;
            m = atomicAdd(bar + j0 * kGridBarStride, 1ull) / nj;
        }
        m = __shfl_sync(0xffffffffu, m, 0);
        int ok = 1;
        if (lane < kGridBarLanes) {
            const unsigned long long nl = (nb - lane + kGridBarLanes - 1) / kGridBarLanes;
            const unsigned long long target = (m + 1) * nl;
            const uint64_t start = global_timer_ns();
            while (ld_acquire_gpu(bar + lane * kGridBarStride) < target) {
                if (global_timer_ns() - start > kWaitLimitNs) {
                    atomicOr(err, kErrWaitTimeout);
                    ok = 0;
                    break;
                }
            }
        }
        ok = __all_sync(0xffffffffu, ok);
        if (lane == 0) {
            __threadfence();
            ok_s = ok;
        }
    }
    __syncthreads();
    return ok_s != 0;
}

struct DecodeSmem {
    uint8_t* st;     // [Smax][kGvStage] stages (phase R: router and token rows)
    int* acc;        // [128][Gmax + 8]
    float* val;      // [128]
    uint64_t* bars;  // [Smax rounded up to even]
    uint32_t* txp;   // [T][Kg / 4] token activation codes, packed word order
    int* tgs;        // [T][Gg] their group sums
    uint32_t* dxp;   // [Kd / 4] middle codes of the current down item
    int* dgs;        // [Gd]
    float* sx;       // [T] token activation scales
    int* rid;        // [T*k] routed expert ids
    float* rw;       // [T*k] routing weights
    float* selv;     // [32] one token's selected logits, in rank order
    uint32_t* keys;  // [E] total-order keys of one token's logits
};

__device__ __forceinline__ DecodeSmem decode_smem(uint8_t* sm, int Sg, int Sd, int T, int k) {
    const int Smax = Sg > Sd ? Sg : Sd, Sb = (Smax + 1) & ~1;
    DecodeSmem d;
    d.st = sm;
    d.acc = reinterpret_cast<int*>(sm + (size_t)Smax * kGvStage);
    d.val = reinterpret_cast<float*>(d.acc + 128 * (Smax * 8 + 8));
    d.bars = reinterpret_cast<uint64_t*>(d.val + 128);
    d.txp = reinterpret_cast<uint32_t*>(d.bars + Sb);
    d.tgs = reinterpret_cast<int*>(d.txp + T * Sg * 64);
    d.dxp = reinterpret_cast<uint32_t*>(d.tgs + T * Sg * 8);
    d.dgs = reinterpret_cast<int*>(d.dxp + Sd * 64);
    d.sx = reinterpret_cast<float*>(d.dgs + Sd * 8);
    d.rid = reinterpret_cast<int*>(d.sx + T);
    d.rw = reinterpret_cast<float*>(d.rid + T * k);
    d.selv = d.rw + T * k;
    d.keys = reinterpret_cast<uint32_t*>(d.selv + 32);
    return d;
}

size_t decode_smem_bytes(int Sg, int Sd, int T, int k, int E) {
    const int Smax = Sg > Sd ? Sg : Sd, Sb = (Smax + 1) & ~1;
    return (size_t)Smax * kGvStage + 128 * (size_t)(Smax * 8 + 8) * 4 + 128 * 4 + (size_t)Sb * 8 +
           (size_t)T * Sg * 64 * 4 + (size_t)T * Sg * 8 * 4 + (size_t)Sd * 64 * 4 +
           (size_t)Sd * 8 * 4 + (size_t)T * 4 + (size_t)T * k * 8 + 32 * 4 + (size_t)E * 4;
}

__device__ __forceinline__ GvSmem gv_view(const DecodeSmem& d, uint32_t* xp, int* gsum, int S) {
    GvSmem m;
    m.st = d.st;
    m.xp = xp;
    m.gsum = gsum;
    m.acc = d.acc;
    m.val = d.val;
    m.bars = d.bars;
    m.G = S * 8;
    m.ld = m.G + 8;
    return m;
}

__global__ void __launch_bounds__(kGvThreads, 1) decode_layer_kernel(const DecodeArgs dl) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ int abort_flag;
    __shared__ float red[kGvWarps];
    const RouterArgs& r = dl.r;
    const GemvArgs& a = dl.g;
    const int T = a.T, k = a.k, H = a.H, I = a.I, n = T * k;
    const int Sg = a.gu_stages, Sd = a.dn_stages, Smax = Sg > Sd ? Sg : Sd;
    const int Kg = Sg * 256, Kd = Sd * 256;
    const int nb = gridDim.x, b = blockIdx.x, tid = threadIdx.x;
    const DecodeSmem d = decode_smem(sm, Sg, Sd, T, k);
    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < Smax; ++s) mbar_init(&d.bars[s], 1);
        fence_barrier_init();
    }
    // (read only after the grid barrier below)
    if (b == 0)
        for (int i = tid; i < n; i += kGvThreads) {
            dl.mmax[i] = 0u;
            dl.ready[i] = 0u;
        }

    // ---- R: logits of this CTA's (token, row) items
    const int Ew = r.Ew, items = T * Ew, rs = H + 16;  // padded rows
    const int my_n = items > b ? (items - b + nb - 1) / nb : 0;
    float* rows_s = reinterpret_cast<float*>(d.st);  // [my_n + T][rs]: item rows, then tokens
    float* x_s = rows_s + (size_t)my_n * rs;
    {
        const int q4 = H / 4;
        for (int idx = tid; idx < (my_n + T) * q4; idx += kGvThreads) {
            const int rr = idx / q4, q = idx % q4;
            const float* src = rr < my_n ? r.w + (size_t)((b + nb * rr) % Ew) * H + 4 * q
                                         : r.x + (size_t)(rr - my_n) * H + 4 * q;
            float* dst = rows_s + (size_t)rr * rs + 4 * q;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src));
        }
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    if (tid < 64) {
        // warps 0, 1: four 16-lane dot groups over this CTA's items
        const bool tf = r.order == kOrderTf32;
        const int H16 = (H / 16) * 16, grp = tid >> 4, j = tid & 15;
        for (int r0 = 0; r0 < my_n; r0 += 4) {  // uniform over the two warps: both reduce
            const int rr = r0 + grp;
            const bool act = rr < my_n;
            const int it = b + nb * (act ? rr : 0), t = it / Ew, e = it % Ew;
            const float* wrow = rows_s + (size_t)(act ? rr : 0) * rs;
            const float* xrow = x_s + (size_t)t * rs;
            float acc = 0.0f;
            if (act) {
                if (tf) {
#pragma unroll 8
                    for (int i = 0; i < H16; i += 16)
                        acc = __fmaf_rn(wrow[i + j], tf32_trunc(xrow[i + j]), acc);
                } else {
#pragma unroll 8
                    for (int i = 0; i < H16; i += 16) acc = __fmaf_rn(wrow[i + j], xrow[i + j], acc);
                }
            }
            const float q = neon16_tree(acc);
            if (act && j == 0)
                r.logits[(size_t)t * Ew + e] =
                    tf ? neon16_finish<true>(q, wrow, xrow, H16, H, r.bias, e, r.E)
                       : neon16_finish<false>(q, wrow, xrow, H16, H, r.bias, e, r.E);
        }
    } else {
        // warps 2..15, at the same time: the tokens' activation rows -> MoE A8
        // codes (s = max|x| / 127, 0 -> 1), from the staged rows; named
        // barrier 1 over these 448 threads
        constexpr int kQ = kGvThreads - 64;
        const int qt = tid - 64, warp = tid >> 5, lane = tid & 31;
        for (int t = 0; t < T; ++t) {
            const float* xr = x_s + (size_t)t * rs;
            float mx = 0.0f;
            for (int ii = qt; ii < H; ii += kQ) mx = fmaxf(mx, fabsf(xr[ii]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0) red[warp] = mx;
            asm volatile("bar.sync 1, %0;" ::"r"(kQ) : "memory");
            mx = red[2];
            for (int wi = 3; wi < kGvWarps; ++wi) mx = fmaxf(mx, red[wi]);
            asm volatile("bar.sync 1, %0;" ::"r"(kQ) : "memory");
            const float sxt = mx == 0.0f ? 1.0f : __fdiv_rn(mx, 127.0f);
            if (!isfinite(sxt) && b == 0 && qt == 0) atomicOr(a.err, kErrNonFinite);
            if (qt == 0) d.sx[t] = sxt;
            const GvSmem mt = gv_view(d, d.txp + t * Sg * 64, d.tgs + t * Sg * 8, Sg);
            for (int wd = qt; wd < Kg / 8; wd += kQ) {  // whole warps (qt and kQ are warp-aligned)
                uint32_t lo = 0, hi = 0;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    const int kk = wd * 8 + jj;
                    const uint32_t q = kk < H ? (uint32_t)(quant_moe(xr[kk], sxt) & 0xFF) : 0u;
                    if (jj < 4) lo |= q << (8 * jj);
                    else hi |= q << (8 * (jj - 4));
                }
                put_word(mt, wd, lo, hi);
            }
        }
    }
    if (!grid_sync(dl.bar, a.err)) return;  // no copy in flight yet

    // ---- T: routing of every token, in every CTA
    if (r.rule == kRouteGroupedSigmoid) {
        const int warp = tid >> 5, lane = tid & 31;
        if (warp < T) grouped_row(r.logits + (size_t)warp * Ew, r, d.rid + warp * k, d.rw + warp * k, lane);
        __syncthreads();
    } else {
        // topk_row's selection by the whole block: an element's rank under
        // (total_cmp desc, id asc) is the number of elements before it; the
        // element of rank r < k is the r-th pick. Then the same softmax over
        // the picks in rank order (src/model/qwen35/moe.rs:51-67).
        for (int t = 0; t < T; ++t) {
            const float* row = r.logits + (size_t)t * Ew;
            bool fin = true;
            for (int e = tid; e < r.E; e += kGvThreads) {
                const float l = __ldcg(row + e);
                fin = fin && isfinite(l);
                d.keys[e] = (uint32_t)total_key(l) ^ 0x80000000u;
            }
            if (__syncthreads_or(!fin) && tid == 0) atomicOr(r.err, kErrNonFinite);
            // P consecutive threads rank one element, each over a share of
            // the keys (P: the largest power of two with P * E threads)
            int P = 1;
            while (P < 32 && 2 * P * r.E <= kGvThreads) P *= 2;
            const int share = (r.E + P - 1) / P;
            for (int base = 0; base < r.E * P; base += kGvThreads) {
                const int idx = base + tid, e = idx / P, part = idx % P;
                int rank = 0;
                uint32_t ke = 0;
                if (e < r.E) {
                    ke = d.keys[e];
                    const int j1 = min(r.E, (part + 1) * share);
                    for (int jj = part * share; jj < j1; ++jj) {
                        const uint32_t kj = d.keys[jj];
                        rank += (kj > ke || (kj == ke && jj < e)) ? 1 : 0;
                    }
                }
                for (int o = 1; o < P; o <<= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
                if (e < r.E && part == 0 && rank < k) {
                    d.rid[t * k + rank] = e;
                    d.selv[rank] = key_value((int32_t)(ke ^ 0x80000000u));
                }
            }
            __syncthreads();
            if (tid < 32) {
                const float top = d.selv[0];
                float w = tid < k ? expf(__fsub_rn(d.selv[tid], top)) : 0.0f;
                float sum = -0.0f;
                for (int rr = 0; rr < k; ++rr) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, w, rr));
                if (tid < k) {
                    w = __fdiv_rn(w, sum);
                    if (r.min_weight != 0.0f && tid >= 1 && w < r.min_weight) w = 0.0f;
                    d.rw[t * k + tid] = w;
                }
            }
            __syncthreads();
        }
    }
    if (b == 0)
        for (int i = tid; i < n; i += kGvThreads) {
            r.ids[i] = d.rid[i];
            r.weights[i] = d.rw[i];
        }

    const int tg = (I + 63) / 64, td = (H + 127) / 128;
    const int n_gu = n * tg, n_dn = n * td;
    uint32_t phases = 0;  // bit s: phase parity of stage barrier s
    // the stages of a kept down item (after a __syncthreads: nobody reads st)
    auto dn_issue = [&](int i) -> bool {
        const int asg = i / td, dt = i % td;
        const int e = d.rid[asg];
        if (!(d.rw[asg] > 0.0f) || e < 0 || e >= a.E) return false;
        if (tid == 0)
            issue_stages(gv_view(d, d.dxp, d.dgs, Sd),
                         a.dn_w + (size_t)e * a.dn_expert_stride + (size_t)dt * a.dn_tile_stride,
                         a.dn_stage_stride, Sd);
        return true;
    };

    // ---- G: gate/up items i = b, b + nb, ...
    for (int i = b; i < n_gu; i += nb) {
        const int asg = i / tg, rt = i % tg, t = asg / k;
        const float w = d.rw[asg];
        const int e = d.rid[asg];
        if (!(w >= 0.0f) && rt == 0 && tid == 0) atomicOr(a.err, kErrBadRoute);
        if (!(w > 0.0f)) continue;  // skipped route: its middle row is never read
        if (e < 0 || e >= a.E) {
            if (tid == 0) atomicOr(a.err, kErrBadExpert);
            continue;
        }
        const GvSmem m = gv_view(d, d.txp + t * Sg * 64, d.tgs + t * Sg * 8, Sg);
        __syncthreads();
        if (tid == 0)
            issue_stages(m, a.gu_w + (size_t)e * a.gu_expert_stride + (size_t)rt * a.gu_tile_stride,
                         a.gu_stage_stride, Sg);
        const bool ok = group_sums_p(m, Sg, phases, &abort_flag, a.err);
        phases ^= (1u << Sg) - 1u;
        __syncthreads();
        if (tid < 128) d.val[tid] = __fmul_rn(fold_row(m, Sg, tid), d.sx[t]);
        __syncthreads();
        if (tid < 64) {  // warps 0 and 1
            float mloc = 0.0f;
            const int c = rt * 64 + tid;
            if (ok && c < I) {
                const float g = d.val[tid], u = d.val[64 + tid];
                const float dd = __fadd_rn(1.0f, expf(-g));
                const float mv = __fmul_rn(__fdiv_rn(g, dd), u);
                a.middle[(size_t)asg * I + c] = mv;
                mloc = fabsf(mv);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
            // the max of the non-NaN values, as the requantiser's fmaxf reduction
            if ((tid & 31) == 0 && mloc > 0.0f) atomicMax(dl.mmax + asg, __float_as_uint(mloc));
            __threadfence();
        }
        // the item's middle values and row max are visible: count it done
        // (also after a stalled copy, flagged: the count stays consistent)
        __syncthreads();
        if (tid == 0) atomicAdd(dl.ready + asg, 1u);
    }
    // this CTA's down items: i = dn0, dn0 + nb, ... (owner (n_gu + i) % nb, so
    // CTAs without gate/up work take the first ones); request the first one's
    // weights before waiting for its middle row
    const int dn0 = ((b - n_gu) % nb + nb) % nb;
    __syncthreads();
    const bool pref = dn0 < n_dn && dn_issue(dn0);

    // ---- D: down items
    for (int i = dn0; i < n_dn; i += nb) {
        const int asg = i / td, dt = i % td, t = asg / k;
        const float w = d.rw[asg];
        const int e = d.rid[asg];
        const bool valid = e >= 0 && e < a.E, kept = w > 0.0f && valid;
        if (w > 0.0f && !valid && tid == 0) atomicOr(a.err, kErrBadExpert);
        if (kept) {
            if (i != dn0 || !pref) {
                __syncthreads();
                dn_issue(i);
            }
            // the assignment's gate/up items are done (bounded: after the limit
            // the call reports a timeout and its outputs are not used)
            if (tid == 0) {
                const uint64_t start = global_timer_ns();
                while (ld_acquire_gpu(dl.ready + asg) < (uint32_t)tg) {
                    if (global_timer_ns() - start > kWaitLimitNs) {
                        atomicOr(a.err, kErrWaitTimeout);
                        break;
                    }
                }
                __threadfence();
            }
            // requantise the assignment's middle row (MoE A8) into this CTA's
            // codes; the row max and the thread's middle values load together
            const float* mrow = a.middle + (size_t)asg * I;
            const GvSmem m = gv_view(d, d.dxp, d.dgs, Sd);
            __syncthreads();  // the previous item's sums are done with dxp; the wait above
            const float mm = __uint_as_float(__ldcg(dl.mmax + asg));
            const float sc = mm == 0.0f ? 1.0f : __fdiv_rn(mm, 127.0f);
            for (int wd = tid; wd < Kd / 8; wd += kGvThreads) {
                float mv[8];
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) mv[jj] = wd * 8 + jj < I ? __ldcg(mrow + wd * 8 + jj) : 0.0f;
                uint32_t lo = 0, hi = 0;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    const int c = wd * 8 + jj;
                    const uint32_t q = c < I ? (uint32_t)(quant_moe(mv[jj], sc) & 0xFF) : 0u;
                    if (jj < 4) lo |= q << (8 * jj);
                    else hi |= q << (8 * (jj - 4));
                }
                put_word(m, wd, lo, hi);
                if (dt == 0 && wd * 8 < a.ld_qm)
                    *reinterpret_cast<uint2*>(a.q_m + (size_t)asg * a.ld_qm + wd * 8) = make_uint2(lo, hi);
            }
            if (dt == 0 && tid == 0) a.s_m[asg] = sc;
            __syncthreads();
            const bool ok = group_sums_p(m, Sd, phases, &abort_flag, a.err);
            phases ^= (1u << Sd) - 1u;
            __syncthreads();
            if (ok && tid < 128) {
                const int c = dt * 128 + tid;
                const float f = fold_row(m, Sd, tid);
                if (c < H) a.y[(size_t)asg * H + c] = __fmul_rn(f, sc);
            }
        }
        if (!last_arrival(&a.counters[a.dn_counter_base + t * td + dt], k)) continue;
        // combine the token's kept ranks in rank order, then the residual
        for (int c = dt * 128 + tid; c < min(H, dt * 128 + 128); c += kGvThreads) {
            float acc = 0.0f;
            for (int rr = 0; rr < k; ++rr) {
                const int as = t * k + rr;
                const float wr = d.rw[as];
                const int er = d.rid[as];
                if (!(wr > 0.0f) || er < 0 || er >= a.E) continue;
                acc = __fmaf_rn(__ldcg(a.y + (size_t)as * H + c), wr, acc);
            }
            if (a.residual) acc = __fadd_rn(a.residual[(size_t)t * H + c], acc);
            a.out[(size_t)t * H + c] = acc;
        }
    }
}

}  // namespace

constexpr int kMaxDevices = 64;

int launch_decode_layer(const DecodeArgs& d, int num_sms, cudaStream_t s) {
    const GemvArgs& a = d.g;
    const int Sg = a.gu_stages, Sd = a.dn_stages, Smax = Sg > Sd ? Sg : Sd;
    if (a.H % 4 != 0 || Sg > 31 || Sd > 31 || d.r.Ew <= 0 || a.k > 32 || d.r.E > 1024 ||
        a.T > 32)
        return -1;
    const size_t smem = decode_smem_bytes(Sg, Sd, a.T, a.k, d.r.E);
    if (smem > kGemvMaxSmem) return -1;
    // phase R stages its item rows and the token rows in the stage region
    const long items = (long)a.T * d.r.Ew, per = (items + num_sms - 1) / num_sms;
    if ((size_t)(per + a.T) * (a.H + 16) * 4 > (size_t)Smax * kGvStage) return -1;
    // the shared-memory limit and the residency check, once per device and
    // size (a larger limit serves every smaller launch): they cost a call's
    // worth of host time each
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
    {
        static std::mutex mu;
        static size_t ready[kMaxDevices] = {};
        std::lock_guard<std::mutex> lock(mu);
        if (ready[dev] < smem) {
            if (cudaFuncSetAttribute(decode_layer_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem) != cudaSuccess)
                return -1;
            int per_sm = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_layer_kernel,
                                                              kGvThreads, smem) != cudaSuccess ||
                per_sm < 1)
                return -1;
            ready[dev] = smem;
        }
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(kGvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_layer_kernel, d) == cudaSuccess ? 0 : -1;
}

}  // namespace moe
