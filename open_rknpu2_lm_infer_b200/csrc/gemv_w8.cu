// Small-batch FFN of a per-channel int8 bank (the shared expert of the
// configurations with one): split-K GEMVs on the CUDA cores.
//
// At one to four tokens the tensor-core path of a single dense expert runs 32
// (gate/up) and 16 (down) CTAs, each streaming 256 KB, plus a requantisation
// launch in between. Here every CTA takes one 128-row tile and one 256-k load
// stage of the bank's own packed layout (two 16 KB k-block tiles in the MMA's
// 128-byte swizzle, one bulk copy): 256 and 128 CTAs for I_s = 2048. Integer
// sums are associative, so the stage partials of a row (int8 x int8 over 256
// k, dp4a) meet in an int32 accumulator by atomic adds and the total is the
// exact int32 dot of the tensor-core path; the last stage of a tile to arrive
// dequantises it as that path's per-channel epilogue does,
// ((float)acc * s_x) * s_w. Gate/up tiles (64 gate + 64 up channels) apply
// SwiGLU and keep each token's max |h|; the last tile to arrive requantises
// the middle rows (requant_kernel's arithmetic). Down tiles write the expert
// rows. Every counter and accumulator is re-zeroed by the CTA that consumed
// it, so consecutive calls (and graph replays) start from zero. No CTA waits
// for another (last-arrival hand-offs), and the one bulk copy per CTA is
// waited on with the bounded mbarrier wait.
//
// Reference semantics: the shared expert of src/model/qwen35/moe.rs:304-349
// and the separate dense FFN of src/model/ling3tiny/moe.rs:378-388 (W8A8 with
// the dense A8 rule) or the joint bank of
// llm_generated_docs/MOE_ROUTED_SHARED_JOINT_20261023.md:19 (MoE A8 codes).
#include "kernels.cuh"
#include "quant.cuh"

namespace moe {

namespace {

constexpr int kW8Threads = 128;                // one tile row per thread
constexpr int kW8Stage = 2 * 128 * 128;        // one load stage: two k-block tiles
constexpr int kW8MaxT = 4;                     // tokens per call

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One arrival on `counter`; true in every thread of the CTA that completes
// `expected` arrivals (it re-zeroes the counter). A fence before, for the
// caller's global writes, and after, for the reads of the last one.
__device__ __forceinline__ bool w8_last_arrival(int* counter, int expected) {
    __shared__ int is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(counter, 1);
        is_last = prev == expected - 1;
        if (is_last) *counter = 0;
    }
    __syncthreads();
    if (is_last) __threadfence();
    return is_last != 0;
}

template <bool GATEUP>
__global__ void __launch_bounds__(kW8Threads) shared_w8_kernel(const W8GemvArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    __shared__ float vals[kW8MaxT][128];
    uint32_t* xs = reinterpret_cast<uint32_t*>(sm + kW8Stage);  // [T][64] activation words
    const int rt = blockIdx.x, ks = blockIdx.y, lr = threadIdx.x, T = a.T;
    const int rows = gridDim.x * 128;
    if (lr == 0) {
        abort_flag = 0;
        mbar_init(&bar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(&bar, kW8Stage);
        bulk_g2s(sm, a.w + (size_t)rt * a.w_tile_stride + (size_t)ks * a.w_stage_stride, kW8Stage,
                 &bar);
    }
    for (int i = lr; i < T * 64; i += kW8Threads) {
        const int t = i >> 6, wd = i & 63;
        xs[i] = *reinterpret_cast<const uint32_t*>(a.q + (size_t)t * a.ld + ks * 256 + 4 * wd);
    }
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, &abort_flag, a.err);
    int acc[kW8MaxT] = {0, 0, 0, 0};
    if (ok) {
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
            const uint8_t* row = sm + kb * 16384 + lr * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {  // 16-byte chunk c holds k 16c..16c+15 of the k-block
                const uint4 wv = *reinterpret_cast<const uint4*>(row + ((c ^ (lr & 7)) << 4));
                const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int t = 0; t < kW8MaxT; ++t) {
                    if (t < T) {
                        const uint32_t* x = xs + t * 64 + kb * 32 + 4 * c;
#pragma unroll
                        for (int i = 0; i < 4; ++i) acc[t] = dp4a_ss(wd[i], x[i], acc[t]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < kW8MaxT; ++t)
        if (t < T && acc[t] != 0) atomicAdd(a.acc + (size_t)t * rows + rt * 128 + lr, acc[t]);
    if (!w8_last_arrival(a.counters + rt, gridDim.y)) return;

    // the tile's exact sums -> dequantised values (the accumulators re-zeroed)
    const float sw = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(a.wscale) +
                                                    (size_t)rt * a.ws_tile_stride)[lr];
    for (int t = 0; t < T; ++t) {
        int32_t* ap = a.acc + (size_t)t * rows + rt * 128 + lr;
        const int v = __ldcg(ap);
        *ap = 0;
        vals[t][lr] = __fmul_rn(__fmul_rn(__int2float_rn(v), a.sx[t]), sw);
    }
    if constexpr (!GATEUP) {
        const int c = rt * 128 + lr;
        if (c < a.n)
            for (int t = 0; t < T; ++t) a.out[(size_t)t * a.n + c] = vals[t][lr];
        return;
    } else {
        __syncthreads();
        // SwiGLU of channel rt * 64 + lr (gate row lr, up row 64 + lr), the
        // tokens' max |h| over the tile (warps 0 and 1)
        if (lr < 64) {
            const int c = rt * 64 + lr;
            for (int t = 0; t < T; ++t) {
                float m = 0.0f;
                if (c < a.n) {
                    const float h = silu_mul(vals[t][lr], vals[t][64 + lr]);
                    a.out[(size_t)t * a.n + c] = h;
                    m = fabsf(h);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                if ((lr & 31) == 0 && m > 0.0f) atomicMax(a.row_max + t, __float_as_uint(m));
            }
        }
        // the last tile requantises the middle rows
        if (!w8_last_arrival(a.counters + gridDim.x, gridDim.x)) return;
        const int n4 = a.n / 4;
        for (int t = 0; t < T; ++t) {
            const float m = __uint_as_float(__ldcg(a.row_max + t));
            const float sc = row_scale(m, a.rule);
            const float inv = __fdiv_rn(1.0f, sc);
            const float4* hr = reinterpret_cast<const float4*>(a.out + (size_t)t * a.n);
            uint32_t* qr = reinterpret_cast<uint32_t*>(a.q_out + (size_t)t * a.ld_q);
            for (int c4 = lr; c4 < n4; c4 += kW8Threads) qr[c4] = quant4(__ldcg(hr + c4), sc, inv, a.rule);
            __syncthreads();  // every thread read the row max before it is re-zeroed
            if (lr == 0) {
                a.q_scale[t] = sc;
                a.row_max[t] = 0u;
            }
        }
    }
}

// The stage's 256 codes of tile row lr (two k-block tiles of 128 rows x 128
// bytes in the 128-byte swizzle, at sm) dotted with 64 activation words.
__device__ __forceinline__ int w8_row_dot(const uint8_t* sm, int lr, const uint32_t* x) {
    int acc = 0;
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
        const uint8_t* row = sm + kb * 16384 + lr * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 wv = *reinterpret_cast<const uint4*>(row + ((c ^ (lr & 7)) << 4));
            const uint32_t* xx = x + kb * 32 + 4 * c;
            acc = dp4a_ss(wv.x, xx[0], acc);
            acc = dp4a_ss(wv.y, xx[1], acc);
            acc = dp4a_ss(wv.z, xx[2], acc);
            acc = dp4a_ss(wv.w, xx[3], acc);
        }
    }
    return acc;
}

// Routed gate/up: grid (T*k assignments, I/64 tiles, K/256 stages). Every CTA
// of a kept assignment quantises its token's stage codes (MoE A8 over the
// whole row, quant_gather's rule), adds its rows' stage sums; the last stage
// of a tile dequantises it and applies SwiGLU; the last tile of the
// assignment quantises the middle row.
__global__ void __launch_bounds__(kW8Threads) routed_w8_gateup_kernel(const W8RoutedArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    __shared__ float red[kW8Threads / 32];
    __shared__ float vals[128];
    uint32_t* xs = reinterpret_cast<uint32_t*>(sm + kW8Stage);  // [64] activation words
    const int asg = blockIdx.x, rt = blockIdx.y, ks = blockIdx.z, lr = threadIdx.x;
    const int t = asg / a.k, tiles = gridDim.y;
    const float w = a.routes[asg];
    const int e = a.ids[asg];
    if (!(w >= 0.0f) && rt == 0 && ks == 0 && lr == 0) atomicOr(a.err, kErrBadRoute);
    if (!(w > 0.0f)) return;  // skipped route: its middle row is never read
    if (e < 0 || e >= a.E) {
        if (rt == 0 && ks == 0 && lr == 0) atomicOr(a.err, kErrBadExpert);
        return;
    }
    if (lr == 0) {
        abort_flag = 0;
        mbar_init(&bar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(&bar, kW8Stage);
        bulk_g2s(sm, a.gu_w + (size_t)e * a.gu_expert_stride + (size_t)rt * a.gu_tile_stride +
                         (size_t)ks * a.gu_stage_stride,
                 kW8Stage, &bar);
    }
    // the token's row maximum, then this stage's 256 codes
    const float* xr = a.x + (size_t)t * a.H;
    float mx = 0.0f;
    for (int i = lr; i < a.H; i += kW8Threads) mx = fmaxf(mx, fabsf(xr[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((lr & 31) == 0) red[lr >> 5] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float sx = row_scale(mx, kQuantMoe);
    const float inv = __fdiv_rn(1.0f, sx);
    if (lr < 64) {
        const int k0 = ks * 256 + 4 * lr;
        const float4 v = make_float4(k0 < a.H ? xr[k0] : 0.0f, k0 + 1 < a.H ? xr[k0 + 1] : 0.0f,
                                     k0 + 2 < a.H ? xr[k0 + 2] : 0.0f, k0 + 3 < a.H ? xr[k0 + 3] : 0.0f);
        xs[lr] = quant4(v, sx, inv, kQuantMoe);
    }
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, &abort_flag, a.err);
    const int rows = tiles * 128 > ((a.H + 127) / 128) * 128 ? tiles * 128 : ((a.H + 127) / 128) * 128;
    if (ok) {
        const int acc = w8_row_dot(sm, lr, xs);
        if (acc != 0) atomicAdd(a.acc + (size_t)asg * rows + rt * 128 + lr, acc);
    }
    int* cnt = a.counters;
    if (!w8_last_arrival(cnt + (size_t)asg * tiles + rt, gridDim.z)) return;
    // the tile: dequantise, SwiGLU of channel rt * 64 + lr, the row's max |h|
    {
        int32_t* ap = a.acc + (size_t)asg * rows + rt * 128 + lr;
        const int v = __ldcg(ap);
        *ap = 0;
        const float sw = a.gu_s[(size_t)e * (a.gu_s_expert_stride / 4) + (size_t)rt * (a.gu_s_tile_stride / 4) + lr];
        vals[lr] = __fmul_rn(__fmul_rn(__int2float_rn(v), sx), sw);
    }
    __syncthreads();
    if (lr < 64) {
        const int c = rt * 64 + lr;
        float m = 0.0f;
        if (c < a.I) {
            const float h = silu_mul(vals[lr], vals[64 + lr]);
            a.middle[(size_t)asg * a.I + c] = h;
            m = fabsf(h);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((lr & 31) == 0 && m > 0.0f) atomicMax(a.row_max + asg, __float_as_uint(m));
    }
    const int n = a.T * a.k;
    if (!w8_last_arrival(cnt + (size_t)n * tiles + asg, tiles)) return;
    // the middle row's codes (requant_kernel's rule and rounding)
    const float m = __uint_as_float(__ldcg(a.row_max + asg));
    const float sc = row_scale(m, kQuantMoe);
    const float ic = __fdiv_rn(1.0f, sc);
    const float4* hr = reinterpret_cast<const float4*>(a.middle + (size_t)asg * a.I);
    uint32_t* qr = reinterpret_cast<uint32_t*>(a.q_m + (size_t)asg * a.ld_qm);
    for (int c4 = lr; c4 < a.I / 4; c4 += kW8Threads) qr[c4] = quant4(__ldcg(hr + c4), sc, ic, kQuantMoe);
    __syncthreads();
    if (lr == 0) {
        a.s_m[asg] = sc;
        a.row_max[asg] = 0u;
    }
}

// Routed down: grid (T*k, H/128 tiles, I/256 stages); the last stage of a
// tile writes the expert rows; the last of a (token, tile)'s k assignments
// (kept or not: one arrival each) combines.
__global__ void __launch_bounds__(kW8Threads) routed_w8_down_kernel(const W8RoutedArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    uint32_t* xs = reinterpret_cast<uint32_t*>(sm + kW8Stage);
    const int asg = blockIdx.x, rt = blockIdx.y, ks = blockIdx.z, lr = threadIdx.x;
    const int t = asg / a.k, tiles = gridDim.y, n = a.T * a.k;
    const int gu_tiles = (a.I + 63) / 64;
    const float w = a.routes[asg];
    const int e = a.ids[asg];
    const bool kept = w > 0.0f && e >= 0 && e < a.E;
    int* cnt = a.counters + (size_t)n * gu_tiles + n;  // down: [n][tiles], then [T][tiles]
    const int rows = gu_tiles * 128 > tiles * 128 ? gu_tiles * 128 : tiles * 128;
    if (kept) {
        if (lr == 0) {
            abort_flag = 0;
            mbar_init(&bar, 1);
            fence_barrier_init();
            mbar_arrive_expect_tx(&bar, kW8Stage);
            bulk_g2s(sm, a.dn_w + (size_t)e * a.dn_expert_stride + (size_t)rt * a.dn_tile_stride +
                             (size_t)ks * a.dn_stage_stride,
                     kW8Stage, &bar);
        }
        if (lr < 64)
            xs[lr] = __ldcg(reinterpret_cast<const uint32_t*>(a.q_m + (size_t)asg * a.ld_qm + ks * 256) + lr);
        __syncthreads();
        if (mbar_wait(&bar, 0, &abort_flag, a.err)) {
            const int acc = w8_row_dot(sm, lr, xs);
            if (acc != 0) atomicAdd(a.acc + (size_t)asg * rows + rt * 128 + lr, acc);
        }
        if (!w8_last_arrival(cnt + (size_t)asg * tiles + rt, gridDim.z)) return;
        int32_t* ap = a.acc + (size_t)asg * rows + rt * 128 + lr;
        const int v = __ldcg(ap);
        *ap = 0;
        const float sw = a.dn_s[(size_t)e * (a.dn_s_expert_stride / 4) + (size_t)rt * (a.dn_s_tile_stride / 4) + lr];
        const int c = rt * 128 + lr;
        if (c < a.H) a.y[(size_t)asg * a.H + c] = __fmul_rn(__fmul_rn(__int2float_rn(v), a.s_m[asg]), sw);
    } else if (ks != 0) {
        return;  // one arrival per skipped assignment
    }
    if (!w8_last_arrival(cnt + (size_t)n * tiles + t * tiles + rt, a.k)) return;
    // the token's kept ranks in rank order, the shared row, the residual
    // (combine_kernel's order and roundings)
    const int c = rt * 128 + lr;
    if (c >= a.H) return;
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
        if (a.gate)
            sv = __fmul_rn(__fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f32(-a.gate[(size_t)t * a.gate_ld]))), sv);
        acc = __fadd_rn(acc, sv);
    }
    if (a.residual) acc = __fadd_rn(a.residual[(size_t)t * a.H + c], acc);
    a.out[(size_t)t * a.H + c] = acc;
}

}  // namespace

int launch_routed_w8(const W8RoutedArgs& a, int part, cudaStream_t s) {
    if (a.T < 1 || a.T > kW8MaxT || a.I % 4 != 0 || a.H % 4 != 0 || a.gu_stages < 1 ||
        a.dn_stages < 1)
        return -1;
    const int n = a.T * a.k;
    const size_t smem = kW8Stage + 256;
    if (part == 0) {
        cudaFuncSetAttribute(routed_w8_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        routed_w8_gateup_kernel<<<dim3(n, (a.I + 63) / 64, a.gu_stages), kW8Threads, smem, s>>>(a);
    } else {
        cudaFuncSetAttribute(routed_w8_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        routed_w8_down_kernel<<<dim3(n, (a.H + 127) / 128, a.dn_stages), kW8Threads, smem, s>>>(a);
    }
    return 0;
}

int launch_shared_w8(const W8GemvArgs& a, bool gateup, int row_tiles, int kstages,
                     cudaStream_t s) {
    if (a.T < 1 || a.T > kW8MaxT || a.n % 4 != 0 || row_tiles < 1 || kstages < 1) return -1;
    const size_t smem = kW8Stage + (size_t)a.T * 256;
    auto k = gateup ? shared_w8_kernel<true> : shared_w8_kernel<false>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<dim3(row_tiles, kstages), kW8Threads, smem, s>>>(a);
    return 0;
}

}  // namespace moe
