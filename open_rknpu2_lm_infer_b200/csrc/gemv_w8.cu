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

}  // namespace

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
