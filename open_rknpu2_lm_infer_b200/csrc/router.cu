// Router logits + softmax top-k (+ renormalisation and optional pruning).
//
// Reference semantics (happyme531/open_rknpu2_lm_infer):
//   logits  : Cpu::dense_head_batch / dense_dot, src/model/cpu.rs:96-153,302-316
//   top-k   : routes(), src/model/qwen35/moe.rs:51-67 (total_cmp desc, lower id on ties,
//             weights = exp(l - l_max) / sum over the selected k)
//   pruning : pruning::apply, src/model/experts/pruning.rs:32-41
//
// The NEON16 order keeps 16 independent FMA lanes per (token, expert) dot —
// lane j accumulates elements 16i + j — then reduces them with the fixed tree
// (l[j]+l[j+4]) + (l[j+8]+l[j+12]) and ((v0+v1)+(v2+v3)) of vaddq/vaddvq, and
// finishes with a separately rounded scalar tail. Every rounding step matches
// the reference, so logits (and hence expert ids) are bit-identical.
#include "kernels.cuh"

namespace moe {

constexpr int kRouterThreads = 256;
constexpr int kRouterEB = 128;          // experts per block pass
constexpr int kRouterChunk = 64;        // hidden elements per smem stage
constexpr int kRouterWStride = kRouterChunk + 16;  // padded row: conflict-free

// grid: (ceil(T/TT), ceil(E/EB)). Each CTA computes logits for TT tokens x EB
// experts into `logits`; the last CTA of a token tile to finish runs top-k.
template <int TT>
__global__ void __launch_bounds__(kRouterThreads)
router_neon16_kernel(const float* __restrict__ x, const float* __restrict__ wr,
                     const float* __restrict__ bias, int T, int H, int E, float* logits,
                     int* tile_counter, int k, float min_weight, int32_t* ids, float* weights,
                     uint32_t* err) {
    constexpr int EPG = kRouterEB / 16;  // experts per 16-thread group
    extern __shared__ __align__(16) float router_smem[];
    float* w_s[2] = {router_smem, router_smem + kRouterEB * kRouterWStride};
    float* x_s[2] = {router_smem + 2 * kRouterEB * kRouterWStride,
                     router_smem + 2 * kRouterEB * kRouterWStride + TT * kRouterChunk};
    __shared__ int is_last;

    const int tid = threadIdx.x;
    const int j = tid & 15;
    const int g = tid >> 4;
    const int t0 = blockIdx.x * TT;
    const int e0 = blockIdx.y * kRouterEB;
    const int ne = min(kRouterEB, E - e0);
    const int nt = min(TT, T - t0);
    const int H16 = (H / 16) * 16;
    const int nchunks = (H16 + kRouterChunk - 1) / kRouterChunk;

    float acc[TT][EPG];
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
        for (int m = 0; m < EPG; ++m) acc[t][m] = 0.0f;

    // stage loader: cp.async 16-byte pieces of the w rows and x rows of one chunk
    auto load_chunk = [&](int c, int buf) {
        const int h0 = c * kRouterChunk;
        const int len = min(kRouterChunk, H16 - h0);  // multiple of 16
        const int q4 = len / 4;
        for (int idx = tid; idx < kRouterEB * (kRouterChunk / 4); idx += kRouterThreads) {
            int e = idx / (kRouterChunk / 4), q = idx % (kRouterChunk / 4);
            float* dst = &w_s[buf][e * kRouterWStride + 4 * q];
            if (e < ne && q < q4 && (((H & 3) == 0))) {
                const float* src = wr + (size_t)(e0 + e) * H + h0 + 4 * q;
                asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)),
                             "l"(src));
            } else if (e < ne && q < q4) {
                for (int c2 = 0; c2 < 4; ++c2) dst[c2] = wr[(size_t)(e0 + e) * H + h0 + 4 * q + c2];
            }
        }
        for (int idx = tid; idx < TT * (kRouterChunk / 4); idx += kRouterThreads) {
            int t = idx / (kRouterChunk / 4), q = idx % (kRouterChunk / 4);
            float* dst = &x_s[buf][t * kRouterChunk + 4 * q];
            if (t < nt && q < q4 && ((H & 3) == 0)) {
                const float* src = x + (size_t)(t0 + t) * H + h0 + 4 * q;
                asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)),
                             "l"(src));
            } else if (t < nt && q < q4) {
                for (int c2 = 0; c2 < 4; ++c2) dst[c2] = x[(size_t)(t0 + t) * H + h0 + 4 * q + c2];
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    if (nchunks > 0) load_chunk(0, 0);
    for (int c = 0; c < nchunks; ++c) {
        const int buf = c & 1;
        if (c + 1 < nchunks) {
            load_chunk(c + 1, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const int steps = min(kRouterChunk, H16 - c * kRouterChunk) / 16;
#pragma unroll
        for (int i = 0; i < kRouterChunk / 16; ++i) {
            if (i < steps) {
                float wv[EPG];
#pragma unroll
                for (int m = 0; m < EPG; ++m)
                    wv[m] = w_s[buf][(g + 16 * m) * kRouterWStride + 16 * i + j];
#pragma unroll
                for (int t = 0; t < TT; ++t) {
                    const float xv = x_s[buf][t * kRouterChunk + 16 * i + j];
#pragma unroll
                    for (int m = 0; m < EPG; ++m) acc[t][m] = __fmaf_rn(wv[m], xv, acc[t][m]);
                }
            }
        }
        __syncthreads();
    }

    // fixed reduction tree over the 16 lanes of each (t, e) dot
#pragma unroll
    for (int t = 0; t < TT; ++t) {
#pragma unroll
        for (int m = 0; m < EPG; ++m) {
            float v = acc[t][m];
            float s1 = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 16));     // a+b / c+d
            float s2 = __fadd_rn(s1, __shfl_down_sync(0xffffffffu, s1, 8, 16));   // (a+b)+(c+d)
            float p = __fadd_rn(s2, __shfl_down_sync(0xffffffffu, s2, 1, 16));    // v0+v1, v2+v3
            float q = __fadd_rn(p, __shfl_down_sync(0xffffffffu, p, 2, 16));      // total
            const int e = g + 16 * m;
            if (j == 0 && t < nt && e < ne) {
                const float* wrow = wr + (size_t)(e0 + e) * H;
                const float* xrow = x + (size_t)(t0 + t) * H;
                for (int h = H16; h < H; ++h) q = __fadd_rn(q, __fmul_rn(wrow[h], xrow[h]));
                if (bias) q = __fadd_rn(q, bias[e0 + e]);
                logits[(size_t)(t0 + t) * E + e0 + e] = q;
            }
        }
    }

    // last CTA of this token tile runs top-k over all E logits
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        int prev = atomicAdd(&tile_counter[blockIdx.x], 1);
        is_last = (prev == (int)gridDim.y - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const int warp = tid >> 5, lane = tid & 31;
    for (int t = warp; t < nt; t += kRouterThreads / 32)
        topk_row(logits + (size_t)(t0 + t) * E, E, k, min_weight, ids + (size_t)(t0 + t) * k,
                 weights + (size_t)(t0 + t) * k, lane, err);
    if (tid == 0) tile_counter[blockIdx.x] = 0;
}

// x86 order: one thread per (token, expert), sequential sum += w*x with a
// separately rounded product (src/model/cpu.rs:148-151).
__global__ void router_sequential_kernel(const float* __restrict__ x, const float* __restrict__ wr,
                                         const float* __restrict__ bias, int T, int H, int E,
                                         float* logits) {
    const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long)T * E) return;
    const int t = (int)(idx / E), e = (int)(idx % E);
    const float* wrow = wr + (size_t)e * H;
    const float* xrow = x + (size_t)t * H;
    float s = 0.0f;
    for (int h = 0; h < H; ++h) s = __fadd_rn(s, __fmul_rn(wrow[h], xrow[h]));
    if (bias) s = __fadd_rn(s, bias[e]);
    logits[idx] = s;
}

__global__ void topk_kernel(const float* __restrict__ logits, int T, int E, int k,
                            float min_weight, int32_t* ids, float* weights, uint32_t* err) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    topk_row(logits + (size_t)warp * E, E, k, min_weight, ids + (size_t)warp * k,
             weights + (size_t)warp * k, lane, err);
}

// One warp selects the top-k of a row of E logits (E <= 1024): k rounds of a
// warp arg-max over (total_cmp key, -id), then softmax over the selected.
__device__ void topk_row(const float* row, int E, int k, float min_weight, int32_t* ids,
                         float* weights, int lane, uint32_t* err) {
    uint32_t taken = 0;  // bit i: element lane + 32*i already selected
    const int per_lane = (E + 31) / 32;
    int my_id = -1;
    bool finite = true;
    for (int i = 0; i < per_lane; ++i) {
        int e = lane + 32 * i;
        if (e < E && !isfinite(row[e])) finite = false;
    }
    if (__any_sync(0xffffffffu, !finite) && lane == 0) atomicOr(err, kErrNonFinite);
    for (int r = 0; r < k; ++r) {
        unsigned long long best = 0ull;
        for (int i = 0; i < per_lane; ++i) {
            int e = lane + 32 * i;
            if (e >= E || (taken >> i) & 1u) continue;
            uint32_t key = (uint32_t)total_key(row[e]) ^ 0x80000000u;
            unsigned long long v = ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)e);
            if (v > best) best = v;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
            if (o > best) best = o;
        }
        const int win = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
        if ((win & 31) == lane) taken |= 1u << (win >> 5);
        if (lane == r) my_id = win;
    }
    // softmax over the selected, in rank order (src/model/qwen35/moe.rs:60-65)
    const int id0 = __shfl_sync(0xffffffffu, my_id, 0);
    const float mx = row[id0];
    float w = 0.0f;
    if (lane < k) w = expf(__fsub_rn(row[my_id], mx));
    float sum = -0.0f;
    for (int r = 0; r < k; ++r) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, w, r));
    if (lane < k) {
        w = __fdiv_rn(w, sum);
        if (min_weight != 0.0f && lane >= 1 && w < min_weight) w = 0.0f;
        ids[lane] = my_id;
        weights[lane] = w;
    }
}

template <int TT>
static void launch_neon16(const RouterArgs& a, cudaStream_t s) {
    const size_t smem = sizeof(float) * (2 * kRouterEB * kRouterWStride + 2 * TT * kRouterChunk);
    static bool configured = false;  // attribute is per function, set once per process
    if (!configured) {
        cudaFuncSetAttribute(router_neon16_kernel<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
        configured = true;
    }
    dim3 grid((a.T + TT - 1) / TT, (a.E + kRouterEB - 1) / kRouterEB);
    router_neon16_kernel<TT><<<grid, kRouterThreads, smem, s>>>(
        a.x, a.w, a.bias, a.T, a.H, a.E, a.logits, a.counters, a.k, a.min_weight, a.ids,
        a.weights, a.err);
}

int launch_router(const RouterArgs& a, cudaStream_t s) {
    if (a.order == 1) {
        const long n = (long)a.T * a.E;
        router_sequential_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
            a.x, a.w, a.bias, a.T, a.H, a.E, a.logits);
        topk_kernel<<<(a.T * 32 + 255) / 256, 256, 0, s>>>(a.logits, a.T, a.E, a.k,
                                                           a.min_weight, a.ids, a.weights, a.err);
        return 0;
    }
    if (a.T >= 2048)
        launch_neon16<16>(a, s);
    else if (a.T >= 64)
        launch_neon16<4>(a, s);
    else
        launch_neon16<1>(a, s);
    return 0;
}

}  // namespace moe
