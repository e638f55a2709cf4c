// Router logits + top-k routing (+ renormalisation and optional pruning).
//
// Reference semantics (happyme531/open_rknpu2_lm_infer):
//   logits  : Cpu::dense_head_batch / dense_dot, src/model/cpu.rs:96-153,302-316;
//             Ling's TF32 NPU linear, src/npu/tf32.rs:142-170 (operands narrowed)
//   softmax : routes(), src/model/qwen35/moe.rs:51-67 (total_cmp desc, lower id on ties,
//             weights = exp(l - l_max) / sum over the selected k)
//   grouped : RoutingScratch::routes, src/model/ling3tiny/moe.rs:146-223 (sigmoid
//             scores, biased selection, top-2 group sums, top groups, routing scale)
//   pruning : pruning::apply, src/model/experts/pruning.rs:32-41
//   gate    : the shared-expert gate row, src/model/qwen35/moe.rs:334-347, is one
//             more weight row after the E experts (logit column E)
//
// The NEON16 order keeps 16 independent FMA lanes per (token, expert) dot —
// lane j accumulates elements 16i + j — then reduces them with the fixed tree
// (l[j]+l[j+4]) + (l[j+8]+l[j+12]) and ((v0+v1)+(v2+v3)) of vaddq/vaddvq, and
// finishes with a separately rounded scalar tail. Every rounding step matches
// the reference, so logits (and hence expert ids) are bit-identical. The TF32
// order runs the same kernels on operands narrowed to TF32; the reference's
// NPU fixes no summation order, only a bound (5e-5 of the f64 sum).
#include "kernels.cuh"
#include "route.cuh"

namespace moe {

__device__ __forceinline__ void route_row(const RouterArgs& a, int t, int lane) {
    const float* row = a.logits + (size_t)t * a.Ew;
    if (a.rule == kRouteGroupedSigmoid)
        grouped_row(row, a, a.ids + (size_t)t * a.k, a.weights + (size_t)t * a.k, lane);
    else
        topk_row(row, a.E, a.k, a.min_weight, a.ids + (size_t)t * a.k,
                 a.weights + (size_t)t * a.k, lane, a.err);
}

// Last CTA of a token tile (all expert blocks done) routes its tokens.
__device__ __forceinline__ void finish_tile(const RouterArgs& a, int tile, int t0, int nt) {
    __shared__ int is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(&a.counters[tile], 1);
        is_last = (prev == (int)gridDim.y - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = warp; t < nt; t += blockDim.x / 32) route_row(a, t0 + t, lane);
    if (threadIdx.x == 0) a.counters[tile] = 0;
}

// Decode-sized router: one token, 8 weight rows per CTA (grid (T, ceil(Ew/8))),
// 128 threads = 8 rows x 16 lanes. The CTA's router rows and the token row
// are staged in shared memory with one batch of 16-byte copies, then each
// thread runs its lane's sequential FMA chain.
constexpr int kDecEB = 8;
template <bool TF32>
__global__ void __launch_bounds__(128) router_decode_kernel(const RouterArgs a) {
    extern __shared__ __align__(16) float rsm[];
    // a small-batch layer launches its gate/up kernel as a programmatic
    // dependent: it may start its own prologue now (it waits for this grid
    // before reading the routing)
    pdl_trigger();
    const int H = a.H;
    const int stride = H + 16;  // padded rows: the two rows of a warp use different banks
    float* w_s = rsm;                     // [8][stride]
    float* x_s = rsm + kDecEB * stride;   // [H]
    const int t = blockIdx.x, e0 = blockIdx.y * kDecEB;
    const int ne = min(kDecEB, a.Ew - e0);
    const int H16 = (H / 16) * 16;
    const bool vec = (H & 3) == 0;
    if (vec) {
        const int q4 = H / 4;
        for (int idx = threadIdx.x; idx < (ne + 1) * q4; idx += blockDim.x) {
            const int r = idx / q4, q = idx % q4;
            const float* src = r < ne ? a.w + (size_t)(e0 + r) * H + 4 * q : a.x + (size_t)t * H + 4 * q;
            float* dst = r < ne ? w_s + r * stride + 4 * q : x_s + 4 * q;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src));
        }
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
    } else {
        for (int idx = threadIdx.x; idx < (ne + 1) * H; idx += blockDim.x) {
            const int r = idx / H, h = idx % H;
            if (r < ne) w_s[r * stride + h] = a.w[(size_t)(e0 + r) * H + h];
            else x_s[h] = a.x[(size_t)t * H + h];
        }
    }
    __syncthreads();
    const int j = threadIdx.x & 15, el = threadIdx.x >> 4;
    float acc = 0.0f;
    if (el < ne) {
        const float* wrow = w_s + el * stride;
#pragma unroll 8
        for (int i = 0; i < H16; i += 16)
            acc = __fmaf_rn(wrow[i + j], xval<TF32>(x_s[i + j]), acc);
    }
    const float q = neon16_tree(acc);
    if (j == 0 && el < ne)
        a.logits[(size_t)t * a.Ew + e0 + el] =
            neon16_finish<TF32>(q, w_s + el * stride, x_s, H16, H, a.bias, e0 + el, a.E);
    finish_tile(a, t, t, 1);
}

// Prefill-sized router (logits only; the routing runs in route_rows_kernel).
// A thread owns TT tokens x 4 weight rows x 4 NEON lanes (j = 4q + c): one
// 16-byte shared-memory read per token and per row covers the 4 lanes' next
// element, lanes (c, c + 1) advance together as one paired FMA (fma.rn.f32x2:
// two independent fmaf roundings), and the 64 (or 32) chains per thread are
// independent. UNR 16-element steps are unrolled together. A warp =
// 4 lane groups q x 8 row groups s (rows s, s + 8, s + 16, s + 24 of the
// warp's 32); a CTA = WY x WX warps = WY*TT tokens x WX*32 rows. The hidden
// dimension streams in chunks of KCH through an STG-deep cp.async ring; row
// strides of KCH + 4 floats keep the 16-byte reads conflict-free. The fixed
// reduction tree of the reference's lanes, (l[c] + l[c+4]) + (l[c+8] +
// l[c+12]) then (v0 + v1) + (v2 + v3), pairs lane groups q ^ 1, then q ^ 2.
template <int TT, int WY, int WX, int KCH, int STG, int UNR, bool TF32>
__global__ void __launch_bounds__(32 * WY * WX) router_tile4_kernel(const RouterArgs a) {
    constexpr int TTc = TT * WY, EBc = 32 * WX;
    constexpr int WS = KCH + 4, XS = KCH + 4;
    constexpr int kStageF = EBc * WS + TTc * XS;
    constexpr int NTH = 32 * WY * WX;
    extern __shared__ __align__(16) float rsm[];
    const int H = a.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q = lane >> 3, sg = lane & 7;
    const int wy = warp / WX, wx = warp % WX;
    const int t0 = blockIdx.x * TTc, e0 = blockIdx.y * EBc;
    const int ne = min(EBc, a.Ew - e0), nt = min(TTc, a.T - t0);
    const int H16 = (H / 16) * 16;
    const int nchunks = (H16 + KCH - 1) / KCH;

    auto load_chunk = [&](int c) {
        float* w_s = rsm + (c % STG) * kStageF;
        float* x_s = w_s + EBc * WS;
        const int h0 = c * KCH;
        const int q4 = min(KCH, H16 - h0) / 4;
        for (int idx = tid; idx < (EBc + TTc) * (KCH / 4); idx += NTH) {
            const int r = idx / (KCH / 4), qq = idx % (KCH / 4);
            if (qq >= q4) continue;
            const bool isw = r < EBc;
            if (isw ? r >= ne : (r - EBc) >= nt) continue;
            const float* src = isw ? a.w + (size_t)(e0 + r) * H + h0 + 4 * qq
                                   : a.x + (size_t)(t0 + r - EBc) * H + h0 + 4 * qq;
            float* dst = isw ? w_s + r * WS + 4 * qq : x_s + (r - EBc) * XS + 4 * qq;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src));
        }
    };

    float2 acc[TT][4][2];
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
        for (int m = 0; m < 4; ++m) acc[t][m][0] = acc[t][m][1] = make_float2(0.0f, 0.0f);

    for (int c = 0; c < STG - 1; ++c) {
        if (c < nchunks) load_chunk(c);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int c = 0; c < nchunks; ++c) {
        asm volatile("cp.async.wait_group %0;" ::"n"(STG - 2) : "memory");
        __syncthreads();
        if (c + STG - 1 < nchunks) load_chunk(c + STG - 1);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const float* w_s = rsm + (c % STG) * kStageF + (wx * 32 + sg) * WS + 4 * q;
        const float* x_s = rsm + (c % STG) * kStageF + EBc * WS + (wy * TT) * XS + 4 * q;
        const int steps = min(KCH, H16 - c * KCH) / 16;
#pragma unroll UNR
        for (int i = 0; i < steps; ++i) {
            float4 xv[TT];
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                xv[t] = *reinterpret_cast<const float4*>(x_s + t * XS + 16 * i);
                xv[t] = make_float4(xval<TF32>(xv[t].x), xval<TF32>(xv[t].y), xval<TF32>(xv[t].z),
                                    xval<TF32>(xv[t].w));
            }
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const float4 wv = *reinterpret_cast<const float4*>(w_s + (8 * m) * WS + 16 * i);
#pragma unroll
                for (int t = 0; t < TT; ++t) {
                    acc[t][m][0] = __ffma2_rn(make_float2(wv.x, wv.y), make_float2(xv[t].x, xv[t].y), acc[t][m][0]);
                    acc[t][m][1] = __ffma2_rn(make_float2(wv.z, wv.w), make_float2(xv[t].z, xv[t].w), acc[t][m][1]);
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
    for (int t = 0; t < TT; ++t) {
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const float l4[4] = {acc[t][m][0].x, acc[t][m][0].y, acc[t][m][1].x, acc[t][m][1].y};
            float v[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float s1 = __fadd_rn(l4[c], __shfl_xor_sync(0xffffffffu, l4[c], 8));
                v[c] = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 16));
            }
            const float tot = __fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3]));
            const int tl = wy * TT + t, el = wx * 32 + sg + 8 * m;
            if (q == 0 && tl < nt && el < ne)
                a.logits[(size_t)(t0 + tl) * a.Ew + e0 + el] = neon16_finish<TF32>(
                    tot, a.w + (size_t)(e0 + el) * H, a.x + (size_t)(t0 + tl) * H, H16, H, a.bias,
                    e0 + el, a.E);
        }
    }
}

// x86 order: one thread per (token, row), sequential sum += w*x with a
// separately rounded product (src/model/cpu.rs:148-151).
__global__ void router_sequential_kernel(const RouterArgs a) {
    const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long)a.T * a.Ew) return;
    const int t = (int)(idx / a.Ew), e = (int)(idx % a.Ew);
    const float* wrow = a.w + (size_t)e * a.H;
    const float* xrow = a.x + (size_t)t * a.H;
    float s = 0.0f;
    for (int h = 0; h < a.H; ++h) s = __fadd_rn(s, __fmul_rn(wrow[h], xrow[h]));
    if (a.bias && e < a.E) s = __fadd_rn(s, a.bias[e]);
    a.logits[idx] = s;
}

__global__ void route_rows_kernel(const RouterArgs a) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= a.T) return;
    route_row(a, warp, lane);
}

template <int TT, int WY, int WX, int KCH, int STG, int UNR, bool TF32>
static void launch_tile4(const RouterArgs& a, cudaStream_t s) {
    constexpr int TTc = TT * WY, EBc = 32 * WX;
    const size_t smem = sizeof(float) * STG * (EBc * (KCH + 4) + TTc * (KCH + 4));
    auto k = router_tile4_kernel<TT, WY, WX, KCH, STG, UNR, TF32>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 grid((a.T + TTc - 1) / TTc, (a.Ew + EBc - 1) / EBc);
    k<<<grid, 32 * WY * WX, smem, s>>>(a);
}

constexpr size_t kDecMaxSmem = 200 * 1024;
static size_t decode_router_smem(int H) { return sizeof(float) * ((size_t)kDecEB * (H + 16) + H); }

bool router_fits(int rows, int hidden, int order) {
    return order == kOrderSequential || rows >= 16 || decode_router_smem(hidden) <= kDecMaxSmem;
}

template <bool TF32>
static int launch_router_t(const RouterArgs& a, cudaStream_t s) {
    if (a.T < 16) {
        const size_t smem = decode_router_smem(a.H);
        if (smem > kDecMaxSmem) return -1;
        cudaFuncSetAttribute(router_decode_kernel<TF32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
        dim3 grid(a.T, (a.Ew + kDecEB - 1) / kDecEB);
        router_decode_kernel<TF32><<<grid, 128, smem, s>>>(a);
        return 0;
    }
    // logits, then one warp per token for the routing (a separate launch: the
    // routing tail of a fused last-CTA step cost more than the launch)
    // T <= 1024: CTAs of 8 tokens x 32 rows (two CTAs per SM) over 128-wide
    // chunks, measured ~2 us faster at T = 512 than 8 x 64 over 64-wide ones;
    // unrolling (4 steps at T = 512, none at T = 4096) measured 1.5 and 12 us
    // faster than the other choice (router + top-k 35.6 and 108.6 us)
    if (a.T <= 1024)
        launch_tile4<2, 4, 1, 128, 3, 4, TF32>(a, s);
    else
        launch_tile4<4, 4, 1, 64, 4, 1, TF32>(a, s);
    route_rows_kernel<<<(a.T * 32 + 255) / 256, 256, 0, s>>>(a);
    return 0;
}

int launch_router(const RouterArgs& args, cudaStream_t s) {
    RouterArgs a = args;
    if (a.Ew <= 0) a.Ew = a.E;
    if (a.order == kOrderSequential) {
        const long n = (long)a.T * a.Ew;
        router_sequential_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a);
        route_rows_kernel<<<(a.T * 32 + 255) / 256, 256, 0, s>>>(a);
        return 0;
    }
    return a.order == kOrderTf32 ? launch_router_t<true>(a, s) : launch_router_t<false>(a, s);
}

}  // namespace moe
