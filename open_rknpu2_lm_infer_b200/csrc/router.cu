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

namespace moe {

// The 16 lanes of one (token, expert) dot live in 16 consecutive threads
// (j = tid & 15); reduce them with the fixed tree of vaddq/vaddvq:
// (l[j]+l[j+4]) + (l[j+8]+l[j+12]), then (v0+v1)+(v2+v3). Result in lane j=0.
__device__ __forceinline__ float neon16_tree(float v) {
    float s1 = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 16));   // a+b / c+d
    float s2 = __fadd_rn(s1, __shfl_down_sync(0xffffffffu, s1, 8, 16)); // (a+b)+(c+d)
    float p = __fadd_rn(s2, __shfl_down_sync(0xffffffffu, s2, 1, 16));  // v0+v1, v2+v3
    return __fadd_rn(p, __shfl_down_sync(0xffffffffu, p, 2, 16));       // total
}

template <bool TF32>
__device__ __forceinline__ float xval(float v) {
    return TF32 ? tf32_trunc(v) : v;
}

// Scalar tail (H % 16 elements, separately rounded products) and the logit
// bias (expert rows only).
template <bool TF32>
__device__ __forceinline__ float neon16_finish(float q, const float* wrow, const float* xrow,
                                               int H16, int H, const float* bias, int e, int E) {
    for (int h = H16; h < H; ++h) q = __fadd_rn(q, __fmul_rn(wrow[h], xval<TF32>(xrow[h])));
    if (bias && e < E) q = __fadd_rn(q, bias[e]);
    return q;
}

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
// element, and the 64 (or 32) chains per thread are independent. A warp =
// 4 lane groups q x 8 row groups s (rows s, s + 8, s + 16, s + 24 of the
// warp's 32); a CTA = WY x WX warps = WY*TT tokens x WX*32 rows. The hidden
// dimension streams in chunks of KCH through an STG-deep cp.async ring; row
// strides of KCH + 4 floats keep the 16-byte reads conflict-free. The fixed
// reduction tree of the reference's lanes, (l[c] + l[c+4]) + (l[c+8] +
// l[c+12]) then (v0 + v1) + (v2 + v3), pairs lane groups q ^ 1, then q ^ 2.
template <int TT, int WY, int WX, int KCH, int STG, bool TF32>
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

    float acc[TT][4][4];
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[t][m][c] = 0.0f;

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
#pragma unroll 1
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
                    acc[t][m][0] = __fmaf_rn(wv.x, xv[t].x, acc[t][m][0]);
                    acc[t][m][1] = __fmaf_rn(wv.y, xv[t].y, acc[t][m][1]);
                    acc[t][m][2] = __fmaf_rn(wv.z, xv[t].z, acc[t][m][2]);
                    acc[t][m][3] = __fmaf_rn(wv.w, xv[t].w, acc[t][m][3]);
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
    for (int t = 0; t < TT; ++t) {
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            float v[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float s1 = __fadd_rn(acc[t][m][c], __shfl_xor_sync(0xffffffffu, acc[t][m][c], 8));
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

// Rows of up to 256 logits: the row is read once into registers (one L2 round
// trip instead of one per round), then the same selection as topk_row.
__device__ __forceinline__ void topk_row_regs(const float* row, int E, int k, float min_weight,
                                              int32_t* ids, float* weights, int lane,
                                              uint32_t* err) {
    constexpr int kPL = 8;
    uint32_t key[kPL];
    float val[kPL];
    bool finite = true;
#pragma unroll
    for (int i = 0; i < kPL; ++i) {
        const int e = lane + 32 * i;
        val[i] = e < E ? __ldcg(row + e) : 0.0f;
        if (e < E && !isfinite(val[i])) finite = false;
        key[i] = (uint32_t)total_key(val[i]) ^ 0x80000000u;
    }
    if (__any_sync(0xffffffffu, !finite) && lane == 0) atomicOr(err, kErrNonFinite);
    uint32_t taken = 0;
    int my_id = -1;
    float my_val = 0.0f, top_val = 0.0f;
    for (int r = 0; r < k; ++r) {
        unsigned long long best = 0ull;
#pragma unroll
        for (int i = 0; i < kPL; ++i) {
            const int e = lane + 32 * i;
            if (e >= E || ((taken >> i) & 1u)) continue;
            const unsigned long long v = ((unsigned long long)key[i] << 32) | (0xFFFFFFFFu - (uint32_t)e);
            if (v > best) best = v;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
            if (o > best) best = o;
        }
        const int win = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
        const float wv = key_value((int32_t)((uint32_t)(best >> 32) ^ 0x80000000u));
        if ((win & 31) == lane) taken |= 1u << (win >> 5);
        if (lane == r) { my_id = win; my_val = wv; }
        if (r == 0) top_val = wv;
    }
    float w = 0.0f;
    if (lane < k) w = expf(__fsub_rn(my_val, top_val));
    float sum = -0.0f;
    for (int r = 0; r < k; ++r) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, w, r));
    if (lane < k) {
        w = __fdiv_rn(w, sum);
        if (min_weight != 0.0f && lane >= 1 && w < min_weight) w = 0.0f;
        ids[lane] = my_id;
        weights[lane] = w;
    }
}

// One warp selects the top-k of a row of E logits (E <= 1024): k rounds of a
// warp arg-max over (total_cmp key, -id), then softmax over the selected.
__device__ void topk_row(const float* row, int E, int k, float min_weight, int32_t* ids,
                         float* weights, int lane, uint32_t* err) {
    if (E <= 256) {
        topk_row_regs(row, E, k, min_weight, ids, weights, lane, err);
        return;
    }
    uint32_t taken = 0;  // bit i: element lane + 32*i already selected
    const int per_lane = (E + 31) / 32;
    int my_id = -1;
    bool finite = true;
    for (int i = 0; i < per_lane; ++i) {
        int e = lane + 32 * i;
        if (e < E && !isfinite(__ldcg(row + e))) finite = false;
    }
    if (__any_sync(0xffffffffu, !finite) && lane == 0) atomicOr(err, kErrNonFinite);
    for (int r = 0; r < k; ++r) {
        unsigned long long best = 0ull;
        for (int i = 0; i < per_lane; ++i) {
            int e = lane + 32 * i;
            if (e >= E || (taken >> i) & 1u) continue;
            uint32_t key = (uint32_t)total_key(__ldcg(row + e)) ^ 0x80000000u;
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
    const float mx = __ldcg(row + id0);
    float w = 0.0f;
    if (lane < k) w = expf(__fsub_rn(__ldcg(row + my_id), mx));
    float sum = -0.0f;
    for (int r = 0; r < k; ++r) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, w, r));
    if (lane < k) {
        w = __fdiv_rn(w, sum);
        if (min_weight != 0.0f && lane >= 1 && w < min_weight) w = 0.0f;
        ids[lane] = my_id;
        weights[lane] = w;
    }
}

// Ling's grouped sigmoid routing for one row, one warp (E <= 256: element
// lane + 32i of the row in sel[i]). Keys are total_cmp keys made unsigned
// (key ^ 0x80000000), so an unsigned compare is the f32 total order; 0 stands
// for "no element" in the top-2 merges (every group has >= 2 elements).
__device__ void grouped_row(const float* row, const RouterArgs& a, int32_t* ids, float* weights,
                            int lane) {
    constexpr int kPL = kGroupedMaxExperts / 32;
    const int E = a.E, k = a.k, width = E / a.groups;
    uint32_t key[kPL];
    bool finite = true;
#pragma unroll
    for (int i = 0; i < kPL; ++i) {
        const int e = lane + 32 * i;
        key[i] = 0u;
        if (e < E) {
            const float l = __ldcg(row + e);
            if (!isfinite(l)) finite = false;
            // selected = score + bias (moe.rs:165-168)
            const float sel = __fadd_rn(sigmoid_ref(l), a.sel_bias[e]);
            key[i] = (uint32_t)total_key(sel) ^ 0x80000000u;
        }
    }
    if (__any_sync(0xffffffffu, !finite) && lane == 0) atomicOr(a.err, kErrNonFinite);

    // group score = the sum of the group's two largest selected values
    // (moe.rs:170-187); lane g keeps group g's
    uint32_t my_gkey = 0u;
    for (int g = 0; g < a.groups; ++g) {
        uint32_t f = 0u, s2 = 0u;
#pragma unroll
        for (int i = 0; i < kPL; ++i) {
            const int e = lane + 32 * i;
            if (e < E && e / width == g) {
                const uint32_t v = key[i];
                if (v > f) { s2 = f; f = v; }
                else if (v > s2) s2 = v;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const uint32_t of = __shfl_xor_sync(0xffffffffu, f, off);
            const uint32_t os = __shfl_xor_sync(0xffffffffu, s2, off);
            s2 = max(min(f, of), max(s2, os));
            f = max(f, of);
        }
        const float gs = __fadd_rn(key_value((int32_t)(f ^ 0x80000000u)),
                                   key_value((int32_t)(s2 ^ 0x80000000u)));
        if (lane == g) my_gkey = (uint32_t)total_key(gs) ^ 0x80000000u;
    }
    // the top_groups groups of (score desc, index asc) (moe.rs:188-198)
    int rank = 0;
    for (int h = 0; h < a.groups; ++h) {
        const uint32_t hk = __shfl_sync(0xffffffffu, my_gkey, h);
        if (hk > my_gkey || (hk == my_gkey && h < lane)) ++rank;
    }
    const uint32_t enabled = __ballot_sync(0xffffffffu, lane < a.groups && rank < a.top_groups);

    // the first k of (selected desc, id asc) among the enabled groups' experts
    // (moe.rs:199-210)
    uint32_t taken = 0;
    int my_id = 0;
    for (int r = 0; r < k; ++r) {
        unsigned long long best = 0ull;
#pragma unroll
        for (int i = 0; i < kPL; ++i) {
            const int e = lane + 32 * i;
            if (e >= E || ((taken >> i) & 1u) || !((enabled >> (e / width)) & 1u)) continue;
            const unsigned long long v =
                ((unsigned long long)key[i] << 32) | (0xFFFFFFFFu - (uint32_t)e);
            if (v > best) best = v;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
            if (o > best) best = o;
        }
        const int win = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
        if ((win & 31) == lane) taken |= 1u << (win >> 5);
        if (lane == r) my_id = win;
    }
    // weights from the unbiased sigmoid, summed in chosen order (moe.rs:211-221)
    const float score = lane < k ? sigmoid_ref(__ldcg(row + my_id)) : 0.0f;
    float sum = -0.0f;
    for (int r = 0; r < k; ++r) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, score, r));
    sum = __fadd_rn(sum, 1e-20f);
    if (lane < k) {
        const float w = k > 1 ? __fdiv_rn(score, sum) : score;
        ids[lane] = my_id;
        weights[lane] = __fmul_rn(w, a.scale);
    }
}

template <int TT, int WY, int WX, int KCH, int STG, bool TF32>
static void launch_tile4(const RouterArgs& a, cudaStream_t s) {
    constexpr int TTc = TT * WY, EBc = 32 * WX;
    const size_t smem = sizeof(float) * STG * (EBc * (KCH + 4) + TTc * (KCH + 4));
    auto k = router_tile4_kernel<TT, WY, WX, KCH, STG, TF32>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 grid((a.T + TTc - 1) / TTc, (a.Ew + EBc - 1) / EBc);
    k<<<grid, 32 * WY * WX, smem, s>>>(a);
}

template <bool TF32>
static int launch_router_t(const RouterArgs& a, cudaStream_t s) {
    if (a.T < 16) {
        const size_t smem = sizeof(float) * ((size_t)kDecEB * (a.H + 16) + a.H);
        if (smem > 200 * 1024) return -1;
        cudaFuncSetAttribute(router_decode_kernel<TF32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
        dim3 grid(a.T, (a.Ew + kDecEB - 1) / kDecEB);
        router_decode_kernel<TF32><<<grid, 128, smem, s>>>(a);
        return 0;
    }
    // logits, then one warp per token for the routing (a separate launch: the
    // routing tail of a fused last-CTA step cost more than the launch)
    // T <= 1024: CTAs of 8 tokens x 32 rows (two CTAs per SM) over 128-wide
    // chunks, measured ~2 us faster at T = 512 than 8 x 64 over 64-wide ones
    if (a.T <= 1024)
        launch_tile4<2, 4, 1, 128, 3, TF32>(a, s);
    else
        launch_tile4<4, 4, 1, 64, 4, TF32>(a, s);
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
