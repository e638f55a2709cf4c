// Routing device functions shared by the router kernels (router.cu) and the
// fused small-batch layer (gemv.cu): the NEON16 reduction of a logit dot, and
// the top-k (softmax) and grouped sigmoid selections of one row of logits.
// Reference semantics in router.cu's header.
#pragma once
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
__device__ inline void topk_row(const float* row, int E, int k, float min_weight, int32_t* ids,
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
__device__ inline void grouped_row(const float* row, const RouterArgs& a, int32_t* ids, float* weights,
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

}  // namespace moe
