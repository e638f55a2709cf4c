// Token dispatch and the element-wise stages around the expert GEMMs:
//   route_count / route_scatter : stable grouping of assignments by expert
//   quant_gather                : dynamic per-token int8 quantisation, written
//                                 straight into the permuted GEMM operand
//   requant                     : gate | up -> SwiGLU middle -> int8 for the down GEMM
//   combine                     : routing-weighted sum (+ shared, + residual)
//
// Reference semantics (happyme531/open_rknpu2_lm_infer):
//   grouping   : assignment order t*k+r inside an expert group, zero routes
//                skipped (src/model/experts/paged.rs:586-600)
//   quantise   : MoE rule s = maxabs/127, round-half-even, zero row -> s = 1
//                (llm_generated_docs/MOE_CPU_FUSION_20261023.md:13); dense rule
//                s = max(maxabs/127, FLT_MIN), round-half-away of x * (1/s)
//                (llm_generated_docs/MODELS.md:26)
//   combine    : out = sum_r fma(y, w_r, out) over ranks with w > 0
//                (src/model/experts/paged.rs:495-506), then + shared
//                (src/model/ling3tiny/moe.rs:378-388), then residual + out
//                (src/model/qwen35/decoder.rs:215-217)
#include <float.h>

#include <algorithm>

#include "kernels.cuh"
#include "quant.cuh"

namespace moe {

__device__ __forceinline__ bool route_kept(float w) { return w > 0.0f; }

// The kernels of this file launch as programmatic dependents of the kernel
// before them on the stream: their launch overlaps that kernel's last CTAs,
// and each waits (pdl_wait, first thing) for it to complete before reading
// anything.
template <typename... KArgs, typename... Args>
static void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Keys: id / div for ids in [0, id_limit) (div = 1: the expert; div = experts
// per rank: the destination rank of expert parallelism). routes == nullptr:
// every assignment is kept.
__global__ void route_count_kernel(const int32_t* __restrict__ ids, const float* __restrict__ routes,
                                   int n, int E, int id_limit, int div, int32_t* hist,
                                   uint32_t* err) {
    pdl_wait();
    extern __shared__ int32_t hist_s[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist_s[e] = 0;
    __syncthreads();
    const int a0 = blockIdx.x * kRouteChunk;
    const int a1 = min(n, a0 + kRouteChunk);
    for (int a = a0 + threadIdx.x; a < a1; a += blockDim.x) {
        const float w = routes ? routes[a] : 1.0f;
        if (!(w >= 0.0f)) atomicOr(err, kErrBadRoute);  // negative or NaN
        if (!route_kept(w)) continue;
        const int id = ids[a];
        if (id < 0 || id >= id_limit) {
            atomicOr(err, kErrBadExpert);
            continue;
        }
        atomicAdd(&hist_s[id / div], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[(size_t)blockIdx.x * E + e] = hist_s[e];
}

// 256 threads. smem: off[E+1], base[E], wcnt[8][E].
__global__ void __launch_bounds__(256)
route_scatter_kernel(const int32_t* __restrict__ ids, const float* __restrict__ routes, int n,
                     int E, int id_limit, int div, const int32_t* __restrict__ hist,
                     int32_t* offsets, int32_t* perm, int32_t* pos, int32_t* shared_offsets,
                     int T) {
    pdl_wait();
    extern __shared__ int32_t sm[];
    int32_t* off_s = sm;               // E+1
    int32_t* base_s = off_s + E + 1;   // E
    int32_t* wcnt = base_s + E;        // 8*E
    const int nb = gridDim.x, b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int tot = 0, pre = 0;
        for (int bb = 0; bb < nb; ++bb) {
            const int h = hist[(size_t)bb * E + e];
            tot += h;
            if (bb < b) pre += h;
        }
        off_s[e] = tot;  // scanned below
        base_s[e] = pre;
    }
    for (int i = threadIdx.x; i < 8 * E; i += blockDim.x) wcnt[i] = 0;
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the expert totals
        const int per = (E + 31) / 32;
        int local = 0;
        for (int i = 0; i < per; ++i) {
            const int e = lane * per + i;
            if (e < E) local += off_s[e];
        }
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - local;
        for (int i = 0; i < per; ++i) {
            const int e = lane * per + i;
            if (e < E) {
                const int c = off_s[e];
                off_s[e] = run;
                run += c;
            }
        }
        if (lane == 31) off_s[E] = incl;
    }
    __syncthreads();
    if (b == 0) {
        for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets[e] = off_s[e];
        if (shared_offsets && threadIdx.x == 0) {
            shared_offsets[0] = 0;
            shared_offsets[1] = T;
        }
    }
    const int a0 = b * kRouteChunk;
    const int a1 = min(n, a0 + kRouteChunk);
    const unsigned lt = (1u << lane) - 1u;
    for (int r0 = a0; r0 < a1; r0 += blockDim.x) {
        const int a = r0 + threadIdx.x;
        int e = -1;
        if (a < a1) {
            const float w = routes ? routes[a] : 1.0f;
            const int id = ids[a];
            if (route_kept(w) && id >= 0 && id < id_limit) e = id / div;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank_w = __popc(peers & lt);
        if (e >= 0 && rank_w == 0) wcnt[warp * E + e] = __popc(peers);
        __syncthreads();
        if (a < a1) {
            if (e >= 0) {
                int before = 0;
                for (int w2 = 0; w2 < warp; ++w2) before += wcnt[w2 * E + e];
                const int p = off_s[e] + base_s[e] + before + rank_w;
                perm[p] = a;
                pos[a] = p;
            } else {
                pos[a] = -1;
            }
        }
        __syncthreads();
        for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
            int s = 0;
            for (int w2 = 0; w2 < 8; ++w2) {
                s += wcnt[w2 * E + ee];
                wcnt[w2 * E + ee] = 0;
            }
            base_s[ee] += s;
        }
        __syncthreads();
    }
}

// Block-wide max of non-negative values (blockDim.x a multiple of 32, <= 1024).
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = red[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
    return m;
}

// One CTA (256 threads) per token: the row is read once into registers
// (V float4 per thread), quantised, and written to q_rows[t] (if given) and
// to every kept permuted slot pos[t*k + r] (if pos given). The padding
// columns of the destinations stay as created (zero). Needs H % 4 == 0.
template <int V>
__global__ void __launch_bounds__(256)
quant_gather_kernel(const float* __restrict__ x, int H, int ld_q, int rule, int k,
                    const int32_t* __restrict__ pos, int8_t* q_rows, float* s_rows,
                    int8_t* q_perm, float* s_perm, __half* h_rows, __half* h_perm, uint32_t* err) {
    pdl_wait();
    __shared__ float red[8];
    __shared__ int slots[32];
    __shared__ int nslot_s;
    const int t = blockIdx.x;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)t * H);
    const int n4 = H / 4;
    float4 v[V];
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = threadIdx.x + 256 * i;
        v[i] = c < n4 ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        m = fmaxf(m, amax4(v[i]));
    }
    if (threadIdx.x == 0) {
        int ns = 0;
        if (pos)
            for (int r = 0; r < k && r < 32; ++r) {
                const int p = pos[(size_t)t * k + r];
                if (p >= 0) slots[ns++] = p;
            }
        nslot_s = ns;
    }
    m = block_max(m, red);  // includes a __syncthreads: slots are visible after it
    const float s = row_scale(m, rule);
    const float inv = __fdiv_rn(1.0f, s);
    const int nslot = nslot_s;
    if (threadIdx.x == 0) {
        if (!isfinite(s)) atomicOr(err, kErrNonFinite);
        if (s_rows) s_rows[t] = s;
        for (int i = 0; i < nslot; ++i) s_perm[slots[i]] = s;
    }
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = threadIdx.x + 256 * i;
        if (c < n4) {
            const uint32_t packed = quant4(v[i], s, inv, rule);
            if (q_rows) reinterpret_cast<uint32_t*>(q_rows + (size_t)t * ld_q)[c] = packed;
            for (int j = 0; j < nslot; ++j)
                reinterpret_cast<uint32_t*>(q_perm + (size_t)slots[j] * ld_q)[c] = packed;
            if (h_rows || h_perm) {
                const uint2 h = codes_to_half4(packed);
                if (h_rows) reinterpret_cast<uint2*>(h_rows + (size_t)t * ld_q)[c] = h;
                if (h_perm)
                    for (int j = 0; j < nslot; ++j)
                        reinterpret_cast<uint2*>(h_perm + (size_t)slots[j] * ld_q)[c] = h;
            }
        }
    }
}

// One CTA (128 threads) per permuted row; rows >= *count exit. Reads the row's
// gate | up halves once (V float4 of each per thread), applies SwiGLU, takes
// the max |h|, quantises.
template <int V>
__global__ void __launch_bounds__(128)
requant_kernel(const float* __restrict__ gate_up, const int32_t* __restrict__ count, int I,
               int ld_q, int rule, int8_t* q, __half* qh, float* sc) {
    pdl_wait();
    __shared__ float red[4];
    const int row = blockIdx.x;
    if (row >= *count) return;
    const float4* gr = reinterpret_cast<const float4*>(gate_up + (size_t)row * 2 * I);
    const float4* ur = reinterpret_cast<const float4*>(gate_up + (size_t)row * 2 * I + I);
    const int n4 = I / 4;
    float4 v[V];
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = threadIdx.x + 128 * i;
        if (c < n4) {
            const float4 g = gr[c], u = ur[c];
            v[i] = make_float4(silu_mul(g.x, u.x), silu_mul(g.y, u.y), silu_mul(g.z, u.z),
                               silu_mul(g.w, u.w));
        } else {
            v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        m = fmaxf(m, amax4(v[i]));
    }
    m = block_max(m, red);
    const float s = row_scale(m, rule);
    const float inv = __fdiv_rn(1.0f, s);
    if (threadIdx.x == 0) sc[row] = s;
    uint32_t* qr = reinterpret_cast<uint32_t*>(q + (size_t)row * ld_q);
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c = threadIdx.x + 128 * i;
        if (c < n4) {
            const uint32_t packed = quant4(v[i], s, inv, rule);
            qr[c] = packed;
            if (qh) reinterpret_cast<uint2*>(qh + (size_t)row * ld_q)[c] = codes_to_half4(packed);
        }
    }
}

// One CTA (256 threads) per token, float4 columns (H % 4 == 0). With a shared
// gate the shared row enters as projected += scale * shared, scale =
// 1 / (1 + exp(-gate)) (src/model/qwen35/moe.rs:334-347, two roundings).
__global__ void __launch_bounds__(256)
combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ pos,
               const float* __restrict__ routes, const float* __restrict__ shared,
               const float* __restrict__ residual, int H, int k, float* out,
               const float* __restrict__ gate, int gate_ld) {
    pdl_wait();
    __shared__ int ps[32];
    __shared__ float ws[32];
    __shared__ float gscale;
    const int t = blockIdx.x;
    if (gate && threadIdx.x == 32)
        gscale = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f32(-gate[(size_t)t * gate_ld])));
    if (threadIdx.x < k) {
        const size_t a = (size_t)t * k + threadIdx.x;
        const float w = routes[a];
        ws[threadIdx.x] = route_kept(w) ? w : 0.0f;
        ps[threadIdx.x] = route_kept(w) ? pos[a] : -1;
    }
    __syncthreads();
    const int n4 = H / 4;
    for (int c = threadIdx.x; c < n4; c += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < k; ++r) {
            const int p = ps[r];
            if (p < 0) continue;
            const float w = ws[r];
            const float4 yv = reinterpret_cast<const float4*>(y + (size_t)p * H)[c];
            acc.x = __fmaf_rn(yv.x, w, acc.x);
            acc.y = __fmaf_rn(yv.y, w, acc.y);
            acc.z = __fmaf_rn(yv.z, w, acc.z);
            acc.w = __fmaf_rn(yv.w, w, acc.w);
        }
        if (shared) {
            float4 sv = reinterpret_cast<const float4*>(shared + (size_t)t * H)[c];
            if (gate) {
                sv.x = __fmul_rn(gscale, sv.x);
                sv.y = __fmul_rn(gscale, sv.y);
                sv.z = __fmul_rn(gscale, sv.z);
                sv.w = __fmul_rn(gscale, sv.w);
            }
            acc.x = __fadd_rn(acc.x, sv.x);
            acc.y = __fadd_rn(acc.y, sv.y);
            acc.z = __fadd_rn(acc.z, sv.z);
            acc.w = __fadd_rn(acc.w, sv.w);
        }
        if (residual) {
            const float4 rv = reinterpret_cast<const float4*>(residual + (size_t)t * H)[c];
            acc.x = __fadd_rn(rv.x, acc.x);
            acc.y = __fadd_rn(rv.y, acc.y);
            acc.z = __fadd_rn(rv.z, acc.z);
            acc.w = __fadd_rn(rv.w, acc.w);
        }
        reinterpret_cast<float4*>(out + (size_t)t * H)[c] = acc;
    }
}

void launch_route_count(const int32_t* ids, const float* routes, int n, int E, int32_t* hist,
                        uint32_t* err, cudaStream_t s, int id_limit, int div) {
    const int nb = (n + kRouteChunk - 1) / kRouteChunk;
    if (nb == 0) return;
    launch_pdl(route_count_kernel, dim3(nb), dim3(256), sizeof(int32_t) * E, s, ids, routes, n, E,
               id_limit > 0 ? id_limit : E, div, hist, err);
}

void launch_route_scatter(const int32_t* ids, const float* routes, int n, int E,
                          const int32_t* hist, int32_t* offsets, int32_t* perm, int32_t* pos,
                          int32_t* shared_offsets, int T, cudaStream_t s, int id_limit, int div) {
    const int nb = (n + kRouteChunk - 1) / kRouteChunk;
    const size_t smem = sizeof(int32_t) * (size_t)(E + 1 + E + 8 * E);
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(route_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    launch_pdl(route_scatter_kernel, dim3(nb > 0 ? nb : 1), dim3(256), smem, s, ids, routes, n, E,
               id_limit > 0 ? id_limit : E, div, hist, offsets, perm, pos, shared_offsets, T);
}

// Expert parallelism: the destination-local expert id of each packed row.
__global__ void ep_expert_ids_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ pos,
                                     int n, int per_rank, int32_t* send_expert) {
    const int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n) return;
    const int p = pos[a];
    if (p >= 0) send_expert[p] = ids[a] % per_rank;
}

void launch_ep_expert_ids(const int32_t* ids, const int32_t* pos, int n, int per_rank,
                          int32_t* send_expert, cudaStream_t s) {
    if (n == 0) return;
    ep_expert_ids_kernel<<<(n + 255) / 256, 256, 0, s>>>(ids, pos, n, per_rank, send_expert);
}

// Rows per destination rank from the grouping offsets.
__global__ void ep_counts_kernel(const int32_t* __restrict__ offsets, int world, int32_t* counts) {
    for (int g = threadIdx.x; g < world; g += blockDim.x) counts[g] = offsets[g + 1] - offsets[g];
}

void launch_ep_counts(const int32_t* offsets, int world, int32_t* counts, cudaStream_t s) {
    ep_counts_kernel<<<1, 256, 0, s>>>(offsets, world, counts);
}

// Received rows -> permuted order: row i (ld bytes) to slot pos[i], its scale too.
__global__ void ep_gather_rows_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                      const int32_t* __restrict__ pos, int ld, int8_t* q_perm,
                                      float* s_perm) {
    const int i = blockIdx.x;
    const int p = pos[i];
    if (p < 0) return;
    const uint4* src = reinterpret_cast<const uint4*>(q + (size_t)i * ld);
    uint4* dst = reinterpret_cast<uint4*>(q_perm + (size_t)p * ld);
    for (int c = threadIdx.x; c < ld / 16; c += blockDim.x) dst[c] = src[c];
    if (threadIdx.x == 0) s_perm[p] = scale[i];
}

void launch_ep_gather_rows(const int8_t* q, const float* scale, const int32_t* pos, int n, int ld,
                           int8_t* q_perm, float* s_perm, cudaStream_t s) {
    if (n == 0) return;
    ep_gather_rows_kernel<<<n, 128, 0, s>>>(q, scale, pos, ld, q_perm, s_perm);
}

__global__ void set_range_kernel(int32_t* offsets, int rows) {
    offsets[0] = 0;
    offsets[1] = rows;
}

void launch_set_range(int32_t* offsets, int rows, cudaStream_t s) {
    set_range_kernel<<<1, 1, 0, s>>>(offsets, rows);
}

void launch_quant_gather(const float* x, int T, int H, int ld_q, int rule, int k,
                         const int32_t* pos, int8_t* q_rows, float* s_rows, int8_t* q_perm,
                         float* s_perm, __half* h_rows, __half* h_perm, uint32_t* err,
                         cudaStream_t s) {
    if (T == 0) return;
    const int v = (H / 4 + 255) / 256;
#define QG(V) launch_pdl(quant_gather_kernel<V>, dim3(T), dim3(256), 0, s, x, H, ld_q, rule, k, pos, q_rows, s_rows, q_perm, s_perm, h_rows, h_perm, err)
    if (v <= 1) QG(1);
    else if (v <= 2) QG(2);
    else if (v <= 4) QG(4);
    else QG(8);
#undef QG
}

void launch_requant(const float* gate_up, const int32_t* count, int max_rows, int I, int ld_q,
                    int rule, int8_t* q, __half* qh, float* sc, cudaStream_t s) {
    if (max_rows == 0) return;
    const int v = (I / 4 + 127) / 128;
#define RQ(V) launch_pdl(requant_kernel<V>, dim3(max_rows), dim3(128), 0, s, gate_up, count, I, ld_q, rule, q, qh, sc)
    if (v <= 1) RQ(1);
    else if (v <= 2) RQ(2);
    else if (v <= 4) RQ(4);
    else if (v <= 8) RQ(8);
    else RQ(16);
#undef RQ
}

__global__ void swap_bytes_kernel(uint4* __restrict__ a, uint4* __restrict__ b, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const uint4 x = a[i];
        a[i] = b[i];
        b[i] = x;
    }
}

void launch_swap_bytes(void* a, void* b, size_t bytes, cudaStream_t s) {
    const size_t n = bytes / 16;
    if (n == 0) return;
    const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 8);
    swap_bytes_kernel<<<blocks, 256, 0, s>>>(static_cast<uint4*>(a), static_cast<uint4*>(b), n);
}

void launch_combine(const float* y, const int32_t* pos, const float* routes, const float* shared,
                    const float* residual, int T, int H, int k, float* out, cudaStream_t s,
                    const float* gate, int gate_ld) {
    if (T == 0) return;
    launch_pdl(combine_kernel, dim3(T), dim3(256), 0, s, y, pos, routes, shared, residual, H, k, out,
               shared ? gate : nullptr, gate_ld);
}

}  // namespace moe
