// Grouped expert GEMMs on the sm_100a tensor cores (tcgen05, kind::i8).
//
// Replaces the gate/up and down GEMMs of the reference's native MoE operator
// (rk_npu_moe_w8_run_f32, called at src/npu/moe.rs:372-386; arithmetic restated
// from llm_generated_docs/MINICPMV47_35A3_FUSED_MOE_20261019.md:77 and
// MOE_CPU_FUSION_20261023.md:12-13): exact INT32 accumulation of int8
// activations x int4/int8 weights, then dequantisation.
//
// Layout ("swap-AB"): the weight tile is the MMA's M=128 operand and the
// tokens of one expert are the N operand, so one TMEM lane = one output
// channel and TMEM columns = tokens. Small token counts (decode) then cost
// N=16 columns instead of a 128-row M tile, and each epilogue thread owns a
// channel whose per-group scale it loads once per group.
//
// Warp roles (320 threads):
//   warp 0      producer: bulk copies of pre-swizzled weight tiles + scales,
//               TMA tensor loads of the permuted activation rows
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 2..5  int4 -> int8 unpack into the 128B-swizzled operand buffer
//   warps 6..9  epilogue: tcgen05.ld, scale, SwiGLU / store
//
// Group-32 formats: one MMA (K = 32 = one group) per TMEM buffer, exact INT32
// per group, accumulated in fp32 by the epilogue as fma(acc_g, s_g, f).
// Per-channel formats: all of K accumulates in TMEM, one dequant per tile.
#include "kernels.cuh"

namespace moe {

constexpr int kGemmThreads = 320;
constexpr int kStages = 4;          // smem ring depth (k-blocks)
constexpr int kScaleStages = 8;     // group-scale ring depth (k-blocks)
constexpr int kTileRows = 128;      // weight rows per tile (MMA M)
constexpr int kKBlock = 128;        // K bytes per stage (one 128B swizzle row)

template <int FMT, int NT>
struct GemmCfg {
    static constexpr bool kW4 = (FMT == kFmtW4G32 || FMT == kFmtW4PC);
    static constexpr bool kGroup = (FMT == kFmtW4G32);
    static constexpr int kPackedBytes = kW4 ? kTileRows * kKBlock / 2 : 0;  // 8 KB
    static constexpr int kOperandBytes = kTileRows * kKBlock;               // 16 KB
    static constexpr int kActBytes = NT * kKBlock;
    static constexpr int kStageBytes = kOperandBytes + kActBytes + kPackedBytes;
    static constexpr int kScaleBytes = kGroup ? 4 * kTileRows * 2 : 0;     // 1 KB
    // TMEM buffers: groups in flight (group formats) or tile accumulators.
    static constexpr int kNBuf = kGroup ? ((512 / NT) < 16 ? (512 / NT) : 16) : 2;
    static constexpr int kCols = kNBuf * NT;
    static constexpr int kAllocCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128
                                    : kCols <= 256 ? 256 : 512;
    static constexpr int kXchgStride = NT + 1;
};

struct TileCoord {
    int e, rt, mt;
};

// Tile t -> (expert, weight row tile, token tile); token tile fastest so the
// CTAs sharing a weight tile run together and reuse it from L2.
__device__ __forceinline__ TileCoord decode_tile(int t, const int* tb, const int* tcnt, int E,
                                                 int row_tiles) {
    int lo = 0, hi = E - 1;  // last e with tb[e] <= t and a non-empty range
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (tb[mid] <= t) lo = mid; else hi = mid - 1;
    }
    // skip back over experts with no tiles that share the same start
    while (lo > 0 && tcnt[lo] == 0) --lo;
    TileCoord c;
    c.e = lo;
    const int local = t - tb[lo];
    c.rt = local / tcnt[lo];
    c.mt = local % tcnt[lo];
    return c;
}

template <int FMT, int EPI, int NT>
__global__ void __launch_bounds__(kGemmThreads, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap act_map, const GemmArgs a) {
    using C = GemmCfg<FMT, NT>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled operand buffers
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* op_w = smem;                                   // [S][16 KB]
    uint8_t* op_a = op_w + kStages * C::kOperandBytes;      // [S][NT*128]
    uint8_t* packed = op_a + kStages * C::kActBytes;        // [S][8 KB] (W4)
    uint8_t* scales = packed + kStages * C::kPackedBytes;   // [SS][1 KB] (group)
    float* xchg = reinterpret_cast<float*>(scales + kScaleStages * C::kScaleBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(xchg + 64 * C::kXchgStride + 2);
    uint64_t* full = bars;
    uint64_t* conv = full + kStages;
    uint64_t* empty = conv + kStages;
    uint64_t* sfull = empty + kStages;
    uint64_t* sempty = sfull + kScaleStages;
    uint64_t* tfull = sempty + kScaleStages;
    uint64_t* tempty = tfull + C::kNBuf;
    uint64_t* done = tempty + C::kNBuf;
    uint64_t* xfull = done + 1;   // up values written (2 warps)
    uint64_t* xempty = xfull + 1; // gate warps done reading (2 warps)
    int* tcnt = reinterpret_cast<int*>(xempty + 1);
    int* tb = tcnt + a.num_experts + 1;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;
    __shared__ int total_tiles_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = a.num_experts;

    if (threadIdx.x == 0) {
        abort_s = 0;
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&conv[i], 4);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kScaleStages; ++i) {
            mbar_init(&sfull[i], 1);
            mbar_init(&sempty[i], 4);
        }
        for (int i = 0; i < C::kNBuf; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 4);
        }
        mbar_init(done, 1);
        mbar_init(xfull, 2);
        mbar_init(xempty, 2);
        fence_barrier_init();
    }
    // tile table: tcnt[e] = token tiles of expert e, tb[e] = first tile index
    if (warp == 2) {
        const int per = (E + 31) / 32;
        int local = 0;
        for (int i = 0; i < per; ++i) {
            int e = lane * per + i;
            if (e < E) {
                int m = a.offsets[e + 1] - a.offsets[e];
                int c = (m + NT - 1) / NT;
                tcnt[e] = c;
                local += c;
            }
        }
        int incl = local;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += v;
        }
        int run = incl - local;
        for (int i = 0; i < per; ++i) {
            int e = lane * per + i;
            if (e < E) {
                tb[e] = run * a.row_tiles;
                run += tcnt[e];
            }
        }
        if (lane == 31) total_tiles_s = incl * a.row_tiles;
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base_s, C::kAllocCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) prefetch_tensormap(&act_map);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_s;
    const int total = total_tiles_s;
    volatile int* abort_flag = &abort_s;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                const TileCoord c = decode_tile(t, tb, tcnt, E, a.row_tiles);
                const int row0 = a.offsets[c.e] + c.mt * NT;
                const uint8_t* wtile = a.w + (size_t)c.e * a.w_expert_stride +
                                       (size_t)c.rt * a.w_tile_stride;
                for (int kb = 0; kb < a.kblocks && ok; ++kb, ++it) {
                    const int s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.err)) { ok = false; break; }
                    constexpr uint32_t wbytes = C::kW4 ? C::kPackedBytes : C::kOperandBytes;
                    mbar_arrive_expect_tx(&full[s], wbytes + C::kActBytes);
                    const uint8_t* wsrc = wtile + (size_t)kb * wbytes;
                    uint8_t* wdst = C::kW4 ? packed + s * C::kPackedBytes : op_w + s * C::kOperandBytes;
                    bulk_g2s(wdst, wsrc, wbytes, &full[s]);
                    tma_load_2d(op_a + s * C::kActBytes, &act_map, kb * kKBlock, row0, &full[s]);
                    if (C::kGroup) {
                        const int ss = it % kScaleStages;
                        const uint32_t sph = (it / kScaleStages) & 1u;
                        if (!mbar_wait(&sempty[ss], sph ^ 1u, abort_flag, a.err)) { ok = false; break; }
                        mbar_arrive_expect_tx(&sfull[ss], C::kScaleBytes);
                        const uint8_t* ssrc = reinterpret_cast<const uint8_t*>(a.wscale) +
                                              (size_t)c.e * a.ws_expert_stride +
                                              (size_t)c.rt * a.ws_tile_stride +
                                              (size_t)kb * C::kScaleBytes;
                        bulk_g2s(scales + ss * C::kScaleBytes, ssrc, C::kScaleBytes, &sfull[ss]);
                    }
                }
            }
            // drain: every issued fill must land before the CTA exits
            const uint32_t first = it > (uint32_t)kStages ? it - kStages : 0u;
            for (uint32_t d = first; d < it; ++d) {
                int dummy = 0;
                mbar_wait(&full[d % kStages], (d / kStages) & 1u, &dummy, a.err);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(kTileRows, NT);
            uint32_t it = 0, gi = 0, ti = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++ti) {
                uint32_t dcol = 0;
                if (!C::kGroup) {
                    const uint32_t buf = ti % 2u;
                    if (!mbar_wait(&tempty[buf], ((ti / 2u) & 1u) ^ 1u, abort_flag, a.err)) break;
                    tc_fence_after();
                    dcol = buf * NT;
                }
                for (int kb = 0; kb < a.kblocks && ok; ++kb, ++it) {
                    const int s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1u;
                    uint64_t* ready = C::kW4 ? &conv[s] : &full[s];
                    if (!mbar_wait(ready, ph, abort_flag, a.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t wa = smem_u32(op_w + s * C::kOperandBytes);
                    const uint32_t ab = smem_u32(op_a + s * C::kActBytes);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint64_t da = smem_desc_k_sw128(wa + 32 * j);
                        const uint64_t db = smem_desc_k_sw128(ab + 32 * j);
                        if (C::kGroup) {
                            const uint32_t buf = gi % C::kNBuf;
                            if (!mbar_wait(&tempty[buf], ((gi / C::kNBuf) & 1u) ^ 1u, abort_flag,
                                           a.err)) { ok = false; break; }
                            tc_fence_after();
                            mma_i8(tmem_base + buf * NT, da, db, idesc, 0u);
                            mma_commit(&tfull[buf]);
                            ++gi;
                        } else {
                            mma_i8(tmem_base + dcol, da, db, idesc, (kb > 0 || j > 0) ? 1u : 0u);
                        }
                    }
                    if (!ok) break;
                    mma_commit(&empty[s]);
                }
                if (!C::kGroup && ok) mma_commit(&tfull[ti % 2u]);
            }
            // all issued MMAs complete before TMEM can be released
            mma_commit(done);
            int dummy = 0;
            mbar_wait(done, 0, &dummy, a.err);
        }
    } else if (warp < 6) {
        // ------------------------------------------------------------ int4 unpack
        if (C::kW4) {
            const int ct = threadIdx.x - 64;  // 0..127
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                for (int kb = 0; kb < a.kblocks; ++kb, ++it) {
                    const int s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1u;
                    if (!mbar_wait(&full[s], ph, abort_flag, a.err)) { ok = false; break; }
                    const uint2* src = reinterpret_cast<const uint2*>(packed + s * C::kPackedBytes);
                    uint4* dst = reinterpret_cast<uint4*>(op_w + s * C::kOperandBytes);
#pragma unroll
                    for (int i = 0; i < C::kPackedBytes / 8 / 128; ++i) {
                        const int idx = ct + 128 * i;
                        const uint2 p = src[idx];
                        // packed byte b holds element b (low nibble) and b+4 (high
                        // nibble) of an 8-element run; each lands as 16 * value.
                        uint4 o;
                        o.x = (p.x << 4) & 0xF0F0F0F0u;
                        o.y = p.x & 0xF0F0F0F0u;
                        o.z = (p.y << 4) & 0xF0F0F0F0u;
                        o.w = p.y & 0xF0F0F0F0u;
                        dst[idx] = o;
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&conv[s]);
                }
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int quad = warp & 3;                 // TMEM lanes 32*quad ...
        const int r = quad * 32 + lane;            // weight row within the tile
        const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
        uint32_t gi = 0, ti = 0, it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++ti) {
            const TileCoord c = decode_tile(t, tb, tcnt, E, a.row_tiles);
            const int m_e = a.offsets[c.e + 1] - a.offsets[c.e];
            const int row0 = a.offsets[c.e] + c.mt * NT;
            const int nvalid = min(NT, m_e - c.mt * NT);
            const int nchunks = (nvalid + 7) / 8;
            // output channel of this lane
            int col;
            bool is_up = false;
            // gate/up tiles hold 64 gate rows then 64 up rows of the same channels
            const bool swiglu_tile = (EPI == kEpiSwiGLU) || (EPI == kEpiAcc && a.swiglu_layout);
            if (swiglu_tile) {
                is_up = r >= 64;
                col = c.rt * 64 + (r & 63);
            } else {
                col = c.rt * kTileRows + r;
            }
            const bool col_ok = col < a.n_valid;
            float facc[NT];
#pragma unroll
            for (int j = 0; j < NT; ++j) facc[j] = 0.0f;
            float wscale_pc = 0.0f;
            if (!C::kGroup) {
                const float* sp = reinterpret_cast<const float*>(
                    reinterpret_cast<const uint8_t*>(a.wscale) + (size_t)c.e * a.ws_expert_stride +
                    (size_t)c.rt * a.ws_tile_stride);
                wscale_pc = sp[r];
            }
            if (C::kGroup) {
                for (int kb = 0; kb < a.kblocks && ok; ++kb, ++it) {
                    const int ss = it % kScaleStages;
                    if (!mbar_wait(&sfull[ss], (it / kScaleStages) & 1u, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    const __half* sc = reinterpret_cast<const __half*>(scales + ss * C::kScaleBytes);
                    float sg[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) sg[j] = __half2float(sc[j * kTileRows + r]);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sempty[ss]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t buf = gi % C::kNBuf;
                        if (!mbar_wait(&tfull[buf], (gi / C::kNBuf) & 1u, abort_flag, a.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t taddr = tmem_base + lane_addr + buf * NT;
                        // W4 codes enter the MMA as 16*w: fold 1/16 into the scale (exact)
                        const float s_eff = C::kW4 ? sg[j] * 0.0625f : sg[j];
                        if (EPI == kEpiAcc) {
#pragma unroll
                            for (int ch = 0; ch < NT / 8; ++ch) {
                                if (ch < nchunks) {
                                    uint32_t v[8];
                                    tmem_ld8(taddr + ch * 8, v);
                                    tmem_wait_ld();
#pragma unroll
                                    for (int q = 0; q < 8; ++q) {
                                        const int jj = ch * 8 + q;
                                        if (jj < nvalid && col_ok) {
                                            int acc = (int)v[q];
                                            if (C::kW4) acc >>= 4;
                                            const int g = kb * 4 + j;
                                            const int ncol = is_up ? a.n_valid + col : col;
                                            a.acc_out[((size_t)(row0 + jj) * (a.kblocks * 4) + g) *
                                                          a.acc_ld + ncol] = acc;
                                        }
                                    }
                                }
                            }
                        } else {
#pragma unroll
                            for (int ch = 0; ch < NT / 8; ++ch) {
                                if (ch < nchunks) {
                                    uint32_t v[8];
                                    tmem_ld8(taddr + ch * 8, v);
                                    tmem_wait_ld();
#pragma unroll
                                    for (int q = 0; q < 8; ++q)
                                        facc[ch * 8 + q] = __fmaf_rn(
                                            __int2float_rn((int)v[q]), s_eff, facc[ch * 8 + q]);
                                }
                            }
                        }
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[buf]);
                        ++gi;
                    }
                }
                if (!ok) break;
            } else {
                const uint32_t buf = ti % 2u;
                if (!mbar_wait(&tfull[buf], (ti / 2u) & 1u, abort_flag, a.err)) break;
                tc_fence_after();
                const uint32_t taddr = tmem_base + lane_addr + buf * NT;
#pragma unroll
                for (int ch = 0; ch < NT / 8; ++ch) {
                    if (ch < nchunks) {
                        uint32_t v[8];
                        tmem_ld8(taddr + ch * 8, v);
                        tmem_wait_ld();
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            int acc = (int)v[q];
                            if (C::kW4) acc >>= 4;
                            if (EPI == kEpiAcc) {
                                const int jj = ch * 8 + q;
                                if (jj < nvalid && col_ok) {
                                    const int ncol = is_up ? a.n_valid + col : col;
                                    a.acc_out[(size_t)(row0 + jj) * a.acc_ld + ncol] = acc;
                                }
                            } else {
                                facc[ch * 8 + q] = __int2float_rn(acc);
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
            }
            if (EPI == kEpiAcc) continue;

            // dequantise with the per-token activation scale
            float val[NT];
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                if (j < nvalid) {
                    const float sx = a.act_scale[row0 + j];
                    if (C::kGroup)
                        val[j] = __fmul_rn(facc[j], sx);
                    else
                        val[j] = __fmul_rn(__fmul_rn(facc[j], sx), wscale_pc);
                } else {
                    val[j] = 0.0f;
                }
            }
            if (EPI == kEpiSwiGLU) {
                // exchange: up lanes (64..127) hand their values to gate lanes
                const uint32_t xph = ti & 1u;
                if (is_up) {
                    if (!mbar_wait(xempty, xph ^ 1u, abort_flag, a.err)) { ok = false; break; }
#pragma unroll
                    for (int j = 0; j < NT; ++j) xchg[(r - 64) * C::kXchgStride + j] = val[j];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xfull);
                } else {
                    if (!mbar_wait(xfull, xph, abort_flag, a.err)) { ok = false; break; }
#pragma unroll
                    for (int j = 0; j < NT; ++j) {
                        if (j < nvalid) {
                            const float gv = val[j];
                            const float uv = xchg[r * C::kXchgStride + j];
                            const float d = __fadd_rn(1.0f, expf(-gv));
                            const float m = __fmul_rn(__fdiv_rn(gv, d), uv);
                            float amax = col_ok ? fabsf(m) : 0.0f;
                            if (col_ok) a.out[(size_t)(row0 + j) * a.ldo + col] = m;
#pragma unroll
                            for (int off = 16; off > 0; off >>= 1)
                                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
                            if (lane == 0) atomicMax(&a.rowmax[row0 + j], __float_as_uint(amax));
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xempty);
                }
            } else {
                if (col_ok) {
#pragma unroll
                    for (int j = 0; j < NT; ++j)
                        if (j < nvalid) a.out[(size_t)(row0 + j) * a.ldo + col] = val[j];
                }
            }
        }
        if (!ok) *abort_flag = 1;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kAllocCols);
    }
}

template <int FMT, int EPI, int NT>
static size_t gemm_smem_bytes(int E) {
    using C = GemmCfg<FMT, NT>;
    size_t b = 1024;  // alignment slack
    b += (size_t)kStages * (C::kOperandBytes + C::kActBytes + C::kPackedBytes);
    b += (size_t)kScaleStages * C::kScaleBytes;
    b += sizeof(float) * (64 * C::kXchgStride + 2);
    b += sizeof(uint64_t) * (3 * kStages + 2 * kScaleStages + 2 * C::kNBuf + 3);
    b += sizeof(int) * (2 * (size_t)E + 2);
    // one CTA per SM: the kernel allocates TMEM up to 512 columns
    return b < 120 * 1024 ? 120 * 1024 : b;
}

template <int FMT, int EPI, int NT>
static int launch_gemm_t(const CUtensorMap& map, const GemmArgs& a, int num_sms,
                         cudaStream_t s) {
    const size_t smem = gemm_smem_bytes<FMT, EPI, NT>(a.num_experts);
    if (smem > 227 * 1024) return -1;
    cudaFuncSetAttribute(grouped_gemm_kernel<FMT, EPI, NT>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const long upper = ((long)(a.max_rows + NT - 1) / NT + a.num_experts) * a.row_tiles;
    const int grid = (int)(upper < num_sms ? (upper > 0 ? upper : 1) : num_sms);
    grouped_gemm_kernel<FMT, EPI, NT><<<grid, kGemmThreads, smem, s>>>(map, a);
    return 0;
}

template <int FMT, int EPI>
static int launch_gemm_nt(const CUtensorMap& map, const GemmArgs& a, int nt, int num_sms,
                          cudaStream_t s) {
    switch (nt) {
        case 16: return launch_gemm_t<FMT, EPI, 16>(map, a, num_sms, s);
        case 32: return launch_gemm_t<FMT, EPI, 32>(map, a, num_sms, s);
        case 64: return launch_gemm_t<FMT, EPI, 64>(map, a, num_sms, s);
        default: return -1;
    }
}

template <int FMT>
static int launch_gemm_epi(const CUtensorMap& map, const GemmArgs& a, int epi, int nt,
                           int num_sms, cudaStream_t s) {
    switch (epi) {
        case kEpiSwiGLU: return launch_gemm_nt<FMT, kEpiSwiGLU>(map, a, nt, num_sms, s);
        case kEpiStore: return launch_gemm_nt<FMT, kEpiStore>(map, a, nt, num_sms, s);
        case kEpiAcc: return launch_gemm_nt<FMT, kEpiAcc>(map, a, nt, num_sms, s);
        default: return -1;
    }
}

int launch_gemm(const CUtensorMap& map, const GemmArgs& a, int fmt, int epi, int nt,
                int num_sms, cudaStream_t s) {
    switch (fmt) {
        case kFmtW4G32: return launch_gemm_epi<kFmtW4G32>(map, a, epi, nt, num_sms, s);
        case kFmtW4PC: return launch_gemm_epi<kFmtW4PC>(map, a, epi, nt, num_sms, s);
        case kFmtW8PC: return launch_gemm_epi<kFmtW8PC>(map, a, epi, nt, num_sms, s);
        default: return -1;
    }
}

}  // namespace moe
