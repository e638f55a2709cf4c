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
// channel and TMEM columns = tokens. Small token counts (decode) cost N=16
// columns instead of a 128-row M tile, and each epilogue thread owns a
// channel whose per-group scale it reads once per group.
//
// Warp roles (704 threads):
//   warp 0       producer: per load stage (kKPS k-blocks) one bulk copy of the
//                weight blocks (+ group scales) and one 3-D TMA copy of the
//                permuted activation rows. A copy request costs ~0.2 us per SM
//                whatever its size, so a stage moves >= 16 KB per request.
//   warp 1       TMEM allocator + single-thread MMA issuer
//   warps 2..5   W4 formats: unpack int4 -> int8 straight into tensor memory,
//                one warp per TMEM lane quadrant, one weight row per thread;
//                the MMA then reads its weight operand from TMEM (no shared
//                memory operand, no proxy fence). W8: idle.
//   warps 6..21  epilogue, four warps per TMEM lane quadrant, each owning a
//                quarter of the token columns (the epilogue is latency-bound,
//                so it gets the most warps)
//
// Group-32 formats: one MMA (K = 32 = one group) per TMEM buffer; the four
// buffers of a k-block form a slot. Every buffer is pre-filled with the bits
// of 12582912.0f (0x4B400000) and the MMA accumulates into it, so the int32
// result read back as a float is exactly 12582912 + 16*acc (|16*acc| < 2^22).
// The epilogue computes f = fma(D - 12582912, s/16, f): an exact subtraction
// and one FMA, equal to fma((float)acc, s, f) bit for bit, without an
// int->float conversion. Per-channel formats: all of K accumulates in TMEM,
// one dequant per tile.
#include "kernels.cuh"

namespace moe {

constexpr int kGemmThreads = 704;
constexpr int kConvWarp0 = 2;         // first unpack warp
constexpr int kConvWarps = 4;
constexpr int kEpiWarp0 = 6;          // first epilogue warp
constexpr int kEpiWarps = 16;
constexpr int kScaleStages = 8;       // group-scale ring depth (k-blocks)
constexpr int kTileRows = 128;        // weight rows per tile (MMA M)
constexpr int kKBlock = 128;          // K bytes per k-block (one 128B swizzle row)
constexpr uint32_t kMagicBits = 0x4B400000u;  // 12582912.0f
constexpr float kMagic = 12582912.0f;

template <int FMT, int NT>
struct GemmCfg {
    static constexpr bool kW4 = (FMT == kFmtW4G32 || FMT == kFmtW4PC);
    static constexpr bool kGroup = (FMT == kFmtW4G32);
    static constexpr int kWBytes = kW4 ? kTileRows * kKBlock / 2 : kTileRows * kKBlock;
    static constexpr int kScaleBytes = kGroup ? 4 * kTileRows * 2 : 0;  // 1 KB per k-block
    static constexpr int kActBytes = NT * kKBlock;           // per k-block
    // weight request of one stage (HBM layout: kKPS weight blocks, then their scales)
    static constexpr int kStageW = kKPS * (kWBytes + kScaleBytes);
    // load stage: [activations kKPS x NT x 128][weights (+ scales)]; W8 weights
    // are the MMA operand tiles, W4 weights are unpacked into TMEM.
    static constexpr int kLoadBytes = kKPS * kActBytes + kStageW;
    // TMEM: [W4 weight operand ring: kLoadStages x kKPS x 32 columns][accumulators]
    static constexpr int kACols = 32;                        // one k-block of int8 weights
    static constexpr int kLoadStages = kW4 ? 4 : ((200 * 1024) / kLoadBytes >= 6 ? 6
                                                  : (200 * 1024) / kLoadBytes);
    static constexpr int kARegion = kW4 ? kLoadStages * kKPS * kACols : 0;
    // group formats: slots of one k-block (4 group buffers of NT columns);
    // per-channel formats: two tile accumulators.
    static constexpr int kSlotCols = kGroup ? 4 * NT : NT;
    static constexpr int kAccFree = 512 - kARegion;
    static constexpr int kNSlot = kGroup ? ((kAccFree / kSlotCols) < 4 ? (kAccFree / kSlotCols) : 4)
                                         : 2;
    static constexpr int kAllocCols = 512;
    static constexpr int kHalf = NT / 4;                      // columns per epilogue warp
    static constexpr int kXchgStride = NT + 1;
    static_assert(kLoadStages >= 2, "smem budget");
    static_assert(kNSlot >= 2, "TMEM budget: group formats need NT <= 32");
    static_assert(kARegion + kNSlot * kSlotCols <= 512, "TMEM budget");
};

struct TileCoord {
    int e, rt, mt;
};

// Tile t -> (expert, weight row tile, token tile); token tile fastest so the
// CTAs sharing a weight tile run together and reuse it from L2.
__device__ __forceinline__ TileCoord decode_tile(int t, const int* tb, const int* tcnt, int E) {
    int lo = 0, hi = E - 1;  // last e with tb[e] <= t (that expert is non-empty)
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (tb[mid] <= t) lo = mid; else hi = mid - 1;
    }
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
    constexpr int SL = C::kLoadStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* load = smem;
    uint8_t* scales = load + SL * C::kLoadBytes;              // [SS][1 KB] (group)
    float* xchg = reinterpret_cast<float*>(scales + kScaleStages * C::kScaleBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(xchg + 64 * C::kXchgStride + 2);
    uint64_t* lfull = bars;           // TMA bytes of stage s landed
    uint64_t* lempty = lfull + SL;    // MMAs that read stage s completed
    uint64_t* ofull = lempty + SL;    // W4 operand of stage s unpacked into TMEM
    uint64_t* sfull = ofull + SL;
    uint64_t* sempty = sfull + kScaleStages;
    uint64_t* tfull = sempty + kScaleStages;
    uint64_t* tempty = tfull + C::kNSlot;
    uint64_t* done = tempty + C::kNSlot;
    uint64_t* xfull = done + 1;    // up values written (8 warps)
    uint64_t* xempty = xfull + 1;  // gate warps done reading (8 warps)
    int* tcnt = reinterpret_cast<int*>(xempty + 1);
    int* tb = tcnt + a.num_experts + 1;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;
    __shared__ int total_tiles_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = a.num_experts;
    // k-block j (< kKPS) of stage s
    auto act_at = [&](int s, int j) { return load + s * C::kLoadBytes + j * C::kActBytes; };
    auto w_at = [&](int s) { return load + s * C::kLoadBytes + kKPS * C::kActBytes; };

    if (threadIdx.x == 0) {
        abort_s = 0;
        for (int i = 0; i < SL; ++i) {
            mbar_init(&lfull[i], 1);
            mbar_init(&lempty[i], 1);
            mbar_init(&ofull[i], kConvWarps);
        }
        for (int i = 0; i < kScaleStages; ++i) {
            mbar_init(&sfull[i], kConvWarps);
            mbar_init(&sempty[i], kEpiWarps);
        }
        for (int i = 0; i < C::kNSlot; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpiWarps);
        }
        mbar_init(done, 1);
        mbar_init(xfull, kEpiWarps / 2);
        mbar_init(xempty, kEpiWarps / 2);
        fence_barrier_init();
    }
    // tile table: tcnt[e] = token tiles of expert e, tb[e] = its first tile index
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
    const uint32_t acc_base = tmem_base + C::kARegion;  // accumulator columns
    const int total = total_tiles_s;
    volatile int* abort_flag = &abort_s;

    // lane quadrant of this warp's TMEM accesses
    const int quad = warp & 3;
    const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
    const int half = (warp - kEpiWarp0) >> 2;  // epilogue column quarter (0..3)
    if (C::kGroup && warp >= kEpiWarp0) {
        // every group buffer starts as the float 12582912.0
        for (int b = 0; b < C::kNSlot * 4; ++b)
            tmem_fill<C::kHalf>(acc_base + lane_addr + b * NT + half * C::kHalf, kMagicBits);
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const int kstages = a.kblocks / kKPS;
            uint32_t it = 0;  // stage counter
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                const TileCoord c = decode_tile(t, tb, tcnt, E);
                const int row0 = a.offsets[c.e] + c.mt * NT;
                const uint8_t* wtile = a.w + (size_t)c.e * a.w_expert_stride +
                                       (size_t)c.rt * a.w_tile_stride;
                for (int st = 0; st < kstages; ++st, ++it) {
                    const int s = it % SL;
                    if (!mbar_wait(&lempty[s], ((it / SL) & 1u) ^ 1u, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&lfull[s], C::kStageW + kKPS * C::kActBytes);
                    bulk_g2s(w_at(s), wtile + (size_t)st * C::kStageW, C::kStageW, &lfull[s]);
                    tma_load_3d(act_at(s, 0), &act_map, 0, row0, st * kKPS, &lfull[s]);
                }
            }
            // drain: every issued copy lands before the CTA can exit
            int never = 0;
            for (uint32_t d = it > (uint32_t)SL ? it - SL : 0u; d < it; ++d)
                mbar_wait(&lfull[d % SL], (d / SL) & 1u, &never, a.err);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // At most one tcgen05.commit per k-block (TMEM slot full) plus one per
        // stage (stage empty): the commit is the costly part of issuing.
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(kTileRows, NT);
            const int kstages = a.kblocks / kKPS;
            uint32_t it = 0, kbc = 0, ti = 0;  // stage, k-block and tile counters
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++ti) {
                uint32_t dcol = 0;
                if (!C::kGroup) {
                    const uint32_t buf = ti % 2u;
                    if (!mbar_wait(&tempty[buf], ((ti / 2u) & 1u) ^ 1u, abort_flag, a.err)) break;
                    tc_fence_after();
                    dcol = buf * NT;
                }
                for (int st = 0; st < kstages && ok; ++st, ++it) {
                    const int s = it % SL;
                    if (!mbar_wait(&lfull[s], (it / SL) & 1u, abort_flag, a.err) ||
                        (C::kW4 && !mbar_wait(&ofull[s], (it / SL) & 1u, abort_flag, a.err))) {
                        ok = false;
                        break;
                    }
#pragma unroll
                    for (int jk = 0; jk < kKPS; ++jk, ++kbc) {
                        uint32_t slot = 0;
                        if (C::kGroup) {
                            slot = kbc % C::kNSlot;
                            if (!mbar_wait(&tempty[slot], ((kbc / C::kNSlot) & 1u) ^ 1u, abort_flag,
                                           a.err)) {
                                ok = false;
                                break;
                            }
                        }
                        tc_fence_after();
                        const uint32_t ab = smem_u32(act_at(s, jk));
                        const uint32_t a_tmem = tmem_base + (s * kKPS + jk) * C::kACols;
                        const uint32_t wa = smem_u32(w_at(s) + jk * C::kWBytes);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const uint64_t db = smem_desc_k_sw128(ab + 32 * j);
                            const uint32_t d = C::kGroup ? acc_base + slot * C::kSlotCols + j * NT
                                                         : acc_base + dcol;
                            const uint32_t acc = C::kGroup ? 1u : ((st > 0 || jk > 0 || j > 0) ? 1u : 0u);
                            if (C::kW4)
                                mma_i8_ts(d, a_tmem + 8 * j, db, idesc, acc);
                            else
                                mma_i8(d, smem_desc_k_sw128(wa + 32 * j), db, idesc, acc);
                        }
                        if (C::kGroup) mma_commit(&tfull[slot]);
                    }
                    if (!ok) break;
                    mma_commit(&lempty[s]);
                }
                if (!C::kGroup && ok) mma_commit(&tfull[ti % 2u]);
            }
            // all issued MMAs complete before TMEM can be released
            mma_commit(done);
            int never = 0;
            mbar_wait(done, 0, &never, a.err);
        }
    } else if (warp < kEpiWarp0) {
        // ------------------------------------------------------------ int4 unpack
        if (C::kW4) {
            const int r = quad * 32 + lane;  // weight row = TMEM lane
            const int ct = threadIdx.x - kConvWarp0 * 32;  // 0..127
            const int kstages = a.kblocks / kKPS;
            uint32_t it = 0, kbc = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                for (int st = 0; st < kstages && ok; ++st, ++it) {
                    // the producer refilled stage s only after the MMAs that read its
                    // previous operands completed, so the TMEM operand slot is free
                    const int s = it % SL;
                    if (!mbar_wait(&lfull[s], (it / SL) & 1u, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
#pragma unroll
                    for (int jk = 0; jk < kKPS; ++jk) {
                        // row r of the k-block: 64 bytes in four 16-byte chunks,
                        // chunk c stored at position c ^ ((r >> 1) & 3) (conflict-free)
                        const uint8_t* rowp = w_at(s) + jk * C::kWBytes + r * 64;
                        uint32_t o[32];
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const uint4 p =
                                *reinterpret_cast<const uint4*>(rowp + ((c ^ ((r >> 1) & 3)) << 4));
                            // packed byte b of word w holds k = 32c+8w+b (low nibble) and
                            // k + 4 (high nibble); each lands as 16 * value.
                            o[8 * c + 0] = (p.x << 4) & 0xF0F0F0F0u;
                            o[8 * c + 1] = p.x & 0xF0F0F0F0u;
                            o[8 * c + 2] = (p.y << 4) & 0xF0F0F0F0u;
                            o[8 * c + 3] = p.y & 0xF0F0F0F0u;
                            o[8 * c + 4] = (p.z << 4) & 0xF0F0F0F0u;
                            o[8 * c + 5] = p.z & 0xF0F0F0F0u;
                            o[8 * c + 6] = (p.w << 4) & 0xF0F0F0F0u;
                            o[8 * c + 7] = p.w & 0xF0F0F0F0u;
                        }
                        tmem_st32(tmem_base + lane_addr + (s * kKPS + jk) * C::kACols, o);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ofull[s]);
                    if (C::kGroup) {
                        // hand the stage's group scales to the epilogue (1 KB per k-block)
                        const uint2* ssrc = reinterpret_cast<const uint2*>(w_at(s) + kKPS * C::kWBytes);
#pragma unroll
                        for (int jk = 0; jk < kKPS; ++jk, ++kbc) {
                            const int ss = kbc % kScaleStages;
                            if (!mbar_wait(&sempty[ss], ((kbc / kScaleStages) & 1u) ^ 1u, abort_flag,
                                           a.err)) {
                                ok = false;
                                break;
                            }
                            static_assert(C::kScaleBytes == 8 * 32 * kConvWarps || !C::kGroup,
                                          "one 8-byte piece of the scales per unpack thread");
                            reinterpret_cast<uint2*>(scales + ss * C::kScaleBytes)[ct] =
                                ssrc[jk * (C::kScaleBytes / 8) + ct];
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&sfull[ss]);
                        }
                    }
                }
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int r = quad * 32 + lane;  // weight row within the tile = TMEM lane
        const int c0 = half * C::kHalf;  // first token column of this warp
        uint32_t ti = 0, it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++ti) {
            const TileCoord c = decode_tile(t, tb, tcnt, E);
            const int m_e = a.offsets[c.e + 1] - a.offsets[c.e];
            const int row0 = a.offsets[c.e] + c.mt * NT;
            const int nvalid = min(NT, m_e - c.mt * NT);
            // output channel of this lane (gate/up tiles: 64 gate rows then 64 up rows)
            const bool swiglu_tile = (EPI == kEpiSwiGLU) || (EPI == kEpiAcc && a.swiglu_layout);
            int col;
            bool is_up = false;
            if (swiglu_tile) {
                is_up = r >= 64;
                col = c.rt * 64 + (r & 63);
            } else {
                col = c.rt * kTileRows + r;
            }
            const bool col_ok = col < a.n_valid;
            // lane q prefetches the scale of token column c0 + q (one register across
            // the K loop); the values are broadcast by shuffles at the tile end
            const float my_sx = (lane < C::kHalf && c0 + lane < nvalid) ? a.act_scale[row0 + c0 + lane]
                                                                        : 0.0f;
            float wscale_pc = 0.0f;
            if (!C::kGroup) {
                const float* sp = reinterpret_cast<const float*>(
                    reinterpret_cast<const uint8_t*>(a.wscale) + (size_t)c.e * a.ws_expert_stride +
                    (size_t)c.rt * a.ws_tile_stride);
                wscale_pc = sp[r];
            }
            float facc[C::kHalf];
#pragma unroll
            for (int q = 0; q < C::kHalf; ++q) facc[q] = 0.0f;

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
                    // one TMEM slot per k-block: wait once, load its four group
                    // buffers, start re-arming them, do the math while the stores
                    // drain, then release the slot
                    const uint32_t slot = it % C::kNSlot;
                    if (!mbar_wait(&tfull[slot], (it / C::kNSlot) & 1u, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sbase = acc_base + lane_addr + slot * C::kSlotCols + c0;
                    // two rounds of two groups: load, re-arm (stores drain meanwhile), math
#pragma unroll
                    for (int j0 = 0; j0 < 4; j0 += 2) {
                        uint32_t v[2][C::kHalf];
#pragma unroll
                        for (int jj = 0; jj < 2; ++jj) tmem_ld<C::kHalf>(sbase + (j0 + jj) * NT, v[jj]);
                        tmem_wait_ld();
#pragma unroll
                        for (int jj = 0; jj < 2; ++jj) tmem_fill<C::kHalf>(sbase + (j0 + jj) * NT, kMagicBits);
#pragma unroll
                        for (int jj = 0; jj < 2; ++jj) {
                            const int j = j0 + jj;
                            if (EPI == kEpiAcc) {
                                const int g = kb * 4 + j;
                                const int ncol = is_up ? a.n_valid + col : col;
#pragma unroll
                                for (int q = 0; q < C::kHalf; ++q) {
                                    if (c0 + q < nvalid && col_ok) {
                                        int acc = (int)(v[jj][q] - kMagicBits);
                                        if (C::kW4) acc >>= 4;
                                        a.acc_out[((size_t)(row0 + c0 + q) * (a.kblocks * 4) + g) *
                                                      a.acc_ld + ncol] = acc;
                                    }
                                }
                            } else {
                                // W4 codes enter the MMA as 16*w: fold 1/16 into the scale (exact)
                                const float s_eff = C::kW4 ? sg[j] * 0.0625f : sg[j];
#pragma unroll
                                for (int q = 0; q < C::kHalf; ++q)
                                    facc[q] = __fmaf_rn(__fsub_rn(__uint_as_float(v[jj][q]), kMagic),
                                                        s_eff, facc[q]);
                            }
                        }
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[slot]);
                }
                if (!ok) break;
            } else {
                const uint32_t buf = ti % 2u;
                if (!mbar_wait(&tfull[buf], (ti / 2u) & 1u, abort_flag, a.err)) break;
                tc_fence_after();
                uint32_t v[C::kHalf];
                tmem_ld<C::kHalf>(acc_base + lane_addr + buf * NT + c0, v);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
#pragma unroll
                for (int q = 0; q < C::kHalf; ++q) {
                    int acc = (int)v[q];
                    if (C::kW4) acc >>= 4;
                    if (EPI == kEpiAcc) {
                        if (c0 + q < nvalid && col_ok) {
                            const int ncol = is_up ? a.n_valid + col : col;
                            a.acc_out[(size_t)(row0 + c0 + q) * a.acc_ld + ncol] = acc;
                        }
                    } else {
                        facc[q] = __int2float_rn(acc);
                    }
                }
            }
            if (EPI == kEpiAcc) continue;

            // dequantise with the per-token activation scale
            float val[C::kHalf];
#pragma unroll
            for (int q = 0; q < C::kHalf; ++q) {
                const float sxq = __shfl_sync(0xffffffffu, my_sx, q);
                if (C::kGroup)
                    val[q] = __fmul_rn(facc[q], sxq);
                else
                    val[q] = __fmul_rn(__fmul_rn(facc[q], sxq), wscale_pc);
            }
            if (EPI == kEpiSwiGLU) {
                // up lanes (64..127) hand their values to the gate lanes of the same channel
                const uint32_t xph = ti & 1u;
                if (is_up) {
                    if (!mbar_wait(xempty, xph ^ 1u, abort_flag, a.err)) { ok = false; break; }
#pragma unroll
                    for (int q = 0; q < C::kHalf; ++q) xchg[(r - 64) * C::kXchgStride + c0 + q] = val[q];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xfull);
                } else {
                    if (!mbar_wait(xfull, xph, abort_flag, a.err)) { ok = false; break; }
#pragma unroll
                    for (int q = 0; q < C::kHalf; ++q) {
                        const int j = c0 + q;
                        if (j < nvalid && col_ok) {
                            const float gv = val[q];
                            const float uv = xchg[r * C::kXchgStride + j];
                            const float d = __fadd_rn(1.0f, expf(-gv));
                            a.out[(size_t)(row0 + j) * a.ldo + col] = __fmul_rn(__fdiv_rn(gv, d), uv);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xempty);
                }
            } else if (col_ok) {
#pragma unroll
                for (int q = 0; q < C::kHalf; ++q)
                    if (c0 + q < nvalid) a.out[(size_t)(row0 + c0 + q) * a.ldo + col] = val[q];
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
    b += (size_t)C::kLoadStages * C::kLoadBytes;
    b += (size_t)kScaleStages * C::kScaleBytes;
    b += sizeof(float) * (64 * C::kXchgStride + 2);
    b += sizeof(uint64_t) * (3 * C::kLoadStages + 2 * kScaleStages + 2 * C::kNSlot + 3);
    b += sizeof(int) * (2 * (size_t)E + 2);
    // one CTA per SM: the kernel allocates all 512 TMEM columns
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
        case 64:
            if constexpr (FMT != kFmtW4G32) return launch_gemm_t<FMT, EPI, 64>(map, a, num_sms, s);
            return -1;
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
