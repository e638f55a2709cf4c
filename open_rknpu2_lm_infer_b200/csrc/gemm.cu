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
//   warps 6..13  epilogue, two warps per TMEM lane quadrant, each owning half
//                of the token columns. The epilogue shares each SM sub-partition
//                with an unpack warp, so it is kept to few instructions per value.
//
// Group-32 formats: one MMA (K = 32 = one group) per TMEM buffer; the four
// buffers of a k-block form a slot. Every buffer holds the bits of 12582912.0f
// (0x4B400000) before its MMA, which adds the int32 sum to them, so the result
// read back as a float is exactly 12582912 + 16*acc (|16*acc| < 2^22). The
// epilogue re-arms the buffers right after loading them and computes
// f = fma(D - 12582912, s/16, f) two values per instruction (f32x2): an exact
// subtraction and one FMA, equal to fma((float)acc, s, f) bit for bit. Per-channel formats: all of K accumulates in TMEM,
// one dequant per tile.
#include "kernels.cuh"

namespace moe {

constexpr int kGemmThreads = 448;
constexpr int kConvWarp0 = 2;         // first unpack warp
constexpr int kConvWarps = 4;
constexpr int kEpiWarp0 = 6;          // first epilogue warp
constexpr int kEpiWarps = 8;
constexpr int kTileRows = 128;        // weight rows per tile (MMA M)
constexpr int kKBlock = 128;          // K bytes per k-block (one 128B swizzle row)
// Shared memory: the load ring gets what is left of 227 KB after the tile
// tables (up to 1024 experts), barriers and the 1 KB alignment slack.
constexpr int kSmemTotal = 227 * 1024;
constexpr int kSmemFixed = 10 * 1024;
constexpr int kMaxLoadStages = 8;
constexpr uint32_t kMagicBits = 0x4B400000u;  // 12582912.0f
constexpr float kMagic = 12582912.0f;

template <int FMT, int NT>
struct GemmCfg {
    static constexpr bool kW4 = (FMT == kFmtW4G32 || FMT == kFmtW4PC);
    static constexpr bool kGroup = (FMT == kFmtW4G32);
    static constexpr int kWBytes = kW4 ? kTileRows * kKBlock / 2 : kTileRows * kKBlock;
    static constexpr int kActBytes = NT * kKBlock;           // per k-block
    static constexpr int kStageW = kKPS * kWBytes;           // weight request of one stage
    // load stage: [activations kKPS x NT x 128][weights]; W8 weights are the MMA
    // operand tiles, W4 weights are unpacked into TMEM.
    static constexpr int kLoadBytes = kKPS * kActBytes + kStageW;
    static constexpr int kLoadBudget = kSmemTotal - kSmemFixed;
    static constexpr int kLoadStages = kLoadBudget / kLoadBytes > kMaxLoadStages
                                           ? kMaxLoadStages : kLoadBudget / kLoadBytes;
    // TMEM: [W4 weight operand ring: kAStages x kKPS x 32 columns][accumulators].
    // The operand ring is shallower than the load ring: unpacking is quick,
    // while HBM latency needs many stages of loads in flight.
    static constexpr int kACols = 32;                        // one k-block of int8 weights
    static constexpr int kAStages = kW4 ? (kGroup ? 2 : 4) : 0;
    static constexpr int kARegion = kAStages * kKPS * kACols;
    // group formats: slots of one k-block (4 group buffers of NT columns);
    // per-channel formats: two tile accumulators.
    static constexpr int kSlotCols = kGroup ? 4 * NT : NT;
    static constexpr int kAccFree = 512 - kARegion;
    static constexpr int kNSlot = kGroup ? ((kAccFree / kSlotCols) < 4 ? (kAccFree / kSlotCols) : 4)
                                         : 2;
    static constexpr int kAllocCols = 512;
    static constexpr int kHalf = NT / 2;                      // columns per epilogue warp
    static_assert(kLoadStages >= 2, "smem budget");
    static_assert(kLoadStages >= kAStages, "operand ring reuse is ordered by the load ring");
    static_assert(kNSlot >= 2, "TMEM budget: group formats need NT <= 32");
    static_assert(kARegion + kNSlot * kSlotCols <= 512, "TMEM budget");
    static_assert(kHalf % 2 == 0, "paired f32x2 epilogue math");
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

// Group scales of (tile, stage) for one weight row: 16 bytes, kKPS k-blocks x 4
// groups of fp16, read through the read-only path two stages ahead of use.
struct ScaleCursor {
    int t, st;
    const uint8_t* base;  // scales of the current tile
};

template <int FMT, int EPI, int NT>
__global__ void __launch_bounds__(kGemmThreads, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap act_map, const GemmArgs a) {
    using C = GemmCfg<FMT, NT>;
    constexpr int SL = C::kLoadStages;
    constexpr int AS = C::kAStages;
    constexpr int AS1 = AS > 0 ? AS : 1;  // ring arithmetic of formats without one
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* load = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(load + SL * C::kLoadBytes);
    uint64_t* lfull = bars;             // TMA bytes of stage s landed
    uint64_t* lempty = lfull + SL;      // MMAs that read stage s completed
    uint64_t* ofull = lempty + SL;      // W4 operand slot a unpacked into TMEM
    uint64_t* tfull = ofull + (AS > 0 ? AS : 1);
    uint64_t* tempty = tfull + C::kNSlot;
    uint64_t* done = tempty + C::kNSlot;
    int* tcnt = reinterpret_cast<int*>(done + 1);
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
        }
        for (int i = 0; i < AS; ++i) mbar_init(&ofull[i], kConvWarps);
        for (int i = 0; i < C::kNSlot; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpiWarps);
        }
        mbar_init(done, 1);
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
    const int kstages = a.kblocks / kKPS;
    volatile int* abort_flag = &abort_s;

    // lane quadrant of this warp's TMEM accesses
    const int quad = warp & 3;
    const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
    const int half = (warp - kEpiWarp0) >> 2;  // epilogue column half (0..1)
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
        // stage (stage empty). Each mbarrier wait on this thread stalls the MMA
        // issue (~150 cycles even when the phase is complete), so it waits on as
        // few as possible: W4 stages only on the unpack warps' barrier (they
        // waited for the stage's copies first), W8 stages on the copies.
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(kTileRows, NT);
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
                    const int ao = it % AS1;
                    if (C::kW4 ? !mbar_wait(&ofull[ao], (it / AS1) & 1u, abort_flag, a.err)
                               : !mbar_wait(&lfull[s], (it / SL) & 1u, abort_flag, a.err)) {
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
                        const uint32_t a_tmem = tmem_base + (ao * kKPS + jk) * C::kACols;
                        const uint32_t wa = smem_u32(w_at(s) + jk * C::kWBytes);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const uint64_t db = smem_desc_k_sw128(ab + 32 * j);
                            const uint32_t d = C::kGroup ? acc_base + slot * C::kSlotCols + j * NT
                                                         : acc_base + dcol;
                            // group formats: each buffer adds one group's sum to the
                            // magic float; per-channel formats: accumulate over K
                            const uint32_t acc = C::kGroup ? 1u : ((st > 0 || jk > 0 || j > 0) ? 1u : 0u);
                            if (C::kW4)
                                mma_i8_ts(d, a_tmem + 8 * j, db, idesc, acc);
                            else
                                mma_i8(d, smem_desc_k_sw128(wa + 32 * j), db, idesc, acc);
                        }
                        if (C::kGroup) mma_commit(&tfull[slot]);
                    }
                    if (!ok) break;
                    // also frees the stage's W4 operand slot for the unpack warps
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
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                for (int st = 0; st < kstages; ++st, ++it) {
                    const int s = it % SL;
                    const int ao = it % AS1;
                    // operand slot ao was last read by the MMAs of stage it - AS; their
                    // commit completed phase (it - AS) / SL of that stage's lempty (it
                    // cannot have moved further: its next phase needs this stage)
                    if (it >= (uint32_t)AS1) {
                        const uint32_t prev = it - AS1;
                        if (!mbar_wait(&lempty[prev % SL], (prev / SL) & 1u, abort_flag, a.err)) {
                            ok = false;
                            break;
                        }
                    }
                    if (!mbar_wait(&lfull[s], (it / SL) & 1u, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
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
                        tmem_st32(tmem_base + lane_addr + (ao * kKPS + jk) * C::kACols, o);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    // the MMA issuer waits on this barrier alone: these warps have
                    // observed the stage's copies (lfull) before arriving
                    if (lane == 0) mbar_arrive(&ofull[ao]);
                }
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int r = quad * 32 + lane;  // weight row within the tile = TMEM lane
        const int c0 = half * C::kHalf;  // first token column of this warp
        // group scales: a cursor two stages ahead of use over the same tile order
        ScaleCursor cur{(int)blockIdx.x, 0, nullptr};
        auto cursor_tile = [&](ScaleCursor& k) {
            k.base = nullptr;
            if (k.t < total) {
                const TileCoord c = decode_tile(k.t, tb, tcnt, E);
                k.base = reinterpret_cast<const uint8_t*>(a.wscale) + (size_t)c.e * a.ws_expert_stride +
                         (size_t)c.rt * a.ws_tile_stride;
            }
        };
        auto cursor_load = [&](ScaleCursor& k) -> uint4 {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (k.base)
                v = __ldg(reinterpret_cast<const uint4*>(k.base + ((size_t)k.st * kTileRows + r) * 16));
            if (++k.st == kstages) {
                k.st = 0;
                k.t += gridDim.x;
                cursor_tile(k);
            }
            return v;
        };
        uint4 pf0 = make_uint4(0u, 0u, 0u, 0u), pf1 = pf0;
        if (C::kGroup) {
            static_assert(kKPS == 2 || !C::kGroup, "16 bytes of group scales per row and stage");
            cursor_tile(cur);
            pf0 = cursor_load(cur);
            pf1 = cursor_load(cur);
        }
        uint32_t ti = 0, it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++ti) {
            const TileCoord c = decode_tile(t, tb, tcnt, E);
            const int m_e = a.offsets[c.e + 1] - a.offsets[c.e];
            const int row0 = a.offsets[c.e] + c.mt * NT;
            const int nvalid = min(NT, m_e - c.mt * NT);
            // output channel of this lane (gate/up tiles: 64 gate rows then 64 up rows)
            const bool swiglu_tile = (EPI == kEpiGateUp) || (EPI == kEpiAcc && a.swiglu_layout);
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
            // this warp's token columns hold no token at all (the expert's last tile):
            // it still takes part in every slot handshake but skips the loads and math
            const bool active = c0 < nvalid;
            float2 facc[C::kHalf / 2];
#pragma unroll
            for (int q = 0; q < C::kHalf / 2; ++q) facc[q] = make_float2(0.0f, 0.0f);

            if (C::kGroup) {
                for (int st = 0; st < kstages && ok; ++st) {
                    const uint4 sc = pf0;
                    pf0 = pf1;
                    pf1 = cursor_load(cur);
                    // the stage's 8 group scales (k-block jk, group j at 4*jk + j), with
                    // the 1/16 of the W4 codes folded in (exact)
                    float2 sg[4];
                    {
                        const uint32_t w[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            sg[i] = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
                            if (C::kW4) sg[i] = __fmul2_rn(sg[i], make_float2(0.0625f, 0.0625f));
                        }
                    }
#pragma unroll 1
                    for (int jk = 0; jk < kKPS; ++jk, ++it) {
                        const int kb = st * kKPS + jk;
                        const float2 sga = jk ? sg[2] : sg[0];  // groups 0, 1 of this k-block
                        const float2 sgb = jk ? sg[3] : sg[1];  // groups 2, 3
                        // one TMEM slot per k-block: wait once, load its four group
                        // buffers, re-arm them, release the slot, then do the math
                        const uint32_t slot = it % C::kNSlot;
                        if (!mbar_wait(&tfull[slot], (it / C::kNSlot) & 1u, abort_flag, a.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sbase = acc_base + lane_addr + slot * C::kSlotCols + c0;
                        // rounds of 8 token columns x 4 groups bound the registers; each
                        // round is loaded, re-armed and folded into its columns' sums
                        // (the group order per column stays 0..3)
                        constexpr int kRound = C::kHalf < 8 ? C::kHalf : 8;
                        const int ncol = is_up ? a.n_valid + col : col;
#pragma unroll
                        for (int r0 = 0; r0 < C::kHalf; r0 += kRound) {
                            uint32_t v[4][kRound];
                            if (active) {
#pragma unroll
                                for (int j = 0; j < 4; ++j) tmem_ld<kRound>(sbase + j * NT + r0, v[j]);
                                tmem_wait_ld();
#pragma unroll
                                for (int j = 0; j < 4; ++j) tmem_ld_pin(v[j]);
                            }
                            // columns of an idle warp are re-armed too: the MMA adds to them
#pragma unroll
                            for (int j = 0; j < 4; ++j) tmem_fill<kRound>(sbase + j * NT + r0, kMagicBits);
                            if (!active) continue;
                            if (EPI == kEpiAcc) {
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
#pragma unroll
                                    for (int q = 0; q < kRound; ++q) {
                                        if (c0 + r0 + q < nvalid && col_ok) {
                                            int acc = (int)(v[j][q] - kMagicBits);
                                            if (C::kW4) acc >>= 4;
                                            a.acc_out[((size_t)(row0 + c0 + r0 + q) * (a.kblocks * 4) + kb * 4 +
                                                       j) * a.acc_ld + ncol] = acc;
                                        }
                                    }
                                }
                            } else {
                                const float2 nm = make_float2(-kMagic, -kMagic);
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    const float2 sp = (j >> 1) ? sgb : sga;
                                    const float sj = (j & 1) ? sp.y : sp.x;
                                    const float2 s2 = make_float2(sj, sj);
#pragma unroll
                                    for (int q = 0; q < kRound / 2; ++q) {
                                        const float2 d = __fadd2_rn(
                                            make_float2(__uint_as_float(v[j][2 * q]), __uint_as_float(v[j][2 * q + 1])),
                                            nm);
                                        facc[r0 / 2 + q] = __ffma2_rn(d, s2, facc[r0 / 2 + q]);
                                    }
                                }
                            }
                        }
                        tmem_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[slot]);
                    }
                }
                if (!ok) break;
            } else {
                const uint32_t buf = ti % 2u;
                if (!mbar_wait(&tfull[buf], (ti / 2u) & 1u, abort_flag, a.err)) break;
                tc_fence_after();
                uint32_t v[C::kHalf];
                tmem_ld<C::kHalf>(acc_base + lane_addr + buf * NT + c0, v);
                tmem_wait_ld();
                tmem_ld_pin(v);
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
                        const float f = __int2float_rn(acc);
                        if (q & 1) facc[q >> 1].y = f; else facc[q >> 1].x = f;
                    }
                }
            }
            if (EPI == kEpiAcc) continue;

            // dequantise with the per-token activation scale
            float val[C::kHalf];
#pragma unroll
            for (int q = 0; q < C::kHalf; ++q) {
                const float sxq = __shfl_sync(0xffffffffu, my_sx, q);
                const float f = (q & 1) ? facc[q >> 1].y : facc[q >> 1].x;
                if (C::kGroup)
                    val[q] = __fmul_rn(f, sxq);
                else
                    val[q] = __fmul_rn(__fmul_rn(f, sxq), wscale_pc);
            }
            if (col_ok) {
                // gate/up tiles: gate channels to the first half of the row, up to the second
                const int ocol = (EPI == kEpiGateUp && is_up) ? a.n_valid + col : col;
#pragma unroll
                for (int q = 0; q < C::kHalf; ++q)
                    if (c0 + q < nvalid) a.out[(size_t)(row0 + c0 + q) * a.ldo + ocol] = val[q];
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
    b += sizeof(uint64_t) * (2 * C::kLoadStages + (C::kAStages > 0 ? C::kAStages : 1) +
                             2 * C::kNSlot + 1);
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
        case kEpiGateUp: return launch_gemm_nt<FMT, kEpiGateUp>(map, a, nt, num_sms, s);
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
