// Grouped expert GEMMs on the sm_100a tensor cores (tcgen05).
//
// Replaces the gate/up and down GEMMs of the reference's native MoE operator
// (rk_npu_moe_w8_run_f32, called at src/npu/moe.rs:372-386; arithmetic restated
// from llm_generated_docs/MINICPMV47_35A3_FUSED_MOE_20261019.md:77 and
// MOE_CPU_FUSION_20261023.md:12-13): int8 activations x int4/int8 weights.
//
// Layout ("swap-AB"): the weight tile is the MMA's M=128 operand and the
// tokens of one expert are the N operand, so one TMEM lane = one output
// channel and TMEM columns = tokens. Small token counts (decode) cost N=16
// columns instead of a 128-row M tile.
//
// Formats:
//   W8 / W4 per-channel  kind::i8, exact int32 accumulation over all of K,
//                        one dequantisation per tile: (acc * s_x) * s_w.
//   W4 group-32 (G32H)   kind::f16: the unpack warps write w * s_group (one
//                        fp16 rounding of an exact product of an int4 code and
//                        an fp16 scale); the activation codes are exact in
//                        fp16; all of K accumulates in fp32. One accumulator
//                        per tile instead of one per group: a K=32 MMA per
//                        group with a TMEM read-back per k-block is bound by
//                        that round trip (measured ~3.5x slower).
//   W4 group-32 (exact)  kind::i8, one MMA (K = 32 = one group) per TMEM
//                        buffer, overwriting it; the four buffers of a k-block
//                        form a slot. The epilogue adds the bits of
//                        12582912.0f to each int32 sum D = 16*acc (an integer
//                        add), which reads back as the float 12582912 + 16*acc
//                        exactly (|16*acc| < 2^22), and computes
//                        f = fma(that - 12582912, s/16, f) two values per
//                        instruction (f32x2), equal to fma((float)acc, s, f) bit
//                        for bit. Used where the result is requantised (the
//                        gate/up GEMM: a rounding difference there flips int8
//                        middle codes) and for the accumulator dump; G32H where
//                        it is not (the down GEMM).
//
// A load stage covers 256 k: one bulk copy of the weights (group-32: with the
// stage's group scales) and one 3-D TMA copy of the permuted activation rows.
// A copy request costs ~0.2 us per SM whatever its size, so stages are large.
//
// Warp roles (448 threads):
//   warp 0       producer
//   warp 1       TMEM allocator + single-thread MMA issuer. Each mbarrier wait
//                on this thread stalls the MMA issue (~150 cycles even when the
//                phase is complete), so it waits on as few barriers as it can.
//   warps 2..5   W4 formats: unpack into tensor memory, one warp per TMEM lane
//                quadrant, one weight row per thread; the MMA reads its weight
//                operand from TMEM (no shared-memory operand, no proxy fence).
//   warps 6..13  epilogue, two warps per TMEM lane quadrant, each owning half
//                of the token columns.
// One CTA per SM (all 512 TMEM columns), except the exact group path at
// 16-token tiles: two CTAs per SM with 256 columns and half the shared memory
// each, so that two k-block pipelines overlap their latencies.
#include "kernels.cuh"

namespace moe {

constexpr int kProdWarp = 0;          // copy producer
constexpr int kMmaWarp = 1;           // TMEM allocator + MMA issuer
constexpr int kConvWarp0 = 2;         // first unpack warp
constexpr int kEpiWarps = 8;
constexpr int kTileRows = 128;        // weight rows per tile (MMA M)
constexpr int kKBlock = 128;          // int8 k per k-block (one 128-byte swizzle row)
constexpr int kStageK = kKPS * kKBlock;  // k per load stage (256)
// Shared memory: the load ring gets what is left of 227 KB after the tile
// tables and grouping offsets (up to 1024 experts), barriers and the 1 KB
// alignment slack.
constexpr int kSmemTotal = 227 * 1024;
constexpr int kSmemFixed = 14 * 1024;
constexpr int kMaxLoadStages = 8;
constexpr bool kGroupDual = true;  // exact group path, 16-token tiles: two CTAs per SM
constexpr uint32_t kMagicBits = 0x4B400000u;  // 12582912.0f
constexpr float kMagic = 12582912.0f;

// kind::f16 instruction descriptor: fp16 A and B, fp32 accumulate, both
// operands K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem]^T, fp16 x fp16 -> fp32, one CTA.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

template <int FMT, int NT>
struct GemmCfg {
    static constexpr bool kF16 = (FMT == kFmtW4G32H);
    static constexpr bool kGroup = (FMT == kFmtW4G32);  // exact per-group sums
    static constexpr bool kW4 = (FMT != kFmtW8PC);
    static constexpr bool kG32Pack = kF16 || kGroup;     // group-32 stage layout
    // weights of one stage in HBM and the part of them one request copies
    static constexpr int kStageWStride = kG32Pack ? 128 * 128 + 128 * 16
                                                  : kKPS * kTileRows * (kW4 ? kKBlock / 2 : kKBlock);
    // (the exact group path copies the stage's group scales too: the epilogue
    // reads them from shared memory)
    static constexpr int kStageW = kStageWStride;
    // activations of one stage: int8 kKPS atoms of NT x 128 B, fp16 2*kKPS
    static constexpr int kAtoms = kF16 ? 2 * kKPS : kKPS;
    static constexpr int kStageAct = kAtoms * NT * 128;
    // load stage: [activations][weights (+ group scales)]
    static constexpr int kLoadBytes = kStageAct + kStageW;
    // exact group path at 16-token tiles: two CTAs per SM, each with half of
    // the shared memory and of the tensor memory, so that two k-block
    // pipelines overlap each other's latencies
    static constexpr bool kDual = kGroup && NT == 16 && kGroupDual;
    static constexpr int kCtasPerSm = kDual ? 2 : 1;
    static constexpr int kLoadBudget = kSmemTotal / kCtasPerSm - kSmemFixed;
    static constexpr int kLoadStages = kLoadBudget / kLoadBytes > kMaxLoadStages
                                           ? kMaxLoadStages : kLoadBudget / kLoadBytes;
    // TMEM: [W4 weight operand ring: kAStages x kStageACols][accumulators]. The
    // operand ring is shallower than the load ring: unpacking is quick, while
    // HBM latency needs many stages of loads in flight.
    static constexpr int kStageACols = kF16 ? 128 : (kW4 ? kKPS * 32 : 0);
    static constexpr int kAStages = kW4 ? (kF16 || kGroup ? 2 : 4) : 0;
    static constexpr int kARegion = kAStages * kStageACols;
    // exact group path: slots of one k-block (4 group buffers of NT columns);
    // other formats: two tile accumulators.
    static constexpr int kSlotCols = kGroup ? 4 * NT : NT;
    static constexpr int kAllocCols = kDual ? 256 : 512;  // TMEM columns of one CTA
    static constexpr int kAccFree = kAllocCols - kARegion;
    static constexpr int kNSlot = kGroup ? ((kAccFree / kSlotCols) < 4 ? (kAccFree / kSlotCols) : 4)
                                         : 2;
    static constexpr int kHalf = NT / 2;                      // columns per epilogue warp
    static constexpr int kMmaPerStage = kF16 ? kStageK / 16 : kKPS * 4;
    // unpack warps: one per TMEM lane quadrant; two for the fp16 conversion
    // (each converts half of a stage's groups), the heaviest per weight
    static constexpr int kConvWarps = kF16 ? 8 : 4;
    static constexpr int kEpiWarp0 = kConvWarp0 + kConvWarps;  // first epilogue warp
    static constexpr int kStoreWarp = kEpiWarp0 + kEpiWarps;   // exact group path only
    // exact group path: two MMA issuers (lane 0 of warp 1 and of this warp) on
    // alternating k-blocks; a thread issues one MMA per ~65 cycles whatever N
    static constexpr int kIssuers = kGroup ? 2 : 1;
    static constexpr int kIssuerWarp2 = kStoreWarp + 1;
    static constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps + (kGroup ? 2 : 0));
    static_assert(kLoadBytes % 1024 == 0, "stage alignment of the swizzled operands");
    static_assert(kLoadStages >= 2, "smem budget");
    static_assert(kLoadStages >= kAStages, "operand ring reuse is ordered by the load ring");
    static_assert(kNSlot >= 2, "TMEM budget: the exact group path needs NT <= 32");
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

// Group-32 packed word (8 offset-binary nibbles; k = 8w + j, j even in nibble
// j/2, j odd in nibble 4 + j/2) -> fp16 pairs (k 2i, 2i+1) times the group
// scale: (1024 + n) - 1032 = w exactly, then one rounding of w * s.
__device__ __forceinline__ void g32_word_to_half(uint32_t word, __half2 s2, uint32_t* out) {
    const __half2 bias = __float2half2_rn(1032.0f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t h = ((word >> (4 * i)) & 0x000F000Fu) | 0x64006400u;
        const __half2 w = __hsub2(*reinterpret_cast<const __half2*>(&h), bias);
        const __half2 v = __hmul2(w, s2);
        out[i] = *reinterpret_cast<const uint32_t*>(&v);
    }
}

// The same word -> 16*w as int8 in k order (two words: k 0..3, k 4..7).
__device__ __forceinline__ void g32_word_to_i8(uint32_t word, uint32_t* out) {
    const uint32_t t = word ^ 0x88888888u;        // offset-binary -> two's complement
    const uint32_t lo = (t << 4) & 0xF0F0F0F0u;   // nibbles 0,2,4,6 = k 0,4,1,5
    const uint32_t hi = t & 0xF0F0F0F0u;          // nibbles 1,3,5,7 = k 2,6,3,7
    out[0] = __byte_perm(lo, hi, 0x6420);         // k 0,1,2,3
    out[1] = __byte_perm(lo, hi, 0x7531);         // k 4,5,6,7
}

// Shared-memory layout of one instantiation. The exact group path's Store
// epilogue (the down GEMM) stages each tile's outputs as [NT][128] f32 for a
// store warp whose bulk copies write them, at the price of load stages (a down
// tile has 6 k-blocks, so the per-tile store cost dominates); its gate/up
// tiles (16 k-blocks, a deeper weight stream) keep every load stage and store
// directly.
template <int FMT, int EPI, int NT>
struct GemmLayout {
    using C = GemmCfg<FMT, NT>;
    static constexpr bool kStaged = C::kGroup && EPI == kEpiStore;
    static constexpr int kStgBytes = kStaged ? NT * 128 * 4 : 0;
    static constexpr int kFit = (C::kLoadBudget - kStgBytes) / C::kLoadBytes;
    static constexpr int kLoadStages = kFit > kMaxLoadStages ? kMaxLoadStages : kFit;
    static_assert(kStgBytes % 1024 == 0, "staging tile alignment (bulk copies)");
    static_assert(kLoadStages >= 2 && kLoadStages >= C::kAStages, "smem budget");
};

template <int FMT, int EPI, int NT>
__global__ void __launch_bounds__(GemmCfg<FMT, NT>::kThreads, GemmCfg<FMT, NT>::kCtasPerSm)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap act_map, const GemmArgs a) {
    using C = GemmCfg<FMT, NT>;
    using Lay = GemmLayout<FMT, EPI, NT>;
    constexpr int SL = Lay::kLoadStages;
    constexpr int AS = C::kAStages;
    constexpr int AS1 = AS > 0 ? AS : 1;  // ring arithmetic of formats without one
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* load = smem;
    // exact group path: the staging tile of the outputs, 1024-byte aligned (the
    // store warp's bulk copies read it from 16-byte aligned rows)
    float* stg = reinterpret_cast<float*>(load + SL * C::kLoadBytes);  // [NT][128]
    uint64_t* bars = reinterpret_cast<uint64_t*>(load + SL * C::kLoadBytes + Lay::kStgBytes);
    uint64_t* lfull = bars;             // TMA bytes of stage s landed
    uint64_t* lempty = lfull + SL;      // MMAs that read stage s completed
    uint64_t* ofull = lempty + SL;      // W4 operand slot a unpacked into TMEM
    uint64_t* tfull = ofull + AS1;
    uint64_t* tempty = tfull + C::kNSlot;
    uint64_t* done = tempty + C::kNSlot;
    uint64_t* sfull = done + 1;         // staging tile written by the epilogue warps
    uint64_t* sempty = sfull + 1;       // staging tile read by the store warp's copies
    int* tcnt = reinterpret_cast<int*>(sempty + 1);
    int* tb = tcnt + a.num_experts + 1;
    int* offs = tb + a.num_experts + 1;  // the grouping offsets, read once
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;
    __shared__ int total_tiles_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = a.num_experts;
    auto act_at = [&](int s) { return load + s * C::kLoadBytes; };
    auto w_at = [&](int s) { return load + s * C::kLoadBytes + C::kStageAct; };

    if (threadIdx.x == 0) {
        abort_s = 0;
        for (int i = 0; i < SL; ++i) {
            mbar_init(&lfull[i], 1);
            // exact group path: the issuers' MMA commits and every epilogue warp
            // (the stage holds the group scales the epilogue reads)
            mbar_init(&lempty[i], C::kGroup ? C::kIssuers + kEpiWarps : 1);
        }
        for (int i = 0; i < AS; ++i) mbar_init(&ofull[i], C::kConvWarps);
        for (int i = 0; i < C::kNSlot; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpiWarps);
        }
        mbar_init(done, C::kIssuers);
        mbar_init(sfull, kEpiWarps);
        mbar_init(sempty, 1);
        fence_barrier_init();
    }
    // tile table: tcnt[e] = token tiles of expert e, tb[e] = its first tile index
    if (warp == kConvWarp0) {
        const int per = (E + 31) / 32;
        int local = 0;
        for (int i = 0; i < per; ++i) {
            int e = lane * per + i;
            if (e < E) {
                const int o0 = a.offsets[e], o1 = a.offsets[e + 1];
                offs[e] = o0;
                if (e == E - 1) offs[E] = o1;
                int c = (o1 - o0 + NT - 1) / NT;
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
    if (warp == kMmaWarp) {
        tmem_alloc(&tmem_base_s, C::kAllocCols);
        tmem_relinquish();
    }
    if (warp == kProdWarp && lane == 0) prefetch_tensormap(&act_map);
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
    if constexpr (C::kGroup) {
        // every group buffer starts as the bits of 12582912.0f: the MMAs
        // accumulate onto them, the epilogue re-arms a slot after reading it
        if (warp >= C::kEpiWarp0 && warp < C::kEpiWarp0 + kEpiWarps) {
            const int c0 = ((warp - C::kEpiWarp0) >> 2) * C::kHalf;
            for (int sl = 0; sl < C::kNSlot; ++sl)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    tmem_fill<C::kHalf>(acc_base + lane_addr + sl * C::kSlotCols + j * NT + c0, kMagicBits);
            tmem_wait_st();
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == kProdWarp) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t it = 0;  // stage counter
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                const TileCoord c = decode_tile(t, tb, tcnt, E);
                const int row0 = offs[c.e] + c.mt * NT;
                const uint8_t* wtile = a.w + (size_t)c.e * a.w_expert_stride +
                                       (size_t)c.rt * a.w_tile_stride;
                for (int st = 0; st < kstages; ++st, ++it) {
                    const int s = it % SL;
                    if (!mbar_wait(&lempty[s], ((it / SL) & 1u) ^ 1u, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&lfull[s], C::kStageW + C::kStageAct);
                    bulk_g2s(w_at(s), wtile + (size_t)st * a.w_stage_stride, C::kStageW, &lfull[s]);
                    tma_load_3d(act_at(s), &act_map, 0, row0, st * C::kAtoms, &lfull[s]);
                }
            }
            // drain: every issued copy lands before the CTA can exit
            int never = 0;
            for (uint32_t d = it > (uint32_t)SL ? it - SL : 0u; d < it; ++d)
                mbar_wait(&lfull[d % SL], (d / SL) & 1u, &never, a.err);
        }
    } else if (warp == kMmaWarp || (C::kGroup && warp == C::kIssuerWarp2)) {
        // ------------------------------------------------------------ MMA issuer
        // One tcgen05.commit per stage (stage empty, which also frees the W4
        // operand slot) and per tile (accumulator full); the exact group path
        // commits per k-block instead of per tile, its two issuers taking the
        // even and the odd k-blocks (each commits its share of every stage).
        const uint32_t me = warp == kMmaWarp ? 0u : 1u;
        if (lane == 0) {
            constexpr uint32_t idesc = C::kF16 ? idesc_f16(kTileRows, NT) : idesc_i8(kTileRows, NT);
            uint32_t it = 0, kbc = 0, ti = 0;  // stage, k-block and tile counters
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++ti) {
                uint32_t dcol = 0;
                if (!C::kGroup) {
                    const uint32_t buf = ti % 2u;
                    if (!mbar_wait_fast(&tempty[buf], ((ti / 2u) & 1u) ^ 1u, abort_flag, a.err)) break;
                    tc_fence_after();
                    dcol = buf * NT;
                }
                for (int st = 0; st < kstages && ok; ++st, ++it) {
                    const int s = it % SL;
                    const int ao = it % AS1;
                    // W4 stages: the unpack warps' barrier alone (they waited for the
                    // stage's copies before arriving); W8 stages: the copies
                    if (C::kW4 ? !mbar_wait_fast(&ofull[ao], (it / AS1) & 1u, abort_flag, a.err)
                               : !mbar_wait_fast(&lfull[s], (it / SL) & 1u, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ab = smem_u32(act_at(s));
                    const uint32_t a_tmem = tmem_base + ao * C::kStageACols;
                    if constexpr (C::kF16) {
                        // 16 MMAs of k = 16: A columns 8j.., B atom j/4 at byte 32*(j%4)
#pragma unroll
                        for (int j = 0; j < C::kMmaPerStage; ++j) {
                            const uint64_t db = smem_desc_k_sw128(ab + (j >> 2) * NT * 128 + 32 * (j & 3));
                            mma_f16_ts(acc_base + dcol, a_tmem + 8 * j, db, idesc,
                                       (st > 0 || j > 0) ? 1u : 0u);
                        }
                    } else {
#pragma unroll
                        for (int jk = 0; jk < kKPS; ++jk, ++kbc) {
                            if (C::kGroup && kbc % C::kIssuers != me) continue;
                            uint32_t slot = 0;
                            if (C::kGroup) {
                                slot = kbc % C::kNSlot;
                                if (!mbar_wait_fast(&tempty[slot], ((kbc / C::kNSlot) & 1u) ^ 1u, abort_flag,
                                               a.err)) {
                                    ok = false;
                                    break;
                                }
                                tc_fence_after();
                            }
                            const uint32_t abk = ab + jk * NT * 128;
                            const uint32_t wa = smem_u32(w_at(s) + jk * kTileRows * kKBlock);
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const uint64_t db = smem_desc_k_sw128(abk + 32 * j);
                                // exact group path: each buffer receives one group's sum
                                // (overwritten); per-channel: accumulate over K
                                const uint32_t d = C::kGroup ? acc_base + slot * C::kSlotCols + j * NT
                                                             : acc_base + dcol;
                                const uint32_t acc =
                                    C::kGroup ? 1u : ((st > 0 || jk > 0 || j > 0) ? 1u : 0u);
                                if (C::kW4)
                                    mma_i8_ts(d, a_tmem + jk * 32 + 8 * j, db, idesc, acc);
                                else
                                    mma_i8(d, smem_desc_k_sw128(wa + 32 * j), db, idesc, acc);
                            }
                            if (C::kGroup) mma_commit(&tfull[slot]);
                        }
                        if (!ok) break;
                    }
                    mma_commit(&lempty[s]);
                }
                if (!C::kGroup && ok) mma_commit(&tfull[ti % 2u]);
            }
            // all issued MMAs complete before TMEM can be released
            mma_commit(done);
            int never = 0;
            mbar_wait(done, 0, &never, a.err);
        }
    } else if (warp >= kConvWarp0 && warp < kConvWarp0 + C::kConvWarps) {
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
                    const uint32_t a_cols = tmem_base + lane_addr + ao * C::kStageACols;
                    if constexpr (C::kG32Pack) {
                        // row r: 128 bytes, 16-byte chunk c = group c of the stage at
                        // position c ^ (r & 7)
                        const uint8_t* rowp = w_at(s) + r * 128;
                        if constexpr (C::kF16) {
                            const uint4 sc = *reinterpret_cast<const uint4*>(w_at(s) + 128 * 128 + r * 16);
                            const int sub = (warp - kConvWarp0) >> 2;  // which half of the groups
                            // this warp's 4 group scales (fp16 pairs): groups 4*sub .. 4*sub+3
                            const uint32_t sg01 = sub ? sc.z : sc.x, sg23 = sub ? sc.w : sc.y;
#pragma unroll
                            for (int cq = 0; cq < 2; ++cq) {  // two chunks = 32 columns
                                const int cp = 2 * sub + cq;
                                uint32_t o[32];
#pragma unroll
                                for (int h = 0; h < 2; ++h) {
                                    const int cl = 2 * cq + h;  // group within this warp's four
                                    const int c = 4 * sub + cl;
                                    const uint4 p = *reinterpret_cast<const uint4*>(rowp + ((c ^ (r & 7)) << 4));
                                    const uint32_t sw = cl < 2 ? sg01 : sg23;
                                    const __half2 s2 = __half2half2(__ushort_as_half(
                                        (unsigned short)((cl & 1) ? (sw >> 16) : (sw & 0xFFFFu))));
                                    g32_word_to_half(p.x, s2, o + 16 * h + 0);
                                    g32_word_to_half(p.y, s2, o + 16 * h + 4);
                                    g32_word_to_half(p.z, s2, o + 16 * h + 8);
                                    g32_word_to_half(p.w, s2, o + 16 * h + 12);
                                }
                                tmem_st32(a_cols + 32 * cp, o);
                            }
                        } else {
#pragma unroll
                            for (int jk = 0; jk < kKPS; ++jk) {  // k-block: chunks 4jk..4jk+3
                                uint32_t o[32];
#pragma unroll
                                for (int h = 0; h < 4; ++h) {
                                    const int c = 4 * jk + h;
                                    const uint4 p = *reinterpret_cast<const uint4*>(rowp + ((c ^ (r & 7)) << 4));
                                    g32_word_to_i8(p.x, o + 8 * h + 0);
                                    g32_word_to_i8(p.y, o + 8 * h + 2);
                                    g32_word_to_i8(p.z, o + 8 * h + 4);
                                    g32_word_to_i8(p.w, o + 8 * h + 6);
                                }
                                tmem_st32(a_cols + 32 * jk, o);
                            }
                        }
                    } else {
#pragma unroll
                        for (int jk = 0; jk < kKPS; ++jk) {
                            // row r of the k-block: 64 bytes in four 16-byte chunks,
                            // chunk c stored at position c ^ ((r >> 1) & 3) (conflict-free)
                            const uint8_t* rowp = w_at(s) + jk * (kTileRows * kKBlock / 2) + r * 64;
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
                            tmem_st32(a_cols + 32 * jk, o);
                        }
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ofull[ao]);
                }
            }
        }
    } else if (C::kGroup && warp == C::kStoreWarp) {
        if constexpr (Lay::kStaged) {
        // ------------------------------------------------------------ store warp
        // Exact group path: each finished tile's outputs, staged by the epilogue
        // warps as [NT tokens][128 channels] f32, go to global memory as one
        // bulk copy per token row (gate/up tiles: a gate and an up half), so the
        // epilogue warps never stall on global stores.
        if (lane == 0 && EPI != kEpiAcc) {
            uint32_t ts = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++ts) {
                if (!mbar_wait(sfull, ts & 1u, abort_flag, a.err)) break;
                const TileCoord c = decode_tile(t, tb, tcnt, E);
                const int row0 = offs[c.e] + c.mt * NT;
                const int nvalid = min(NT, offs[c.e + 1] - row0);
                for (int j = 0; j < nvalid; ++j) {
                    const int orow = (EPI == kEpiStore && a.out_rows) ? a.out_rows[row0 + j] : row0 + j;
                    float* dst = a.out + (size_t)orow * a.ldo;
                    const float* src = stg + j * kTileRows;
                    if (EPI == kEpiGateUp) {
                        const int cols = min(64, a.n_valid - c.rt * 64);
                        bulk_s2g(dst + c.rt * 64, src, (uint32_t)cols * 4u);
                        bulk_s2g(dst + a.n_valid + c.rt * 64, src + 64, (uint32_t)cols * 4u);
                    } else {
                        const int cols = min(kTileRows, a.n_valid - c.rt * kTileRows);
                        bulk_s2g(dst + c.rt * kTileRows, src, (uint32_t)cols * 4u);
                    }
                }
                bulk_commit();
                bulk_wait_read();
                mbar_arrive(sempty);
            }
            bulk_wait_all();
        }
        }  // kStaged
    } else if (warp >= C::kEpiWarp0) {
        // ------------------------------------------------------------ epilogue
        const int half = (warp - C::kEpiWarp0) >> 2;  // column half (0..1)
        const int r = quad * 32 + lane;             // weight row within the tile = TMEM lane
        const int c0 = half * C::kHalf;             // first token column of this warp
        if constexpr (C::kGroup) {
            // Exact group path. A tile's coordinates are worked out, and its
            // activation scales loaded, during the tile before (between its first
            // TMEM loads and their wait): nothing at a tile boundary waits for
            // memory or for the binary search of the tile table.
            struct TileInfo {
                int row0, nvalid;
                int oc;    // this lane's output column (gate | up rows: up at n + channel), -1: none
                float sx;  // lane q: the activation scale of token column c0 + q
            };
            auto tile_info = [&](int t) -> TileInfo {
                TileInfo ti_{0, 0, -1, 0.0f};
                if (t >= total) return ti_;
                const TileCoord c = decode_tile(t, tb, tcnt, E);
                ti_.row0 = offs[c.e] + c.mt * NT;
                ti_.nvalid = min(NT, offs[c.e + 1] - ti_.row0);
                const bool swiglu_tile = (EPI == kEpiGateUp) || (EPI == kEpiAcc && a.swiglu_layout);
                const bool is_up = swiglu_tile && r >= 64;
                const int col = swiglu_tile ? c.rt * 64 + (r & 63) : c.rt * kTileRows + r;
                if (col < a.n_valid) ti_.oc = is_up ? a.n_valid + col : col;
                if (EPI != kEpiAcc && lane < C::kHalf && c0 + lane < ti_.nvalid)
                    ti_.sx = __ldg(a.act_scale + ti_.row0 + c0 + lane);
                return ti_;
            };
            TileInfo cur = tile_info(blockIdx.x), nxt = cur;
            uint32_t it = 0, ist = 0, ts = 0;  // k-blocks, load stages, staged tiles
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                const int row0 = cur.row0, nvalid = cur.nvalid, ocol = cur.oc;
                const bool col_ok = cur.oc >= 0;
                bool side_done = false;
                auto side = [&]() { nxt = tile_info(t + gridDim.x); };
                float2 facc[C::kHalf / 2];
#pragma unroll
                for (int q = 0; q < C::kHalf / 2; ++q) facc[q] = make_float2(0.0f, 0.0f);
                const bool active = c0 < nvalid;  // idle warps still take part in the handshakes
                for (int st = 0; st < kstages && ok; ++st, ++ist) {
                    float2 sg[4];
#pragma unroll 1
                    for (int jk = 0; jk < kKPS; ++jk, ++it) {
                        const int kb = st * kKPS + jk;
                        const uint32_t slot = it % C::kNSlot;
                        if (!mbar_wait(&tfull[slot], (it / C::kNSlot) & 1u, abort_flag, a.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        if (jk == 0) {
                            // the stage's 8 group scales of row r (k-block jk, group j at
                            // 4 * jk + j) from the load stage, whose refill waits for
                            // every epilogue warp; the 1/16 of the W4 codes folded in
                            const uint8_t* ws = w_at(ist % SL) + 128 * 128;
                            const uint4 sc = *reinterpret_cast<const uint4*>(ws + r * 16);
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&lempty[ist % SL]);
                            const uint32_t w[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                sg[i] = __fmul2_rn(__half22float2(*reinterpret_cast<const __half2*>(&w[i])),
                                                   make_float2(0.0625f, 0.0625f));
                        }
                        const float2 sga = jk ? sg[2] : sg[0];  // groups 0, 1 of this k-block
                        const float2 sgb = jk ? sg[3] : sg[1];  // groups 2, 3
                        const uint32_t sbase = acc_base + lane_addr + slot * C::kSlotCols + c0;
                        // rounds of 8 token columns x 4 groups bound the registers; each
                        // round is loaded, re-armed and folded into its columns' sums
                        // (the group order per column stays 0..3)
                        constexpr int kRound = C::kHalf < 8 ? C::kHalf : 8;
#pragma unroll
                        for (int r0 = 0; r0 < C::kHalf && active; r0 += kRound) {
                            uint32_t v[4][kRound];
#pragma unroll
                            for (int j = 0; j < 4; ++j) tmem_ld<kRound>(sbase + j * NT + r0, v[j]);
                            if (!side_done) {
                                // in the shadow of the loads: the previous tile's
                                // outputs, the next tile's coordinates
                                side();
                                side_done = true;
                            }
                            tmem_wait_ld();
#pragma unroll
                            for (int j = 0; j < 4; ++j) tmem_ld_pin(v[j]);
                            if (EPI == kEpiAcc) {
#pragma unroll
                                for (int j = 0; j < 4; ++j)
#pragma unroll
                                    for (int q = 0; q < kRound; ++q)
                                        if (c0 + r0 + q < nvalid && col_ok)
                                            a.acc_out[((size_t)(row0 + c0 + r0 + q) * (a.kblocks * 4) + kb * 4 +
                                                       j) * a.acc_ld + ocol] =
                                                (int)(v[j][q] - kMagicBits) >> 4;
                            } else {
                                // the buffer holds the int32 0x4B400000 + 16 * acc, whose
                                // bits are the float 12582912 + 16 * acc (|16 * acc| < 2^22)
                                const float2 nm = make_float2(-kMagic, -kMagic);
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    const float2 sp = (j >> 1) ? sgb : sga;
                                    const float sj = (j & 1) ? sp.y : sp.x;
                                    const float2 s2 = make_float2(sj, sj);
#pragma unroll
                                    for (int q = 0; q < kRound / 2; ++q) {
                                        const float2 d = __fadd2_rn(
                                            make_float2(__uint_as_float(v[j][2 * q]),
                                                        __uint_as_float(v[j][2 * q + 1])),
                                            nm);
                                        facc[r0 / 2 + q] = __ffma2_rn(d, s2, facc[r0 / 2 + q]);
                                    }
                                }
                            }
                        }
                        {
                            const uint32_t sb = acc_base + lane_addr + slot * C::kSlotCols + c0;
#pragma unroll
                            for (int j = 0; j < 4; ++j) tmem_fill<C::kHalf>(sb + j * NT, kMagicBits);
                            tmem_wait_st();
                        }
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[slot]);
                        if (!side_done) {  // a warp with no valid column loads nothing
                            side();
                            side_done = true;
                        }
                    }
                }
                if (!ok) break;
                if (Lay::kStaged) {
                    // stage the dequantised tile for the store warp (its previous
                    // tile's copies have read the buffer once sempty completes)
                    if (!mbar_wait(sempty, (ts & 1u) ^ 1u, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
#pragma unroll
                    for (int q = 0; q < C::kHalf; ++q)
                        stg[(c0 + q) * kTileRows + r] = __fmul_rn((q & 1) ? facc[q >> 1].y : facc[q >> 1].x,
                                                                  __shfl_sync(0xffffffffu, cur.sx, q));
                    fence_proxy_async_smem();  // generic writes -> the bulk copies' reads
                    __syncwarp();
                    if (lane == 0) mbar_arrive(sfull);
                    ++ts;
                } else if (EPI != kEpiAcc) {
#pragma unroll
                    for (int q = 0; q < C::kHalf; ++q) {
                        const int j = c0 + q;
                        const float val = __fmul_rn((q & 1) ? facc[q >> 1].y : facc[q >> 1].x,
                                                    __shfl_sync(0xffffffffu, cur.sx, q));
                        if (j < nvalid && col_ok) {
                            const int orow = (EPI == kEpiStore && a.out_rows) ? a.out_rows[row0 + j] : row0 + j;
                            a.out[(size_t)orow * a.ldo + ocol] = val;
                        }
                    }
                }
                cur = nxt;
            }
            if (!ok) *abort_flag = 1;
        } else {
        // the activation scales of a tile (lane q: token column c0 + q), loaded
        // a whole tile ahead of use: at a tile boundary the epilogue then
        // reads nothing from global memory before its first accumulator
        auto tile_sx = [&](int t) -> float {
            if (t >= total) return 0.0f;
            const TileCoord c = decode_tile(t, tb, tcnt, E);
            const int row0 = offs[c.e] + c.mt * NT;
            const int nvalid = min(NT, offs[c.e + 1] - row0);
            return (lane < C::kHalf && c0 + lane < nvalid) ? __ldg(a.act_scale + row0 + c0 + lane) : 0.0f;
        };
        float next_sx = tile_sx(blockIdx.x);
        uint32_t ti = 0;  // tiles seen
        bool ok = true;
        for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++ti) {
            const TileCoord c = decode_tile(t, tb, tcnt, E);
            const int m_e = offs[c.e + 1] - offs[c.e];
            const int row0 = offs[c.e] + c.mt * NT;
            const int nvalid = min(NT, m_e - c.mt * NT);
            const float my_sx = next_sx;
            next_sx = tile_sx(t + gridDim.x);
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
            const int ocol = is_up ? a.n_valid + col : col;  // gate | up halves of a row


            float wscale_pc = 0.0f;
            if (!C::kF16) {
                const float* sp = reinterpret_cast<const float*>(
                    reinterpret_cast<const uint8_t*>(a.wscale) + (size_t)c.e * a.ws_expert_stride +
                    (size_t)c.rt * a.ws_tile_stride);
                wscale_pc = sp[r];
            }
            const uint32_t buf = ti % 2u;
            if (!mbar_wait(&tfull[buf], (ti / 2u) & 1u, abort_flag, a.err)) break;
            tc_fence_after();
            // the warp's columns in chunks of at most 32 (registers)
            constexpr int kChunk = C::kHalf < 32 ? C::kHalf : 32;
            uint32_t v[C::kHalf];
#pragma unroll
            for (int q0 = 0; q0 < C::kHalf; q0 += kChunk) {
                uint32_t (&vc)[kChunk] = *reinterpret_cast<uint32_t(*)[kChunk]>(v + q0);
                tmem_ld<kChunk>(acc_base + lane_addr + buf * NT + c0 + q0, vc);
            }
            tmem_wait_ld();
            tmem_ld_pin(v);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
#pragma unroll
            for (int q = 0; q < C::kHalf; ++q) {
                const int j = c0 + q;
                if (EPI == kEpiAcc) {
                    int acc = (int)v[q];
                    if (C::kW4) acc >>= 4;
                    if (j < nvalid && col_ok) a.acc_out[(size_t)(row0 + j) * a.acc_ld + ocol] = acc;
                } else {
                    const float sxq = __shfl_sync(0xffffffffu, my_sx, q);
                    float val;
                    if (C::kF16) {
                        val = __fmul_rn(__uint_as_float(v[q]), sxq);
                    } else {
                        int acc = (int)v[q];
                        if (C::kW4) acc >>= 4;
                        val = __fmul_rn(__fmul_rn(__int2float_rn(acc), sxq), wscale_pc);
                    }
                    if (j < nvalid && col_ok) {
                        const int orow = (EPI == kEpiStore && a.out_rows) ? a.out_rows[row0 + j] : row0 + j;
                        a.out[(size_t)orow * a.ldo + (EPI == kEpiGateUp ? ocol : col)] = val;
                    }
                }
            }
        }
        if (!ok) *abort_flag = 1;
        }  // per-channel formats
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kAllocCols);
    }
}

template <int FMT, int EPI, int NT>
static size_t gemm_smem_bytes(int E) {
    using C = GemmCfg<FMT, NT>;
    size_t b = 1024;  // alignment slack
    using Lay = GemmLayout<FMT, EPI, NT>;
    b += (size_t)Lay::kLoadStages * C::kLoadBytes;
    b += sizeof(uint64_t) * (2 * Lay::kLoadStages + (C::kAStages > 0 ? C::kAStages : 1) +
                             2 * C::kNSlot + 3);
    b += Lay::kStgBytes;
    b += sizeof(int) * (3 * (size_t)E + 3);
    // one CTA per SM: the kernel allocates all 512 TMEM columns
    // one CTA per SM (it allocates all 512 TMEM columns) unless two share it
    return (C::kCtasPerSm == 1 && b < 120 * 1024) ? 120 * 1024 : b;
}

template <int FMT, int EPI, int NT>
static int launch_gemm_t(const CUtensorMap& map, const GemmArgs& a, int num_sms,
                         cudaStream_t s) {
    const size_t smem = gemm_smem_bytes<FMT, EPI, NT>(a.num_experts);
    if (smem > 227 * 1024) return -1;
    cudaFuncSetAttribute(grouped_gemm_kernel<FMT, EPI, NT>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const long upper = ((long)(a.max_rows + NT - 1) / NT + a.num_experts) * a.row_tiles;
    const long slots = (long)num_sms * GemmCfg<FMT, NT>::kCtasPerSm;
    const int grid = (int)(upper < slots ? (upper > 0 ? upper : 1) : slots);
    grouped_gemm_kernel<FMT, EPI, NT><<<grid, GemmCfg<FMT, NT>::kThreads, smem, s>>>(map, a);
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
    {
        switch (epi) {
            case kEpiGateUp: return launch_gemm_nt<FMT, kEpiGateUp>(map, a, nt, num_sms, s);
            case kEpiStore: return launch_gemm_nt<FMT, kEpiStore>(map, a, nt, num_sms, s);
            case kEpiAcc:
                if constexpr (FMT != kFmtW4G32H) return launch_gemm_nt<FMT, kEpiAcc>(map, a, nt, num_sms, s);
                return -1;
            default: return -1;
        }
    }
}

int launch_gemm(const CUtensorMap& map, const GemmArgs& a, int fmt, int epi, int nt,
                int num_sms, cudaStream_t s) {
    switch (fmt) {
        case kFmtW4G32: return launch_gemm_epi<kFmtW4G32>(map, a, epi, nt, num_sms, s);
        case kFmtW4G32H: return launch_gemm_epi<kFmtW4G32H>(map, a, epi, nt, num_sms, s);
        case kFmtW4PC: return launch_gemm_epi<kFmtW4PC>(map, a, epi, nt, num_sms, s);
        case kFmtW8PC: return launch_gemm_epi<kFmtW8PC>(map, a, epi, nt, num_sms, s);
        default: return -1;
    }
}

}  // namespace moe
