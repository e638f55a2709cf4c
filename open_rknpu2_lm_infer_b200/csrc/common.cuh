// Device-side building blocks for the sm_100a MoE kernels: mbarriers with
// bounded waits, bulk/tensor async copies (each into this CTA only), tcgen05
// TMEM allocation, MMA issue and TMEM loads, written as inline PTX.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace moe {

// Error bits written to the workspace status word (atomicOr). Host code maps
// them to MOE_B200_ERR_DEVICE_* return codes.
enum : uint32_t {
    kErrWaitTimeout = 1u << 0,   // an mbarrier wait gave up (pipeline stalled)
    kErrBadExpert = 1u << 1,     // an expert id outside [0, experts)
    kErrNonFinite = 1u << 2,     // non-finite router logit or activation scale
    kErrBadRoute = 1u << 3,      // routing weight negative or NaN
    kErrCapacity = 1u << 4,      // more rows than the workspace holds
};

// Upper bound for any spin on an mbarrier: ~2 s of wall time measured by the
// global timer. After it the waiter records kErrWaitTimeout and gives up.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

// try_wait with a suspend-time hint: a waiting thread sleeps until the phase
// completes (or the hint elapses) instead of spinning and taking issue slots
// from the single-thread producer and MMA roles.
constexpr uint32_t kSuspendHintNs = 1000000;  // 1 ms upper bound per try

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}

// Bounded wait on a phase parity. Returns false (and flags the error) when the
// limit passes or when another role of the CTA has already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag, uint32_t* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_timer_ns() - start > kWaitLimitNs) {
            *abort_flag = 1;
            atomicOr(err, kErrWaitTimeout);
            return false;
        }
    }
}

// try_wait without a suspend-time hint: returns when the phase completes or
// after a short system-dependent time.
__device__ __forceinline__ bool mbar_poll(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// The bounded wait of the pipelined kernels: polls without a suspend hint (a
// thread suspended with a long hint was measured to resume well after the
// phase completed), checks the abort flag and the time limit every 64 polls.
static __device__ __noinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity,
                                                   volatile int* abort_flag, uint32_t* err) {
    const uint64_t start = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_poll(bar, parity)) return true;
        if ((i & 63u) == 0u) {
            if (*abort_flag) return false;
            if (global_timer_ns() - start > kWaitLimitNs) {
                *abort_flag = 1;
                atomicOr(err, kErrWaitTimeout);
                return false;
            }
        }
    }
}

// Only the first poll inline: a loop issuing MMAs then holds one try_wait and
// a branch per wait (an inline spin loop measured ~2x the per-MMA issue cost
// of the issuing thread, even when never entered).
__device__ __forceinline__ bool mbar_wait_fast(uint64_t* bar, uint32_t parity,
                                               volatile int* abort_flag, uint32_t* err) {
    if (mbar_poll(bar, parity)) return true;
    return mbar_wait_spin(bar, parity, abort_flag, err);
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while its predecessor still runs. pdl_wait() blocks
// until the predecessor grid has completed with its memory visible (it returns
// at once when there is no such predecessor); pdl_trigger() lets this grid's
// own dependents begin to launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Generic-proxy smem writes -> visible to the async proxy (tensor core reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completing on an mbarrier.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled tensor copy global -> this CTA's shared memory. x must be a multiple
// of 16 bytes for the 8-bit element type used here.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 3-D tiled tensor copy global -> this CTA's shared memory.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, int32_t z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// 1-D bulk copy of this CTA's shared memory to global memory (bulk async-group
// completion: bulk_commit, then bulk_wait_read before the source is reused).
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_s2g(void* gmem_dst, const void* smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
                 "r"(smem_u32(smem_src)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the copies committed so far have read their shared-memory sources
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// ... and completed their writes
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 (5th-generation tensor core, tensor memory) -------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, one CTA.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, int8 x int8 -> int32, one CTA. A is K-major
// in tensor memory: lane m holds row m, each 32-bit column 4 consecutive k.
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 consecutive 32-bit columns of this thread's lane from registers.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// Arrive on an mbarrier once every previously issued tcgen05 op of this
// thread has completed (single-CTA form).
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The registers a tcgen05.ld writes hold their values only after
// tcgen05.wait::ld, but the compiler sees them as outputs of the load itself
// and may schedule arithmetic on them before the wait. Passing each register
// through an empty volatile asm after the wait pins every use behind it.
template <int N>
__device__ __forceinline__ void tmem_ld_pin(uint32_t (&r)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// 32 lanes x 8 columns of 32-bit: thread i gets lane (base+i), 8 columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%"
        "14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}

// N consecutive 32-bit columns of this thread's lane (N = 4, 8, 16 or 32).
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 4) {
        tmem_ld4(taddr, r);
    } else if constexpr (N == 8) {
        tmem_ld8(taddr, r);
    } else if constexpr (N == 16) {
        tmem_ld16(taddr, r);
    } else {
        static_assert(N == 32, "tmem_ld width");
        tmem_ld32(taddr, r);
    }
}

// Fill N consecutive 32-bit columns of this thread's lane with one value.
template <int N>
__device__ __forceinline__ void tmem_fill(uint32_t taddr, uint32_t v) {
    if constexpr (N == 4) {
        asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%1,%1,%1};" ::"r"(taddr),
                     "r"(v)
                     : "memory");
    } else if constexpr (N == 8) {
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
            "r"(v)
            : "memory");
    } else if constexpr (N == 16) {
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
            "%1,%1,%1};" ::"r"(taddr),
            "r"(v)
            : "memory");
    } else {
        static_assert(N == 32, "tmem_fill width");
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
            "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
            "r"(v)
            : "memory");
    }
}

__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored in the
// 128-byte swizzle layout: rows of 128 bytes, 8-row atoms of 1024 bytes.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);        // start address
    d |= (uint64_t)(1u) << 16;                            // leading byte offset (16 B)
    d |= (uint64_t)(1024u >> 4) << 32;                    // stride byte offset: 8 rows
    d |= (uint64_t)(1u) << 46;                            // descriptor version (sm_100)
    d |= (uint64_t)(2u) << 61;                            // SWIZZLE_128B
    return d;
}

// Instruction descriptor: kind::i8, signed A and B, int32 accumulate,
// both operands K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// Order-preserving 32-bit key of Rust's f32::total_cmp.
__device__ __forceinline__ int32_t total_key(float v) {
    int32_t b = __float_as_int(v);
    return b ^ (int32_t)((uint32_t)(b >> 31) >> 1);
}
// total_key is an involution on the bit pattern: the key's value back.
__device__ __forceinline__ float key_value(int32_t key) {
    return __int_as_float(key ^ (int32_t)((uint32_t)(key >> 31) >> 1));
}

// f32 exp for the sigmoid gates: the double-precision exp rounded once to
// f32, i.e. the correctly rounded f32 result up to double rounding. The
// glibc expf (the C library the reference builds against) differs from it by
// one ulp on about 1 in 13,000 f32 arguments.
__device__ __forceinline__ float exp_f32(float x) { return __double2float_rn(exp((double)x)); }

// sigmoid of src/ops/activation.rs:7-14: exp's argument is kept <= 0.
__device__ __forceinline__ float sigmoid_ref(float x) {
    if (x >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f32(-x)));
    const float e = exp_f32(x);
    return __fdiv_rn(e, __fadd_rn(1.0f, e));
}

// TF32 narrowing of the NPU linear (src/npu/tf32.rs): the low 13 mantissa
// bits are dropped (truncation, not rounding).
__device__ __forceinline__ float tf32_trunc(float v) {
    return __uint_as_float(__float_as_uint(v) & ~0x1FFFu);
}

}  // namespace moe
