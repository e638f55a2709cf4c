// Device-initiated expert-parallel exchange over NVLink peer memory.
//
// Every rank owns one exchange region, mapped into every other rank's address
// space (CUDA IPC, plain peer mappings):
//   recv_q      [world][cap][row_bytes]  rows from source s land in slot s
//   recv_scale  [world][cap] f32         their activation scales
//   recv_expert [world][cap] i32         their local expert ids
//   recv_cnt    [world] i32, recv_base [world] i32  rows sent by s, and the
//                                        sender's packed offset of that block
//   y_back      [cap][H] f32             expert rows returned to this rank, at
//                                        its own packed positions
//   flags_rows  [world] u64, flags_y [world] u64    the step number of the last
//                                        rows / y block a source finished
// A step: the sender copies each destination's block of packed rows straight
// into the destination's slot, then (last CTA, after a system-scope fence)
// stores the step number into the destination's flag for this source; the
// destination waits (bounded) until every source's flag reached the step.
// The y rows go back the same way. No host synchronisation: the split sizes
// stay on the device, so a whole layer step can be captured in a CUDA graph.
// A rank that does not arrive makes the others give up after the wait limit
// with kErrWaitTimeout in their status word; nothing spins without a bound.
#include "kernels.cuh"

namespace moe {

namespace {

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// The last CTA of the grid to get here returns true (its writes and everyone
// else's are then complete and fenced system-wide).
__device__ __forceinline__ bool grid_last(int* counter) {
    __shared__ int is_last;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(counter, 1);
        is_last = prev == (int)(gridDim.x * gridDim.y) - 1;
        if (is_last) *counter = 0;
    }
    __syncthreads();
    if (is_last) __threadfence_system();
    return is_last;
}

__global__ void ep_begin_kernel(uint64_t* step) { *step += 1; }

// grid (blocks, world destinations). Copies this rank's packed block for
// destination d into d's region, slot `rank`.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const ExchangeArgs a,
                                                          const int8_t* __restrict__ send_q,
                                                          const float* __restrict__ send_scale,
                                                          const int32_t* __restrict__ send_expert,
                                                          const int32_t* __restrict__ counts) {
    const int d = blockIdx.y;
    int off = 0;
    for (int j = 0; j < d; ++j) off += counts[j];
    const int cnt = counts[d];
    uint8_t* peer = a.peers[d];
    const bool fits = cnt >= 0 && cnt <= a.cap;
    if (!fits && blockIdx.x == 0 && threadIdx.x == 0) atomicOr(a.err, kErrCapacity);
    if (fits) {
        int8_t* rq = reinterpret_cast<int8_t*>(peer + a.off_q) + ((size_t)a.rank * a.cap) * a.row_bytes;
        float* rs = reinterpret_cast<float*>(peer + a.off_scale) + (size_t)a.rank * a.cap;
        int32_t* re = reinterpret_cast<int32_t*>(peer + a.off_expert) + (size_t)a.rank * a.cap;
        const int v16 = (int)(a.row_bytes / 16);
        const size_t total = (size_t)cnt * v16;
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
             i += (size_t)gridDim.x * blockDim.x) {
            const size_t row = i / v16, c = i % v16;
            reinterpret_cast<uint4*>(rq + row * a.row_bytes)[c] =
                reinterpret_cast<const uint4*>(send_q + (off + row) * a.row_bytes)[c];
        }
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cnt; i += gridDim.x * blockDim.x) {
            rs[i] = send_scale[off + i];
            re[i] = send_expert[off + i];
        }
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            reinterpret_cast<int32_t*>(peer + a.off_cnt)[a.rank] = cnt;
            reinterpret_cast<int32_t*>(peer + a.off_base)[a.rank] = off;
        }
    }
    if (grid_last(a.done) && threadIdx.x < a.world)
        st_release_sys(reinterpret_cast<uint64_t*>(a.peers[threadIdx.x] + a.off_flag_rows) + a.rank,
                       *a.step);
}

// One CTA: thread s waits until source s finished the step (bounded), then
// marks the received rows valid (mask 1) or padding (mask 0).
__global__ void ep_wait_kernel(const ExchangeArgs a, int which, float* mask) {
    __shared__ int ok_all;
    if (threadIdx.x == 0) ok_all = 1;
    __syncthreads();
    const uint64_t* flags =
        reinterpret_cast<const uint64_t*>(a.peers[a.rank] + (which == 0 ? a.off_flag_rows : a.off_flag_y));
    const uint64_t step = *a.step;
    if (threadIdx.x < a.world) {
        const uint64_t start = global_timer_ns();
        while (ld_acquire_sys(flags + threadIdx.x) < step) {
            if (global_timer_ns() - start > kWaitLimitNs) {
                atomicOr(a.err, kErrWaitTimeout);
                ok_all = 0;
                break;
            }
        }
    }
    __syncthreads();
    if (which != 0 || !mask) return;
    const int32_t* cnt = reinterpret_cast<const int32_t*>(a.peers[a.rank] + a.off_cnt);
    for (int i = threadIdx.x; i < a.world * a.cap; i += blockDim.x) {
        const int s = i / a.cap, r = i % a.cap;
        mask[i] = (ok_all && r < cnt[s]) ? 1.0f : 0.0f;
    }
}

// grid (blocks, world sources): expert rows of source s back to s's y_back at
// the sender's packed positions.
__global__ void __launch_bounds__(256) ep_return_kernel(const ExchangeArgs a,
                                                        const float* __restrict__ y) {
    const int s = blockIdx.y;
    const uint8_t* own = a.peers[a.rank];
    const int cnt = reinterpret_cast<const int32_t*>(own + a.off_cnt)[s];
    const int base = reinterpret_cast<const int32_t*>(own + a.off_base)[s];
    if (cnt >= 0 && cnt <= a.cap && base >= 0 && base + cnt <= a.cap) {
        float* dst = reinterpret_cast<float*>(a.peers[s] + a.off_y) + (size_t)base * a.H;
        const float* src = y + (size_t)s * a.cap * a.H;
        const size_t total = (size_t)cnt * a.H / 4;
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
             i += (size_t)gridDim.x * blockDim.x)
            reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
    } else if (blockIdx.x == 0 && threadIdx.x == 0) {
        atomicOr(a.err, kErrCapacity);
    }
    if (grid_last(a.done) && threadIdx.x < a.world)
        st_release_sys(reinterpret_cast<uint64_t*>(a.peers[threadIdx.x] + a.off_flag_y) + a.rank,
                       *a.step);
}

}  // namespace

void launch_ep_begin(uint64_t* step, cudaStream_t s) { ep_begin_kernel<<<1, 1, 0, s>>>(step); }

void launch_ep_dispatch(const ExchangeArgs& a, const int8_t* send_q, const float* send_scale,
                        const int32_t* send_expert, const int32_t* counts, cudaStream_t s) {
    ep_dispatch_kernel<<<dim3(a.blocks, a.world), 256, 0, s>>>(a, send_q, send_scale, send_expert,
                                                             counts);
}

void launch_ep_wait(const ExchangeArgs& a, int which, float* mask, cudaStream_t s) {
    ep_wait_kernel<<<1, 256, 0, s>>>(a, which, mask);
}

void launch_ep_return(const ExchangeArgs& a, const float* y, cudaStream_t s) {
    ep_return_kernel<<<dim3(a.blocks, a.world), 256, 0, s>>>(a, y);
}

}  // namespace moe
