// Pre-norm of the layer stack: RMSNorm (src/ops/norm.rs:81-106).
//
// y[r, i] = (x[r, i] * scale_r) * w_i, scale_r = 1 / sqrt(sum_i x[r, i]^2 / width + eps),
// w_i replaced by 1 + w_i for zero-centred weights. The reference sums the
// squares with an iterator sum, one row at a time: each product rounded, then
// added in column order. That sum is a chain of `width` dependent adds per
// row, so one lane owns one row: a warp stages 32 rows x 32 columns in shared
// memory (coalesced row reads), then every lane adds its own row's 32 squares
// in order. The output pass re-reads x row by row, coalesced, with the row's
// scale broadcast from its lane. Every step is the correctly rounded IEEE
// operation the reference performs (multiply, add, divide, square root), so
// the result is bit-exact.
#include "kernels.cuh"

namespace moe {

namespace {

__global__ void __launch_bounds__(32) rms_norm_kernel(const float* __restrict__ x,
                                                      const float* __restrict__ w, int rows,
                                                      int width, float eps, int zero_centered,
                                                      float* out) {
    __shared__ float tile[32][33];  // [row][column], padded: conflict-free both ways
    const int lane = threadIdx.x;
    const int r0 = blockIdx.x * 32;
    float sum = -0.0f;  // the reference's float sum starts from -0.0
    for (int c0 = 0; c0 < width; c0 += 32) {
        const int c = c0 + lane;
#pragma unroll 8
        for (int j = 0; j < 32; ++j) {
            const int r = r0 + j;
            tile[j][lane] = (r < rows && c < width) ? x[(size_t)r * width + c] : 0.0f;
        }
        __syncwarp();
        const int n = min(32, width - c0);
        for (int i = 0; i < n; ++i) {
            const float v = tile[lane][i];
            sum = __fadd_rn(sum, __fmul_rn(v, v));
        }
        __syncwarp();
    }
    const float scale =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)width), eps)));
    const int nr = min(32, rows - r0);
    for (int j = 0; j < nr; ++j) {
        const float sj = __shfl_sync(0xffffffffu, scale, j);
        const float* xr = x + (size_t)(r0 + j) * width;
        float* yr = out + (size_t)(r0 + j) * width;
        for (int i = lane; i < width; i += 32) {
            const float wv = zero_centered ? __fadd_rn(1.0f, w[i]) : w[i];
            yr[i] = __fmul_rn(__fmul_rn(xr[i], sj), wv);
        }
    }
}

}  // namespace

void launch_rms_norm(const float* x, const float* w, int rows, int width, float eps,
                     int zero_centered, float* out, cudaStream_t s) {
    rms_norm_kernel<<<(rows + 31) / 32, 32, 0, s>>>(x, w, rows, width, eps, zero_centered, out);
}

}  // namespace moe
