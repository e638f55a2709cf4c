// Element-wise quantisation helpers shared by the dispatch kernels and the
// fused gate/up epilogue of the group-32 GEMM.
//
// Reference semantics (happyme531/open_rknpu2_lm_infer):
//   MoE A8   : s = maxabs/127, q = round-half-even(x / s), clamp +-127, zero
//              row -> s = 1 (llm_generated_docs/MOE_CPU_FUSION_20261023.md:13)
//   dense A8 : s = max(maxabs/127, FLT_MIN), q = round-half-away(x * (1/s))
//              (llm_generated_docs/MODELS.md:26)
//   SwiGLU   : h = (g / (1 + exp(-g))) * u, x86 native/cpu_kernels/swiglu.cpp:23-25
//              with the gate/up split of Cpu::swiglu (src/model/cpu.rs:269-294)
#pragma once
#include <cuda_fp16.h>
#include <float.h>

#include "kernels.cuh"

namespace moe {

__device__ __forceinline__ int quant_one(float x, float s, float inv, int rule) {
    float v = rule == kQuantMoe ? __fdiv_rn(x, s) : roundf(__fmul_rn(x, inv));
    int q = rule == kQuantMoe ? __float2int_rn(v) : (int)v;
    return q > 127 ? 127 : (q < -127 ? -127 : q);
}

__device__ __forceinline__ uint32_t quant4(float4 v, float s, float inv, int rule) {
    return (uint32_t)(quant_one(v.x, s, inv, rule) & 0xFF) |
           ((uint32_t)(quant_one(v.y, s, inv, rule) & 0xFF) << 8) |
           ((uint32_t)(quant_one(v.z, s, inv, rule) & 0xFF) << 16) |
           ((uint32_t)(quant_one(v.w, s, inv, rule) & 0xFF) << 24);
}

// The four int8 codes of a packed word as two fp16 pairs (exact: |q| <= 127),
// the activation operand of the fp16 tensor-core path of group-32 weights.
__device__ __forceinline__ uint2 codes_to_half4(uint32_t packed) {
    const __half2 a = __halves2half2(__int2half_rn((int8_t)(packed & 0xFF)),
                                     __int2half_rn((int8_t)((packed >> 8) & 0xFF)));
    const __half2 b = __halves2half2(__int2half_rn((int8_t)((packed >> 16) & 0xFF)),
                                     __int2half_rn((int8_t)(packed >> 24)));
    return make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}

__device__ __forceinline__ float amax4(float4 v) {
    return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

__device__ __forceinline__ float row_scale(float m, int rule) {
    if (m == 0.0f) return 1.0f;
    float s = __fdiv_rn(m, 127.0f);
    if (rule == kQuantDense && !(s >= FLT_MIN)) s = FLT_MIN;
    return s;
}

// h = (g / (1 + exp(-g))) * u with IEEE division and multiply (no contraction).
__device__ __forceinline__ float silu_mul(float g, float u) {
    const float d = __fadd_rn(1.0f, expf(-g));
    return __fmul_rn(__fdiv_rn(g, d), u);
}

}  // namespace moe
