// gelu.cuh -- GELU(tanh) as the reference computes it (geluKernel,
// transformer.cu:68-75; the ffnUpKernel epilogue, :276-277), shared by the
// bias+GELU row kernel and the up-projection GEMM epilogue.  The cubic term
// is fused as the reference's nvcc build fuses it; tanhf is CUDA's (no
// fast-math):
//   out = u * (0.5f * (1.0f + tanhf(0.7978845608f * (u + 0.044715f*u*u*u))))
#pragma once

#include "gbx_common.cuh"

namespace gbx {

__device__ __forceinline__ float gelu_tanh(float u)
{
    const float inner = fmaf((0.044715f * u) * u, u, u);
    return u * (0.5f * (1.0f + tanhf(0.7978845608f * inner)));
}

// The same operations on two elements at a time: sm_100's packed fp32
// instructions (__fmul2_rn / __ffma2_rn / __fadd2_rn) round each component
// exactly as the scalar __fmul_rn / __fmaf_rn / __fadd_rn do, so the result
// is bit-identical to gelu_tanh on each component, in half the arithmetic
// instructions (tanhf itself stays scalar).
__device__ __forceinline__ float2 gelu_tanh2(float2 u)
{
    const float2 t = __fmul2_rn(__fmul2_rn(make_float2(0.044715f, 0.044715f), u), u);
    const float2 k = __fmul2_rn(make_float2(0.7978845608f, 0.7978845608f), __ffma2_rn(t, u, u));
    const float2 th = make_float2(tanhf(k.x), tanhf(k.y));
    return __fmul2_rn(u, __fmul2_rn(make_float2(0.5f, 0.5f), __fadd2_rn(make_float2(1.0f, 1.0f), th)));
}

__device__ __forceinline__ float4 gelu4(float4 u)
{
    return cat2(gelu_tanh2(lo2(u)), gelu_tanh2(hi2(u)));
}

}  // namespace gbx
