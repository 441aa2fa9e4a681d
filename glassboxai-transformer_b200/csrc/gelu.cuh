// gelu.cuh -- GELU(tanh) as the reference computes it (geluKernel,
// transformer.cu:68-75; the ffnUpKernel epilogue, :276-277), shared by the
// bias+GELU row kernel and the up-projection GEMM epilogue.  The cubic term
// is fused as the reference's nvcc build fuses it; tanhf is CUDA's (no
// fast-math):
//   out = u * (0.5f * (1.0f + tanhf(0.7978845608f * (u + 0.044715f*u*u*u))))
#pragma once

namespace gbx {

__device__ __forceinline__ float gelu_tanh(float u)
{
    const float inner = fmaf((0.044715f * u) * u, u, u);
    return u * (0.5f * (1.0f + tanhf(0.7978845608f * inner)));
}

}  // namespace gbx
