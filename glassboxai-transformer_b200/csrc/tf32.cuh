// tf32.cuh -- the tf32 pair of an fp32 value, as gbx_linear's operands carry
// it: hi = x rounded to tf32 (10 explicit mantissa bits, to nearest, ties
// away from zero; the hardware cvt.rna.tf32.f32), lo = (x - hi) rounded the
// same way.  hi + lo carries 21 of x's 24 significant bits.  Where rounding
// x overflows to infinity, hi is x truncated instead; lo is 0 when hi is not
// finite.
#pragma once

#include <stdint.h>

namespace gbx {

__device__ __forceinline__ float to_tf32(float x)
{
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__device__ __forceinline__ void split_value(float x, float& hi, float& lo)
{
    hi = to_tf32(x);
    if (isinf(hi) && !isinf(x)) hi = __uint_as_float(__float_as_uint(x) & 0xffffe000u);   // rounding overflowed
    lo = isfinite(hi) ? to_tf32(x - hi) : 0.0f;
}

__device__ __forceinline__ void split4(float4 v, float4& hi, float4& lo)
{
    split_value(v.x, hi.x, lo.x);
    split_value(v.y, hi.y, lo.y);
    split_value(v.z, hi.z, lo.z);
    split_value(v.w, hi.w, lo.w);
}

}  // namespace gbx
