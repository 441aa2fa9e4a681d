// decode.cuh -- GGUF element decode shared by the embedding, dequant and
// logits kernels.  f16 follows the reference's GGUFLoader::float16ToFloat32
// (transformer.cu:508-527) bit for bit, including its quirks; bf16 is
// GGUFLoader::bfloat16ToFloat32 (:529-534), the 16 bits as the top half of an
// fp32.  Tables are read in 4-element words: one 16-byte load for f32, one
// 8-byte load for f16/bf16.
#pragma once

#include <cuda_fp16.h>

#include "gbx_common.cuh"

namespace gbx {

// GGUF dtype code -> template index.
enum { TF32 = 0, TF16 = 1, TBF16 = 2 };

// Reference float16ToFloat32 (transformer.cu:508-527), as fp32 bits:
// normal halves re-biased exactly; +-0 -> +0 (sign dropped, :514);
// subnormals mantissa * 2^-24 (exact); +-inf kept; any NaN -> 0x7fc00000 (:521).
__device__ __forceinline__ uint32_t f16_to_f32_bits(uint32_t h)
{
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1fu;
    const uint32_t man = h & 0x3ffu;
    const uint32_t normal = sign | ((ex + 112u) << 23) | (man << 13);
    const uint32_t sub = sign | __float_as_uint(__uint2float_rn(man) * 5.9604644775390625e-8f);
    const uint32_t infnan = man ? 0x7fc00000u : (sign | 0x7f800000u);
    return ex == 0 ? (man ? sub : 0u) : (ex == 31 ? infnan : normal);
}

__device__ __forceinline__ float f16_to_f32(uint32_t h) { return __uint_as_float(f16_to_f32_bits(h)); }

template <int T>
__device__ __forceinline__ float load1(const void* base, int64_t e)
{
    if (T == TF32) return __ldg(static_cast<const float*>(base) + e);
    uint32_t h = __ldg(static_cast<const unsigned short*>(base) + e);
    return T == TF16 ? f16_to_f32(h) : __uint_as_float(h << 16);
}

// Raw 4-element words: a float4 of an f32 table, a uint2 of an f16/bf16 one.
template <int T>
struct Raw4 {
    using type = uint2;
};
template <>
struct Raw4<TF32> {
    using type = float4;
};

template <int T>
__device__ __forceinline__ typename Raw4<T>::type load_raw4(const void* base, int64_t e)
{
    if constexpr (T == TF32) return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(base) + e));
    else return __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + e));
}

template <int T>
__device__ __forceinline__ typename Raw4<T>::type zero_raw4()
{
    if constexpr (T == TF32) return make_float4(0.f, 0.f, 0.f, 0.f);
    else return make_uint2(0u, 0u);
}

template <int T>
__device__ __forceinline__ float4 decode4(typename Raw4<T>::type w)
{
    if constexpr (T == TF32) {
        return w;
    } else if constexpr (T == TF16) {
        return make_float4(f16_to_f32(w.x & 0xffffu), f16_to_f32(w.x >> 16), f16_to_f32(w.y & 0xffffu),
                           f16_to_f32(w.y >> 16));
    } else {
        return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u),
                           __uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u));
    }
}

// The same 4 elements through the hardware conversion (cvt.f32.f16, exact
// for every finite half and for +-inf), without the reference's two f16
// quirks: -0 stays -0 and a NaN keeps its payload.  For consumers that add
// the decoded value (the embedding sum, the logits dot product) only the
// sign of a zero sum can differ, and the embedding restores it (see
// embed_vec4_kernel); a GPU fp32 add returns the canonical NaN whatever the
// payload.
template <int T>
__device__ __forceinline__ float4 decode4_arith(typename Raw4<T>::type w)
{
    if constexpr (T == TF16) {
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
        return make_float4(lo.x, lo.y, hi.x, hi.y);
    } else {
        return decode4<T>(w);
    }
}

inline int dtype_index(int dt)
{
    switch (dt) {
    case GBX_DT_F32: return TF32;
    case GBX_DT_F16: return TF16;
    case GBX_DT_BF16: return TBF16;
    default: return -1;
    }
}

constexpr int kLogitsMaxRows = 8;   // hidden rows per pass of gbx_logits

}  // namespace gbx
