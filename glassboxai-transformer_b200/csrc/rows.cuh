// rows.cuh -- the row-group engine shared by LayerNorm and softmax.
//
// A row of n4 = len/4 float4s is owned by a group of TPR consecutive threads
// (TPR a power of two); thread `lane` of the group holds float4s
// lane, lane+TPR, ..., lane+(V4-1)*TPR in registers, so a warp's loads of one
// k are 32 consecutive 16-byte pieces (coalesced) and the row is read from
// HBM exactly once.  A CTA of kRowCTA threads holds kRowCTA/TPR rows and walks
// the row space grid-stride, so the loop bound is uniform across the CTA and
// __syncthreads is legal inside it.
//
// Shape selection (row_shape): rows of up to 32 float4s use one group of
// pow2ceil(n4) threads with one float4 each; longer rows use 32..256 threads
// with V4 <= 8 float4s each, which keeps the row (plus the residual operand
// while it is being added) in registers for rows of up to 8192 floats.
#pragma once

#include "gbx_common.cuh"

namespace gbx {

constexpr int kRowCTA = 256;
constexpr int kRowMaxV4 = 8;
constexpr int kRowMaxTPR = 256;

struct RowShape {
    int tpr, v4;
};

// Returns false when the row is too long for the register path.
inline bool row_shape(int n4, RowShape* s)
{
    if (n4 <= 0) return false;
    if (n4 <= 32) {
        int t = 1;
        while (t < n4) t <<= 1;
        s->tpr = t;
        s->v4 = 1;
        return true;
    }
    int t = 32;
    while ((n4 + t - 1) / t > kRowMaxV4) t <<= 1;
    if (t > kRowMaxTPR) return false;
    s->tpr = t;
    s->v4 = (n4 + t - 1) / t;
    return true;
}

// Sum / max over the TPR threads of this thread's row group.  For TPR > 32
// the warps of a group combine through `red` (kRowCTA/32 floats); every
// thread of the group adds the partials in the same order, so all of them
// get the same value.  Callers alternate two `red` buffers between
// consecutive reductions: the barrier inside each reduction then separates
// the reads of one buffer from its next writes.
template <int TPR>
__device__ __forceinline__ float row_sum(float v, float* red)
{
    if constexpr (TPR <= 32) {
        return group_sum<TPR>(v);
    } else {
        v = group_sum<32>(v);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
        __syncthreads();
        const int first = (threadIdx.x / TPR) * (TPR / 32);
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < TPR / 32; ++w) s += red[first + w];
        return s;
    }
}

template <int TPR>
__device__ __forceinline__ float row_max(float v, float* red)
{
    if constexpr (TPR <= 32) {
        return group_max<TPR>(v);
    } else {
        v = group_max<32>(v);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
        __syncthreads();
        const int first = (threadIdx.x / TPR) * (TPR / 32);
        float m = red[first];
#pragma unroll
        for (int w = 1; w < TPR / 32; ++w) m = fmaxf(m, red[first + w]);
        return m;
    }
}

// Block-wide sum for the general (any length) kernels: every thread gets the
// total.  `red` holds kRowCTA/32 floats; same alternation rule as above.
__device__ __forceinline__ float block_sum(float v, float* red)
{
    v = group_sum<32>(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kRowCTA / 32; ++w) s += red[w];
    return s;
}

__device__ __forceinline__ float block_max(float v, float* red)
{
    v = group_max<32>(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = red[0];
#pragma unroll
    for (int w = 1; w < kRowCTA / 32; ++w) m = fmaxf(m, red[w]);
    return m;
}

// Expands F(TPR, V4) for every shape row_shape can return; evaluates to the
// call's result, or `fallback` for an impossible shape.
#define GBX_ROW_DISPATCH(shape, F, fallback)                                                   \
    [&]() {                                                                                    \
        switch ((shape).tpr) {                                                                 \
        case 1: return F(1, 1);                                                                \
        case 2: return F(2, 1);                                                                \
        case 4: return F(4, 1);                                                                \
        case 8: return F(8, 1);                                                                \
        case 16: return F(16, 1);                                                              \
        case 32:                                                                               \
            switch ((shape).v4) {                                                              \
            case 1: return F(32, 1);                                                           \
            case 2: return F(32, 2);                                                           \
            case 3: return F(32, 3);                                                           \
            case 4: return F(32, 4);                                                           \
            case 5: return F(32, 5);                                                           \
            case 6: return F(32, 6);                                                           \
            case 7: return F(32, 7);                                                           \
            case 8: return F(32, 8);                                                           \
            }                                                                                  \
            break;                                                                             \
        case 64:                                                                               \
            switch ((shape).v4) {                                                              \
            case 5: return F(64, 5);                                                           \
            case 6: return F(64, 6);                                                           \
            case 7: return F(64, 7);                                                           \
            case 8: return F(64, 8);                                                           \
            }                                                                                  \
            break;                                                                             \
        case 128:                                                                              \
            switch ((shape).v4) {                                                              \
            case 5: return F(128, 5);                                                          \
            case 6: return F(128, 6);                                                          \
            case 7: return F(128, 7);                                                          \
            case 8: return F(128, 8);                                                          \
            }                                                                                  \
            break;                                                                             \
        case 256:                                                                              \
            switch ((shape).v4) {                                                              \
            case 5: return F(256, 5);                                                          \
            case 6: return F(256, 6);                                                          \
            case 7: return F(256, 7);                                                          \
            case 8: return F(256, 8);                                                          \
            }                                                                                  \
            break;                                                                             \
        }                                                                                      \
        return (fallback);                                                                     \
    }()

}  // namespace gbx
