// rows.cuh -- the row-group engine shared by LayerNorm and softmax.
//
// A row of n4 = len/4 float4s is owned by a group of TPR consecutive threads
// (TPR a power of two); thread `lane` of the group holds float4s
// lane, lane+TPR, ..., lane+(V4-1)*TPR in registers, so a warp's loads of one
// k are 32 consecutive 16-byte pieces (coalesced) and the row is read from
// HBM exactly once.
//
// Launch shape: one full grid, each CTA owning RPC = CTA/TPR consecutive rows
// (no grid-stride loop; CTAs of 128 or 256 threads, RowCTA and
// small_row_grid below).  Measured on B200, a full grid of short-lived CTAs
// streams these rows at 95-106% of the measured copy bandwidth, where a
// persistent grid of the same kernels reached 87-97%: resident CTAs then
// work on neighbouring rows, and each SM keeps starting fresh loads while
// older CTAs finish their arithmetic.
//
// Shape selection (row_shape): rows of up to 32 float4s use one group of
// pow2ceil(n4) threads with one float4 each; longer rows use the smallest
// power-of-two TPR in [32, 1024] that leaves each thread at most 4 float4s
// (rows of up to 16384 floats).  Few float4s per thread keep the register
// count low enough for 5-8 resident CTAs per SM.
#pragma once

#include "gbx_common.cuh"

namespace gbx {

constexpr int kRowMaxV4 = 4;
constexpr int kRowMaxTPR = 1024;

// Threads per CTA for a group width: CT (128 or 256, chosen per kernel), or
// the group itself when wider.
template <int TPR, int CT = 256>
struct RowCTA {
    static constexpr int threads = TPR > CT ? TPR : CT;
    static constexpr int rows = threads / TPR;
    static constexpr int warps = threads / 32;
    // a resident-CTA count stated for CTAs of 256 threads, in CTAs of this
    // size (the same register budget per thread)
    static constexpr int per256(int ctas) { return ctas * 256 / threads > 0 ? ctas * 256 / threads : 1; }
};

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
    while ((n4 + t - 1) / t > kRowMaxV4 && t < kRowMaxTPR) t <<= 1;
    const int v4 = (n4 + t - 1) / t;
    if (v4 > kRowMaxV4) return false;
    s->tpr = t;
    s->v4 = v4;
    return true;
}

// Sum / max over the TPR threads of this thread's row group.  For TPR > 32
// the warps of a group combine through `red` (RowCTA<TPR>::warps floats);
// every thread of the group adds the partials in the same order, so all of
// them get the same value.  Callers alternate two `red` buffers between
// consecutive reductions: the barrier inside each reduction then separates
// the reads of one buffer from its next writes.  Every thread of the CTA
// must call these (they contain __syncthreads for TPR > 32).
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

// Block-wide sum / max for the general (any length) kernels, which run
// kGeneralCTA threads: every thread gets the total.  `red` holds
// kGeneralCTA/32 floats; same alternation rule as above.
constexpr int kGeneralCTA = 256;

__device__ __forceinline__ float block_sum(float v, float* red)
{
    v = group_sum<32>(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kGeneralCTA / 32; ++w) s += red[w];
    return s;
}

__device__ __forceinline__ float block_max(float v, float* red)
{
    v = group_max<32>(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = red[0];
#pragma unroll
    for (int w = 1; w < kGeneralCTA / 32; ++w) m = fmaxf(m, red[w]);
    return m;
}

// Number of CTAs of the full-grid launch for `rows` rows at group width TPR,
// or -1 when it exceeds the grid limit.
// CTA size of a row launch.  Measured on B200: a grid of many 256-thread
// CTAs streams a little better (the XL prefill softmax, 204,800 CTAs: 962
// against 967 us with 128 threads), while a launch of few CTAs is latency-
// bound and gains from twice as many half-size ones (the GPT-2 XL decode
// step 1.224 -> 1.144 ms, the GPT-2 small chain 96.5 -> 93.4 us, graph
// replay).  Row kernels that take 128 either way (the attention softmax,
// the plain LayerNorm, the fused embedding) fix it; the others ask here:
// 128 threads when the 256-thread grid would hold fewer than
// kSmallGridCTAsPerSM CTAs per SM.
constexpr int kSmallGridCTAsPerSM = 32;
bool small_row_grid(int64_t ctas_at_256);   // status.cu

template <int TPR, int CT = 256>
inline int64_t row_grid(int64_t rows)
{
    const int64_t g = (rows + RowCTA<TPR, CT>::rows - 1) / RowCTA<TPR, CT>::rows;
    return g > 0x7fffffffLL ? -1 : g;
}

// Expands F(TPR, V4) for every shape row_shape can return; evaluates to the
// call's result, or `fallback` for an impossible shape.
#define GBX_ROW_CASE34(shape, F, T)                                                            \
    case T:                                                                                    \
        switch ((shape).v4) {                                                                  \
        case 3: return F(T, 3);                                                                \
        case 4: return F(T, 4);                                                                \
        }                                                                                      \
        break;

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
            }                                                                                  \
            break;                                                                             \
        GBX_ROW_CASE34(shape, F, 64)                                                         \
        GBX_ROW_CASE34(shape, F, 128)                                                         \
        GBX_ROW_CASE34(shape, F, 256)                                                         \
        GBX_ROW_CASE34(shape, F, 512)                                                         \
        GBX_ROW_CASE34(shape, F, 1024)                                                         \
        }                                                                                      \
        return static_cast<int>(fallback);                                                     \
    }()

}  // namespace gbx
