// select.cu -- next-token selection over logits rows, replacing the host loop
// of TransformerModel::generate (transformer.cu:994-1028):
//
//   best = first j with the row maximum (a strict `>` scan from j = 0, :994-1001)
//   T <= 0.01: selected = best                                   (:1004-1005)
//   else:      l_j = (float)((double)logit_j / T)                (:1007: float /= double)
//              m = max_j l_j; e_j = expf(l_j - m); s = sum_j e_j (fp32)   (:1009-1014)
//              p_j = e_j / s                                      (:1015)
//              selected = first j with u <= sum_{i<=j} p_i, accumulated in double,
//                         0 when no j qualifies                   (:1017-1026)
//
// u is the caller's uniform draw in [0, 1) (the reference draws it from its
// mt19937, :1017-1018), one per row.  One CTA of 1024 threads per row: the
// row is staged in shared memory with coalesced loads (rows up to 55k
// entries; longer rows are read from global memory), each thread owns a
// contiguous segment of it, and block-wide reductions and a block-wide
// exclusive scan (in double) combine the segments.  The fp32 sum is taken in
// segment-then-tree order rather than the reference's sequential order, so
// the p_j agree to a relative 1e-7 and the selection agrees except when u
// falls within that distance of a cumulative boundary.
#include <float.h>

#include "gbx_common.cuh"

namespace gbx {

constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;

struct ArgMax {
    float v;
    int i;
};

// larger value wins; on equal values the smaller index (the reference keeps
// the first maximum); NaN never wins (the reference's `>` is false for it)
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b)
{
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

template <class T, class Op>
__device__ __forceinline__ T block_reduce(T v, T* red, Op op)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    T r = red[0];
    for (int w = 1; w < kSelWarps; ++w) r = op(r, red[w]);
    __syncthreads();
    return r;
}

__device__ __forceinline__ ArgMax shfl_argmax(ArgMax a, int o)
{
    ArgMax b;
    b.v = __shfl_xor_sync(0xffffffffu, a.v, o);
    b.i = __shfl_xor_sync(0xffffffffu, a.i, o);
    return b;
}

// Exclusive prefix sum of one double per thread across the CTA.
__device__ __forceinline__ double block_exclusive_scan(double v, double* warp_tot)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    double incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        double t = lane < kSelWarps ? warp_tot[lane] : 0.0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double n = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += n;
        }
        if (lane < kSelWarps) warp_tot[lane] = t;   // inclusive over warps
    }
    __syncthreads();
    const double before = (warp ? warp_tot[warp - 1] : 0.0) + (incl - v);
    __syncthreads();
    return before;
}

template <bool SMEM>
__global__ void __launch_bounds__(kSelThreads)
select_kernel(const float* __restrict__ logits, int64_t rows, int vocab, double temperature,
              const double* __restrict__ uniforms, int32_t* __restrict__ out_ids, int32_t* __restrict__ out_best,
              float* __restrict__ out_best_logit)
{
    extern __shared__ float s_row[];
    __shared__ ArgMax red_am[kSelWarps];
    __shared__ float red_f[kSelWarps];
    __shared__ double red_d[kSelWarps];
    __shared__ int red_i[kSelWarps];

    const int64_t row = blockIdx.x;
    const float* g = logits + row * vocab;
    float* x = SMEM ? s_row : nullptr;
    if (SMEM) {
        for (int j = threadIdx.x; j < vocab; j += kSelThreads) s_row[j] = __ldg(g + j);
        __syncthreads();
    }
    auto at = [&](int j) -> float { return SMEM ? x[j] : __ldg(g + j); };

    const int seg = (vocab + kSelThreads - 1) / kSelThreads;
    const int j0 = min(vocab, (int)threadIdx.x * seg), j1 = min(vocab, j0 + seg);

    // best: first maximum; a NaN first entry pins the answer to 0
    ArgMax am{-INFINITY, 0x7fffffff};
    for (int j = j0; j < j1; ++j) {
        const float v = at(j);
        if (v > am.v || (am.i == 0x7fffffff && !(v != v))) am = ArgMax{v, j};
    }
    {
        ArgMax v = am;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = better(v, shfl_argmax(v, o));
        if ((threadIdx.x & 31) == 0) red_am[threadIdx.x >> 5] = v;
        __syncthreads();
        ArgMax r = red_am[0];
        for (int w = 1; w < kSelWarps; ++w) r = better(r, red_am[w]);
        __syncthreads();
        am = r;
    }
    const float first = at(0);
    int best = am.i == 0x7fffffff ? 0 : am.i;
    float best_v = am.i == 0x7fffffff ? first : am.v;
    if (first != first) {   // the reference's bestLogit starts as NaN: nothing compares greater
        best = 0;
        best_v = first;
    }

    int selected = best;
    if (temperature > 0.01) {
        // l_j = (float)(logit_j / T) in double, as `l /= temperature` with a
        // float l and a double T
        float m = -INFINITY;
        for (int j = j0; j < j1; ++j) m = fmaxf(m, (float)((double)at(j) / temperature));
        m = block_reduce(m, red_f, [](float a, float b) { return fmaxf(a, b); });
        float s = 0.0f;
        for (int j = j0; j < j1; ++j) s += expf((float)((double)at(j) / temperature) - m);
        s = block_reduce(s, red_f, [](float a, float b) { return a + b; });
        double part = 0.0;
        for (int j = j0; j < j1; ++j) part += (double)(expf((float)((double)at(j) / temperature) - m) / s);
        double cum = block_exclusive_scan(part, red_d);
        const double u = uniforms[row];
        int found = 0x7fffffff;
        for (int j = j0; j < j1; ++j) {
            cum += (double)(expf((float)((double)at(j) / temperature) - m) / s);
            if (u <= cum) {
                found = j;
                break;
            }
        }
        found = block_reduce(found, red_i, [](int a, int b) { return min(a, b); });
        selected = found == 0x7fffffff ? 0 : found;
    }
    if (threadIdx.x == 0) {
        out_ids[row] = selected;
        if (out_best) out_best[row] = best;
        if (out_best_logit) out_best_logit[row] = best_v;
    }
}

}  // namespace gbx

using namespace gbx;

extern "C" int gbx_select_tokens(const float* logits, int64_t rows, int vocab, double temperature,
                                 const double* uniforms, int32_t* out_ids, int32_t* out_best, float* out_best_logit,
                                 gbx_stream_t stream)
{
    if (rows < 0 || vocab <= 0) return set_error(GBX_EINVAL, "gbx_select_tokens: rows=%lld vocab=%d",
                                                 (long long)rows, vocab);
    if (rows == 0) return GBX_OK;
    if (!logits || !out_ids) return set_error(GBX_EINVAL, "gbx_select_tokens: null pointer");
    if (!(temperature <= 0.01) && !uniforms)
        return set_error(GBX_EINVAL, "gbx_select_tokens: temperature %g needs uniforms", temperature);
    if (temperature != temperature) return set_error(GBX_EINVAL, "gbx_select_tokens: temperature is NaN");
    if (rows > 0x7fffffffLL) return set_error(GBX_ERANGE, "gbx_select_tokens: too many rows");
    DeviceInfo di;
    if (device_info(&di) != GBX_OK) return GBX_ECUDA;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const size_t smem = (size_t)vocab * sizeof(float);
    // leave room for the kernel's static shared memory
    if (smem + 4096 <= (size_t)di.max_smem_optin) {
        if (smem > 48 * 1024 && cudaFuncSetAttribute(select_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)smem) != cudaSuccess)
            return check_launch("gbx_select_tokens: shared-memory attribute");
        select_kernel<true><<<(unsigned)rows, kSelThreads, smem, s>>>(logits, rows, vocab, temperature, uniforms,
                                                                     out_ids, out_best, out_best_logit);
    } else {
        select_kernel<false><<<(unsigned)rows, kSelThreads, 0, s>>>(logits, rows, vocab, temperature, uniforms,
                                                                   out_ids, out_best, out_best_logit);
    }
    return check_launch("gbx_select_tokens");
}
