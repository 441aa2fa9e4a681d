// logits.cu -- tied-weight logits (replaces computeLogitsKernel,
// transformer.cu:296-307, launched at :898-900 on the final-LayerNorm row):
//   logits[r, v] = sum_j h[r, j] * dec(wte[v, j])
// for up to kLogitsMaxRows hidden rows per pass, reading the token table in
// its GGUF encoding (dec() gives the values of the reference's host dequant;
// f16 goes through the hardware conversion, whose only differences, the sign
// of zero and NaN payloads, cannot change the sum), so the [vocab, d] table
// crosses HBM once per pass whatever the number of rows.  This is an HBM-bound GEMV: one warp per
// vocabulary row, lanes striding the row in 4-element chunks (8-byte
// f16/bf16 or 16-byte f32 loads), the hidden rows staged once per CTA in
// shared memory, fp32 accumulation, one shuffle reduction per row.  The
// reference accumulates sequentially (sum += hidden[j] * tokenEmb[...]); the
// sums here differ from it in order only.
#include "gbx_common.cuh"
#include "decode.cuh"

namespace gbx {

constexpr int kLogitsThreads = 256;                  // 8 warps
constexpr int kLogitsRowsPerWarp = 4;                // vocabulary rows per warp
constexpr int kLogitsVocabPerCTA = (kLogitsThreads / 32) * kLogitsRowsPerWarp;

template <int T, int R>
__global__ void __launch_bounds__(kLogitsThreads)
logits_vec_kernel(const float* __restrict__ h, int rows, const void* __restrict__ wte, float* __restrict__ logits,
                  int vocab, int d)
{
    extern __shared__ float4 s_h[];   // [R][n4]
    const int n4 = d >> 2;
    for (int i = threadIdx.x; i < R * n4; i += kLogitsThreads) {
        const int r = i / n4;
        s_h[i] = r < rows ? __ldg(reinterpret_cast<const float4*>(h) + (int64_t)r * n4 + (i - r * n4))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int v0 = blockIdx.x * kLogitsVocabPerCTA + warp * kLogitsRowsPerWarp;
    for (int j = 0; j < kLogitsRowsPerWarp; ++j) {
        const int v = v0 + j;
        if (v >= vocab) break;   // warp-uniform
        const int64_t rowe = (int64_t)v * d;
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.0f;
        constexpr int UNROLL = 4;
        for (int c0 = lane; c0 < n4; c0 += 32 * UNROLL) {
            typename Raw4<T>::type w[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                const int c = c0 + 32 * u;
                w[u] = c < n4 ? load_raw4<T>(wte, rowe + 4 * c) : zero_raw4<T>();
            }
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                const int c = c0 + 32 * u;
                if (c < n4) {
                    // the sign of a zero product or the payload of a NaN
                    // cannot change the fp32 sum, so the hardware f16
                    // conversion serves
                    const float4 x = decode4_arith<T>(w[u]);
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const float4 hh = s_h[r * n4 + c];
                        acc[r] = fmaf(hh.x, x.x, acc[r]);
                        acc[r] = fmaf(hh.y, x.y, acc[r]);
                        acc[r] = fmaf(hh.z, x.z, acc[r]);
                        acc[r] = fmaf(hh.w, x.w, acc[r]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float s = group_sum<32>(acc[r]);
            if (lane == 0 && r < rows) logits[(int64_t)r * vocab + v] = s;
        }
    }
}

// General path (any d, any alignment): one warp per vocabulary row, scalar loads.
template <int T>
__global__ void __launch_bounds__(kLogitsThreads)
logits_general_kernel(const float* __restrict__ h, int rows, const void* __restrict__ wte,
                      float* __restrict__ logits, int vocab, int d)
{
    const int lane = threadIdx.x & 31;
    const int64_t v = (int64_t)blockIdx.x * (kLogitsThreads / 32) + (threadIdx.x >> 5);
    if (v >= vocab) return;
    for (int r = 0; r < rows; ++r) {
        float acc = 0.0f;
        for (int j = lane; j < d; j += 32) acc = fmaf(h[(int64_t)r * d + j], load1<T>(wte, v * d + j), acc);
        acc = group_sum<32>(acc);
        if (lane == 0) logits[(int64_t)r * vocab + v] = acc;
    }
}

template <int T, int R>
static int launch_logits_vec(const float* h, int rows, const void* wte, float* logits, int vocab, int d,
                             cudaStream_t s)
{
    auto k = logits_vec_kernel<T, R>;
    const size_t smem = (size_t)R * d * sizeof(float);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return check_launch("gbx_logits: shared-memory attribute");
    const int grid = (vocab + kLogitsVocabPerCTA - 1) / kLogitsVocabPerCTA;
    k<<<grid, kLogitsThreads, smem, s>>>(h, rows, wte, logits, vocab, d);
    return GBX_OK;
}

template <int T>
static int launch_logits(const float* h, int64_t rows, const void* wte, float* logits, int vocab, int d,
                         cudaStream_t s)
{
    const int es = T == TF32 ? 4 : 2;
    DeviceInfo di;
    if (device_info(&di) != GBX_OK) return GBX_ECUDA;
    const bool vec = d % 4 == 0 && aligned16(h) && ((uintptr_t)wte % (4 * es)) == 0 &&
                     (size_t)kLogitsMaxRows * d * sizeof(float) <= (size_t)di.max_smem_optin;
    for (int64_t r0 = 0; r0 < rows; r0 += kLogitsMaxRows) {
        const int n = (int)(rows - r0 < kLogitsMaxRows ? rows - r0 : kLogitsMaxRows);
        const float* hr = h + r0 * d;
        float* lr = logits + r0 * vocab;
        int rc = GBX_OK;
        if (vec) {
            if (n == 1) rc = launch_logits_vec<T, 1>(hr, n, wte, lr, vocab, d, s);
            else if (n == 2) rc = launch_logits_vec<T, 2>(hr, n, wte, lr, vocab, d, s);
            else if (n <= 4) rc = launch_logits_vec<T, 4>(hr, n, wte, lr, vocab, d, s);
            else rc = launch_logits_vec<T, 8>(hr, n, wte, lr, vocab, d, s);
        } else {
            const int grid = (vocab + kLogitsThreads / 32 - 1) / (kLogitsThreads / 32);
            logits_general_kernel<T><<<grid, kLogitsThreads, 0, s>>>(hr, n, wte, lr, vocab, d);
        }
        if (rc != GBX_OK) return rc;
    }
    return check_launch("gbx_logits");
}

}  // namespace gbx

using namespace gbx;

extern "C" int gbx_logits(const float* h, int64_t rows, const void* wte, int wte_dtype, float* logits, int vocab,
                          int d, gbx_stream_t stream)
{
    const int t = dtype_index(wte_dtype);
    if (t < 0) return set_error(GBX_EDTYPE, "gbx_logits: unsupported GGUF dtype %d", wte_dtype);
    if (rows < 0 || vocab <= 0 || d <= 0)
        return set_error(GBX_EINVAL, "gbx_logits: rows=%lld vocab=%d d=%d", (long long)rows, vocab, d);
    if (rows == 0) return GBX_OK;
    if (!h || !wte || !logits) return set_error(GBX_EINVAL, "gbx_logits: null pointer");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (t) {
    case TF32: return launch_logits<TF32>(h, rows, wte, logits, vocab, d, s);
    case TF16: return launch_logits<TF16>(h, rows, wte, logits, vocab, d, s);
    default: return launch_logits<TBF16>(h, rows, wte, logits, vocab, d, s);
    }
}
