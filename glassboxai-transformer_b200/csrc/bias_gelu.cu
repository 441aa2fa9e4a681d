// bias_gelu.cu -- bias + GELU(tanh) (replaces the ffnUpKernel epilogue,
// transformer.cu:272, 276-277, and geluKernel, :68-75).
//
// Layout: a full grid of CTAs, each owning one band of T float4 columns of
// kGeluU consecutive rows.  A thread loads its column's 4 bias values once,
// issues the kGeluU row loads before any arithmetic, and writes each result
// with a streaming 16-byte store.  (On B200 this launch shape streamed at the
// measured copy bandwidth; a persistent grid walking the rows reached 81%.)
// The formula is the reference's, with the cubic term fused as the
// reference's nvcc build fuses it, and CUDA's tanhf (no fast-math):
//   u = in + bias; out = u * (0.5f * (1.0f + tanhf(0.7978845608f * (u + 0.044715f*u*u*u))))
#include "gbx_common.cuh"
#include "rows.cuh"
#include "gelu.cuh"

namespace gbx {

// Rows per thread: kGeluU in large launches, kGeluSmallU in launches of few
// CTAs (rows.cuh's small-grid rule, counted in 256-thread CTAs), where more
// CTAs with less work each finish sooner.  Measured on B200 (graph replay):
// the GPT-2 XL decode step 1.146 ms with 4 rows, 1.135 with 1, 1.113 with 2;
// the GPT-2 small chain 94-98 us with 4, 88 with 1 or 2; GPT-2 medium
// (large launches) unchanged.
// (large launches, XL prefill 32,768 x 6400: 248-250 us with 4 rows, 256 with
// 2, 291 with 8 (spills at the 32-register budget).)
constexpr int kGeluU = 4;
constexpr int kGeluSmallU = 2;

// Two elements per packed instruction (gelu4, add4): bit-identical to the
// scalar form, and on B200 12% fewer instructions per launch (96.3 M
// against 109.2 M on 16,384 rows of 6400), so that under the power cap the
// XL prefill's launch takes 249-250 us in the chain against 276 us.

// blockIdx.x = slab * bands + band.  At most 32 registers (4 CTAs of the
// widest band per SM): the kernel issues a long tanhf per element, and on
// B200 it streamed 13% faster with 6 resident 320-thread CTAs per SM than
// with 3 (56 registers) or 5 (40); no spills at this bound.
template <bool BIAS, int U>
__global__ void __launch_bounds__(512, 4)
bias_gelu_vec_kernel(const float* in, float* out, const float* __restrict__ bias, int64_t rows, int n4, int bands)
{
    grid_dependency_wait();   // see launch_row_kernel
    allow_dependents();
    const int band = (int)(blockIdx.x % (unsigned)bands);
    const int64_t r0 = (int64_t)(blockIdx.x / (unsigned)bands) * U;
    const int c = band * blockDim.x + threadIdx.x;
    if (c >= n4) return;
    const int64_t F = 4LL * n4;
    const float4 b = BIAS ? ld_param4(bias + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
        v[u] = (r0 + u < rows) ? ld_stream(in + (r0 + u) * F + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < U; ++u) {
        if (r0 + u < rows) {
            float4 x = v[u];
            if (BIAS) x = add4(x, b);
            st_stream(out + (r0 + u) * F + 4 * c, gelu4(x));
        }
    }
}

__global__ void __launch_bounds__(256)
bias_gelu_general_kernel(const float* in, float* out, const float* __restrict__ bias, int64_t rows, int F)
{
    const int64_t total = rows * F;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        float u = in[i];
        if (bias) u = u + bias[i % F];
        out[i] = gelu_tanh(u);
    }
}

// Column band width: the largest multiple of 32 in [128, 512] that divides
// n4 (no idle lanes), else 256 (short rows: n4 rounded up to a warp).
static int gelu_band(int n4)
{
    if (n4 < 128) return (n4 + 31) / 32 * 32;
    for (int t = 512; t >= 128; t -= 32)
        if (n4 % t == 0) return t;
    return 256;
}

template <bool BIAS>
static int launch_gelu_vec(const float* in, float* out, const float* bias, int64_t rows, int n4,
                           cudaStream_t stream)
{
    const int T = gelu_band(n4);
    const int bands = (n4 + T - 1) / T;
    const int64_t grid = (int64_t)bands * ((rows + kGeluU - 1) / kGeluU);
    // a launch of few CTAs (counted in 256-thread equivalents) takes fewer rows per thread
    const bool small = small_row_grid(grid * T / 256);
    const int64_t g = small ? (int64_t)bands * ((rows + kGeluSmallU - 1) / kGeluSmallU) : grid;
    if (g > 0x7fffffffLL)
        return set_error(GBX_ERANGE, "gbx_bias_gelu: rows=%lld F=%d needs too many CTAs", (long long)rows, 4 * n4);
    if (small)
        launch_row_kernel(bias_gelu_vec_kernel<BIAS, kGeluSmallU>, dim3((unsigned)g), dim3(T), 0, stream, in, out,
                          bias, rows, n4, bands);
    else
        launch_row_kernel(bias_gelu_vec_kernel<BIAS, kGeluU>, dim3((unsigned)g), dim3(T), 0, stream, in, out, bias,
                          rows, n4, bands);
    return check_launch("gbx_bias_gelu");
}

}  // namespace gbx

using namespace gbx;

extern "C" int gbx_bias_gelu(const float* in, float* out, const float* bias, int64_t rows, int F,
                             gbx_stream_t stream)
{
    if (rows < 0 || F <= 0) return set_error(GBX_EINVAL, "gbx_bias_gelu: rows=%lld F=%d", (long long)rows, F);
    if (rows == 0) return GBX_OK;
    if (!in || !out) return set_error(GBX_EINVAL, "gbx_bias_gelu: null pointer");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (F % 4 == 0 && aligned16(in) && aligned16(out) && (!bias || aligned16(bias))) {
        return bias ? launch_gelu_vec<true>(in, out, bias, rows, F / 4, s)
                    : launch_gelu_vec<false>(in, out, bias, rows, F / 4, s);
    }
    const int grid = persistent_grid(bias_gelu_general_kernel, 256, 0, (rows * F + 255) / 256, 4);
    if (grid < 1) return GBX_ECUDA;
    bias_gelu_general_kernel<<<grid, 256, 0, s>>>(in, out, bias, rows, F);
    return check_launch("gbx_bias_gelu");
}
