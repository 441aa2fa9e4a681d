// layernorm.cu -- LayerNorm and fused residual-add + LayerNorm
// (replaces layerNormKernel, transformer.cu:77-124, and the residual
// epilogues of projectionKernel / ffnDownKernel, transformer.cu:262, :292).
//
// Per row: one HBM read of x (and r), h = r + x kept in registers, mean and
// the exact two-pass population variance from registers via warp shuffles,
// one HBM write of y (and h).  gamma/beta/bias rows are read through the
// read-only path: every CTA of the full-grid launch touches the same few KB,
// which stay in L2 and L1.  The arithmetic is the reference's:
//   mean = sum/d; var = sum((x-mean)^2)/d (variance terms fused as the
//   reference's nvcc build fuses them); inv = rsqrtf(var + eps);
//   y = fmaf((x - mean) * inv, gamma, beta)
// and differs from it only in the order of the two sums (shuffle tree here,
// shared-memory tree there).
#include "rows.cuh"
#include "tf32.cuh"

namespace gbx {

// y_lo non-null: y and y_lo receive the tf32 pair of the output (tf32.cuh)
// instead of the fp32 output, for gbx_linear.
// Resident CTAs per SM the row kernels are compiled for (a register budget of
// 65536 / (CTA threads x this)); 1 leaves the compiler free.  Measured on
// B200 (32,768 rows of 1600): the LayerNorm at 6 (40 registers) 70.1 us
// against 80.2 us free (48 registers, 5 CTAs); residual + LayerNorm best free
// (50 registers): capped at 6 it spills and takes 130 against 127.5 us.
#ifndef GBX_LN_MIN_CTAS
#define GBX_LN_MIN_CTAS 6
#endif
#ifndef GBX_RLN_MIN_CTAS
#define GBX_RLN_MIN_CTAS 1
#endif

// CT: threads per CTA (rows.cuh).  The plain LayerNorm runs CTAs of 128:
// 68.1-69.1 against 70.0-70.1 us for 32,768 rows of 1600 in CTAs of 256.
template <int TPR, int V4, bool RESID, int CT>
__global__ void __launch_bounds__(RowCTA<TPR, CT>::threads,
                                  RowCTA<TPR, CT>::threads > 256
                                      ? 1
                                      : RowCTA<TPR, CT>::per256(RESID ? GBX_RLN_MIN_CTAS : GBX_LN_MIN_CTAS))
ln_vec_kernel(const float* x, const float* r, const float* __restrict__ xbias, float* h_out, float* y, float* y_lo,
              const float* __restrict__ gamma, const float* __restrict__ beta, int64_t rows, int d, int64_t ld,
              float eps)
{
    grid_dependency_wait();   // see launch_row_kernel
    allow_dependents();
    using C = RowCTA<TPR, CT>;
    __shared__ float red[2][C::warps];
    const int n4 = d >> 2;
    const int lane = threadIdx.x & (TPR - 1);
    const int64_t row = (int64_t)blockIdx.x * C::rows + threadIdx.x / TPR;
    const bool valid = row < rows;
    const int64_t in_off = row * ld;   // x, r, h_out
    const int64_t off = row * d;       // y, y_lo
    const float fd = (float)d;

    // Per-lane base pointers with compile-time offsets (k * TPR float4s), and
    // "float4 k * TPR + lane exists" as one compare against lim: no
    // per-element index math or pointer tests inside the unrolled loops.
    const int lim = n4 - lane;
    const float* const xrow = x + in_off + 4 * lane;
    float4 v[V4];
#pragma unroll
    for (int k = 0; k < V4; ++k)
        v[k] = (valid && k * TPR < lim) ? ld_stream(xrow + 4 * k * TPR) : make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (RESID) {
        const float* const rrow = r + in_off + 4 * lane;
        float4 rv[V4];
#pragma unroll
        for (int k = 0; k < V4; ++k)
            rv[k] = (valid && k * TPR < lim) ? ld_stream(rrow + 4 * k * TPR) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (xbias) {
            const float* const brow = xbias + 4 * lane;
#pragma unroll
            for (int k = 0; k < V4; ++k)
                if (k * TPR < lim) v[k] = add4(v[k], ld_param4(brow + 4 * k * TPR));
        }
#pragma unroll
        for (int k = 0; k < V4; ++k) v[k] = add4(rv[k], v[k]);
        if (h_out && valid) {
            float* const hrow = h_out + in_off + 4 * lane;
#pragma unroll
            for (int k = 0; k < V4; ++k)
                if (k * TPR < lim) st_stream(hrow + 4 * k * TPR, v[k]);
        }
    }

    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < V4; ++k) s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    s = row_sum<TPR>(s, red[0]);
    const float mean = s / fd;

    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < V4; ++k) {
        if (k * TPR < lim) {
            const float4 dv = sub4s(v[k], mean);
            q = fmaf(dv.x, dv.x, q);
            q = fmaf(dv.y, dv.y, q);
            q = fmaf(dv.z, dv.z, q);
            q = fmaf(dv.w, dv.w, q);
        }
    }
    q = row_sum<TPR>(q, red[1]);
    const float inv = rsqrtf(q / fd + eps);

    if (!valid) return;
    float* const yrow = y + off + 4 * lane;
    if (gamma && beta && !y_lo) {
        // the common case, with no per-element pointer tests
        const float* const grow = gamma + 4 * lane;
        const float* const brow = beta + 4 * lane;
#pragma unroll
        for (int k = 0; k < V4; ++k) {
            if (k * TPR < lim) {
                const float4 g = ld_param4(grow + 4 * k * TPR), b = ld_param4(brow + 4 * k * TPR);
                st_stream(yrow + 4 * k * TPR, ln_affine4(v[k], mean, inv, g, b));
            }
        }
        return;
    }
#pragma unroll
    for (int k = 0; k < V4; ++k) {
        const int c = k * TPR + lane;
        if (k * TPR < lim) {
            const float4 g = gamma ? ld_param4(gamma + 4 * c) : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
            const float4 b = beta ? ld_param4(beta + 4 * c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            const float4 o = ln_affine4(v[k], mean, inv, g, b);
            if (y_lo) {
                float4 hi, lo;
                split4(o, hi, lo);
                st_stream(yrow + 4 * k * TPR, hi);
                st_stream(y_lo + off + 4 * c, lo);
            } else {
                st_stream(yrow + 4 * k * TPR, o);
            }
        }
    }
}

// General path (any d, any alignment): one CTA per row, three passes over the
// row in global memory, like the reference, with shuffle reductions.  When
// RESID and h_out is given, pass 0 materialises h there and later passes read
// it back; without h_out, h = r + (x + xbias) is recomputed in each pass.
template <bool RESID>
__global__ void __launch_bounds__(kGeneralCTA)
ln_general_kernel(const float* x, const float* r, const float* __restrict__ xbias, float* h_out,
                  float* y, float* y_lo, const float* __restrict__ gamma, const float* __restrict__ beta,
                  int64_t rows, int d, int64_t ld, float eps)
{
    __shared__ float red[2][kGeneralCTA / 32];
    const float fd = (float)d;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const int64_t in_off = row * ld;   // x, r, h_out
        const int64_t off = row * d;       // y, y_lo
        auto hval = [&](int i) -> float {
            if (!RESID) return x[in_off + i];
            if (h_out) return h_out[in_off + i];
            const float xv = xbias ? x[in_off + i] + xbias[i] : x[in_off + i];
            return r[in_off + i] + xv;
        };
        if (RESID && h_out) {
            for (int i = threadIdx.x; i < d; i += kGeneralCTA) {
                const float xv = xbias ? x[in_off + i] + xbias[i] : x[in_off + i];
                h_out[in_off + i] = r[in_off + i] + xv;
            }
            __syncthreads();
        }
        float s = 0.0f;
        for (int i = threadIdx.x; i < d; i += kGeneralCTA) s += hval(i);
        const float mean = block_sum(s, red[0]) / fd;
        float q = 0.0f;
        for (int i = threadIdx.x; i < d; i += kGeneralCTA) {
            const float diff = hval(i) - mean;
            q = fmaf(diff, diff, q);
        }
        const float inv = rsqrtf(block_sum(q, red[1]) / fd + eps);
        for (int i = threadIdx.x; i < d; i += kGeneralCTA) {
            const float g = gamma ? gamma[i] : 1.0f;
            const float b = beta ? beta[i] : 0.0f;
            const float o = fmaf((hval(i) - mean) * inv, g, b);
            if (y_lo) {
                float hi, lo;
                split_value(o, hi, lo);
                y[off + i] = hi;
                y_lo[off + i] = lo;
            } else {
                y[off + i] = o;
            }
        }
        __syncthreads();   // pass-0 writes of the next row vs this row's reads
    }
}

template <int TPR, int V4, bool RESID>
static int launch_ln_vec(const float* x, const float* r, const float* xbias, float* h_out, float* y, float* y_lo,
                         const float* g, const float* b, int64_t rows, int d, int64_t ld, float eps,
                         cudaStream_t stream)
{
    const int64_t grid256 = row_grid<TPR, 256>(rows);
    auto small = [&]() -> int {
        const int64_t grid128 = row_grid<TPR, 128>(rows);
        if (grid128 < 0) return GBX_ERANGE;
        launch_row_kernel(ln_vec_kernel<TPR, V4, RESID, 128>, dim3((unsigned)grid128), dim3(RowCTA<TPR, 128>::threads),
                          0, stream, x, r, xbias, h_out, y, y_lo, g, b, rows, d, ld, eps);
        return GBX_OK;
    };
    if constexpr (!RESID) {
        return small();
    } else {
        if (grid256 >= 0 && small_row_grid(grid256)) return small();
        if (grid256 < 0) return GBX_ERANGE;
        launch_row_kernel(ln_vec_kernel<TPR, V4, RESID, 256>, dim3((unsigned)grid256), dim3(RowCTA<TPR, 256>::threads),
                          0, stream, x, r, xbias, h_out, y, y_lo, g, b, rows, d, ld, eps);
    }
    return GBX_OK;
}

// ld: row stride of x, r and h_out in floats (d for contiguous rows); y and
// y_lo rows are always contiguous.
template <bool RESID>
static int launch_ln(const char* what, const float* x, const float* r, const float* xbias, float* h_out, float* y,
                     float* y_lo, const float* g, const float* b, int64_t rows, int d, int64_t ld, float eps,
                     cudaStream_t stream)
{
    RowShape shape;
    const bool vec = d % 4 == 0 && ld % 4 == 0 && row_shape(d / 4, &shape) && aligned16(x) && aligned16(y) &&
                     (!y_lo || aligned16(y_lo)) && (!RESID || aligned16(r)) && (!h_out || aligned16(h_out)) &&
                     (!xbias || aligned16(xbias)) && (!g || aligned16(g)) && (!b || aligned16(b));
    if (vec) {
#define GBX_LN_CALL(T, V) launch_ln_vec<T, V, RESID>(x, r, xbias, h_out, y, y_lo, g, b, rows, d, ld, eps, stream)
        const int rc = GBX_ROW_DISPATCH(shape, GBX_LN_CALL, GBX_ERANGE);
#undef GBX_LN_CALL
        if (rc != GBX_OK) return set_error(rc, "%s: rows=%lld d=%d out of range", what, (long long)rows, d);
    } else {
        auto k = ln_general_kernel<RESID>;
        const int grid = persistent_grid(k, kGeneralCTA, 0, rows, 4);
        if (grid < 1) return GBX_ECUDA;
        k<<<grid, kGeneralCTA, 0, stream>>>(x, r, xbias, h_out, y, y_lo, g, b, rows, d, ld, eps);
    }
    return check_launch(what);
}

}  // namespace gbx

using namespace gbx;

extern "C" int gbx_layernorm(const float* x, float* y, const float* gamma, const float* beta,
                             int64_t rows, int d, float eps, gbx_stream_t stream)
{
    if (rows < 0 || d <= 0) return set_error(GBX_EINVAL, "gbx_layernorm: rows=%lld d=%d", (long long)rows, d);
    if (rows == 0) return GBX_OK;
    if (!x || !y) return set_error(GBX_EINVAL, "gbx_layernorm: null pointer");
    return launch_ln<false>("gbx_layernorm", x, nullptr, nullptr, nullptr, y, nullptr, gamma, beta, rows, d, d, eps,
                            reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gbx_layernorm_pair(const float* x, float* y_hi, float* y_lo, const float* gamma, const float* beta,
                                  int64_t rows, int d, float eps, gbx_stream_t stream)
{
    if (rows < 0 || d <= 0) return set_error(GBX_EINVAL, "gbx_layernorm_pair: rows=%lld d=%d", (long long)rows, d);
    if (rows == 0) return GBX_OK;
    if (!x || !y_hi || !y_lo) return set_error(GBX_EINVAL, "gbx_layernorm_pair: null pointer");
    if (y_lo == x || y_lo == y_hi) return set_error(GBX_EINVAL, "gbx_layernorm_pair: y_lo must not alias x or y_hi");
    return launch_ln<false>("gbx_layernorm_pair", x, nullptr, nullptr, nullptr, y_hi, y_lo, gamma, beta, rows, d,
                            d, eps, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gbx_residual_layernorm(const float* x, const float* r, const float* xbias, float* h_out,
                                      float* y, const float* gamma, const float* beta, int64_t rows,
                                      int d, float eps, gbx_stream_t stream)
{
    if (rows < 0 || d <= 0)
        return set_error(GBX_EINVAL, "gbx_residual_layernorm: rows=%lld d=%d", (long long)rows, d);
    if (rows == 0) return GBX_OK;
    if (!x || !r || !y) return set_error(GBX_EINVAL, "gbx_residual_layernorm: null pointer");
    if (h_out && h_out == y) return set_error(GBX_EINVAL, "gbx_residual_layernorm: h_out and y must differ");
    return launch_ln<true>("gbx_residual_layernorm", x, r, xbias, h_out, y, nullptr, gamma, beta, rows, d, d, eps,
                           reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gbx_final_layernorm(const float* x, const float* r, float* y, const float* gamma, const float* beta,
                                   int64_t n_seq, int seq, int d, float eps, gbx_stream_t stream)
{
    if (n_seq < 0 || seq <= 0 || d <= 0)
        return set_error(GBX_EINVAL, "gbx_final_layernorm: n_seq=%lld seq=%d d=%d", (long long)n_seq, seq, d);
    if (n_seq == 0) return GBX_OK;
    if (!r || !y) return set_error(GBX_EINVAL, "gbx_final_layernorm: null pointer");
    const int64_t ld = (int64_t)seq * d;      // from one sequence's last row to the next's
    const int64_t first = (int64_t)(seq - 1) * d;
    if (seq > 1) {
        // y rows are packed, the input rows are strided: another CTA's input
        // row could lie under this CTA's output row.
        const uintptr_t y0 = (uintptr_t)y, y1 = (uintptr_t)(y + n_seq * d);
        for (const float* in : {x, r}) {
            if (!in) continue;
            const uintptr_t a0 = (uintptr_t)in, a1 = (uintptr_t)(in + n_seq * ld);
            if (a0 < y1 && y0 < a1) return set_error(GBX_EINVAL, "gbx_final_layernorm: y overlaps an input");
        }
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (x)
        return launch_ln<true>("gbx_final_layernorm", x + first, r + first, nullptr, nullptr, y, nullptr, gamma, beta,
                               n_seq, d, ld, eps, st);
    return launch_ln<false>("gbx_final_layernorm", r + first, nullptr, nullptr, nullptr, y, nullptr, gamma, beta, n_seq,
                            d, ld, eps, st);
}
