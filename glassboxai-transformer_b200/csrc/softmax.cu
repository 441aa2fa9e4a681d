// softmax.cu -- row softmax (replaces softmaxKernel, transformer.cu:126-166,
// which the reference launches once per head, :839-842), and the same softmax
// fused with the score epilogue of attentionScoresKernel
// (transformer.cu:213-232: divide by sqrt(headDim), -1e9f above the diagonal).
//
// Per row: one HBM read into registers, max by warp shuffles (seeded with
// -1e30f like the reference), e = expf(x - max) kept in registers, sum by
// shuffles, out = e / sum, one HBM write.  The reference makes three reads
// and two writes of every element.
//
// Division.  out = e / sum is evaluated as q = e * r, q += (e - q*sum) * r
// with r = 1/sum (IEEE, once per row) and both steps as FMAs: the residual
// e - q*sum is exact, and one correction step from a faithful quotient and
// the correctly rounded reciprocal gives the correctly rounded quotient
// (Markstein's theorem) whenever no intermediate is subnormal.  Outputs are
// therefore the IEEE quotients the reference computes, except possibly for
// subnormal outputs (absolute error below 1e-38).  The per-element IEEE
// divide has a slow path that every masked entry (e = 0) takes; on B200 it
// cut the kernel's throughput from 6.5 to 4.3 TB/s on causal score rows.
// The same identity gives the score scaling x / scale (an exact multiply when
// scale is a power of two, as sqrt(64) = 8 is for GPT-2's 64-wide heads).
//
// Because max is exact and expf is the same CUDA function, every e is
// bit-identical to the reference's; only the order of the sum differs.
#include <type_traits>

#include "rows.cuh"
#include "tf32.cuh"

namespace gbx {

__device__ __forceinline__ float div_by(float a, float b, float rb)
{
    const float q = a * rb;
    return fmaf(fmaf(-q, b, a), rb, q);
}

// div_by on four quotients a / b with one reciprocal rb, two per packed
// instruction: fmaf(-q, b, a) is the same exact value as fmaf(q, -b, a)
// before its one rounding, so the result is div_by's bit for bit.
__device__ __forceinline__ float4 div4_by(float4 a, float b, float rb)
{
    const float4 q = mul4s(a, rb);
    return fma4s(fma4s(q, -b, a), rb, q);
}

// Score epilogue of the attention variant: the query of row p (p = row % S)
// sees key columns 0 .. p + q_off; later columns hold -1e9f
// (transformer.cu:220-221), earlier ones raw / scale (:228).
struct ScoreEpilogue {
    int S;
    int q_off;
    float scale;
    bool causal;
    FastDiv div_S;   // S, for the 32-bit row index of the vector path
};

// POW2: scale is a power of two, so raw / scale == raw * (1/scale) exactly.
// PAIR_OUT: out and out_lo receive the tf32 pair of each probability
// (tf32.cuh), the operand form of the attention-output contraction; with
// the causal prefill mask (q_off 0) only columns below
// round_up(p + 1, 256) are written: the rest are zero, and the
// contraction, whose row tiles are 128 or 256 rows high, never reads them.
// (PAIR_OUT held to 8 resident CTAs of 256 threads, 32 registers: 6%
// faster on B200 than its unbounded 48 registers, a few bytes spilled.
// The attention form without the pair is compiled for GBX_ATTN_SM_MIN_CTAS
// resident CTAs of 256 threads' worth of registers (rows.cuh, per256): at 6
// (40 registers, no spill) 1032 us for 819,200 causal rows of 1024 in CTAs
// of 256, against 1137 us unbounded (47 registers) and 1033 us at 8.  The
// plain softmax is best left free, GBX_SM_MIN_CTAS 1 (40 registers, 6 CTAs):
// 962 us against 968 us at 8 CTAs (32 registers) on the same rows.)
#ifndef GBX_ATTN_SM_MIN_CTAS
#define GBX_ATTN_SM_MIN_CTAS 6
#endif
#ifndef GBX_SM_MIN_CTAS
#define GBX_SM_MIN_CTAS 1
#endif
// CT: threads per CTA (rows.cuh).  The attention form runs CTAs of 128:
// 947-948 against 1042 us for 819,200 causal rows of 1024 in CTAs of 256
// (its early causal rows finish fast, and smaller CTAs refill the SMs
// sooner).  The plain form takes 256 for large grids, 128 for small ones
// (CTAs of 512 on the XL prefill rows: 961 against 962 us alone, but the XL
// prefill step then took 73.6-74.0 against 69.9 ms).
template <int TPR, int V4, bool ATTN, bool POW2, bool PAIR_OUT, int CT>
__global__ void __launch_bounds__(RowCTA<TPR, CT>::threads,
                                  RowCTA<TPR, CT>::threads > 256
                                      ? (PAIR_OUT ? 2048 / RowCTA<TPR, CT>::threads : 1)
                                      : RowCTA<TPR, CT>::per256(PAIR_OUT ? 8
                                                                : ATTN   ? GBX_ATTN_SM_MIN_CTAS
                                                                         : GBX_SM_MIN_CTAS))
softmax_vec_kernel(const float* in, float* out, float* out_lo, int64_t rows, int L, ScoreEpilogue ep)
{
    grid_dependency_wait();   // see launch_row_kernel
    allow_dependents();
    using C = RowCTA<TPR, CT>;
    __shared__ float red[2][C::warps];
    const int n4 = L >> 2;
    const int lane = threadIdx.x & (TPR - 1);
    const int64_t row = (int64_t)blockIdx.x * C::rows + threadIdx.x / TPR;
    const bool valid = row < rows;
    const int64_t off = row * L;

    // last visible column of this row (attention variant; rows < 2^32 there)
    int last = L - 1;
    float rscale = 1.0f;
    if (ATTN) {
        if (ep.causal) {
            const uint32_t r32 = valid ? (uint32_t)row : 0u;
            const uint32_t p = r32 - fast_div(r32, ep.div_S) * (uint32_t)ep.S;
            last = (int)min((int64_t)L - 1, (int64_t)p + ep.q_off);
        }
        rscale = 1.0f / ep.scale;
    }

    float4 v[V4];
#pragma unroll
    for (int k = 0; k < V4; ++k) {
        const int c = k * TPR + lane;
        // chunks entirely past `last` are never read
        const bool need = valid && c < n4 && (!ATTN || 4 * c <= last);
        v[k] = need ? ld_stream(in + off + 4 * c) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        if (ATTN && c < n4) {
            float* e = &v[k].x;
            if (4 * c + 3 <= last) {
#pragma unroll
                for (int j = 0; j < 4; ++j) e[j] = POW2 ? e[j] * rscale : div_by(e[j], ep.scale, rscale);
            } else if (4 * c > last) {
                v[k] = make_float4(-1e9f, -1e9f, -1e9f, -1e9f);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    e[j] = (4 * c + j > last) ? -1e9f : (POW2 ? e[j] * rscale : div_by(e[j], ep.scale, rscale));
            }
        }
    }
    float m = -1e30f;
#pragma unroll
    for (int k = 0; k < V4; ++k) m = fmaxf(m, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
    m = row_max<TPR>(m, red[0]);

    // every masked entry holds -1e9f, so they all share one exponential
    const float e_mask = ATTN ? expf(-1e9f - m) : 0.0f;
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < V4; ++k) {
        const int c = k * TPR + lane;
        if (c < n4) {
            if (ATTN && 4 * c > last) {
                v[k] = make_float4(e_mask, e_mask, e_mask, e_mask);
            } else {
                const float4 dv = sub4s(v[k], m);
                v[k] = make_float4(expf(dv.x), expf(dv.y), expf(dv.z), expf(dv.w));
            }
            s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
        }
    }
    s = row_sum<TPR>(s, red[1]);

    // PAIR_OUT: columns written (a multiple of 4)
    const int wend = (PAIR_OUT && ATTN && ep.causal && ep.q_off == 0) ? min(L, ((last + 256) >> 8) << 8) : L;
    if (valid) {
        const float r = 1.0f / s;
#pragma unroll
        for (int k = 0; k < V4; ++k) {
            const int c = k * TPR + lane;
            if (c < n4 && (!PAIR_OUT || 4 * c < wend)) {
                const float4 q = div4_by(v[k], s, r);
                if constexpr (PAIR_OUT) {
                    float4 hi, lo;
                    split4(q, hi, lo);
                    st_stream(out + off + 4 * c, hi);
                    st_stream(out_lo + off + 4 * c, lo);
                } else {
                    st_stream(out + off + 4 * c, q);
                }
            }
        }
    }
}

// General path (any L, any alignment, rows longer than the register path):
// one CTA per row, the reference's three passes with shuffle reductions.
template <bool ATTN, bool PAIR_OUT>
__global__ void __launch_bounds__(kGeneralCTA)
softmax_general_kernel(const float* in, float* out, float* out_lo, int64_t rows, int L, ScoreEpilogue ep)
{
    __shared__ float red[2][kGeneralCTA / 32];
    const float rscale = ATTN ? 1.0f / ep.scale : 1.0f;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float* ir = in + row * L;
        float* orow = out + row * L;
        const int last = (ATTN && ep.causal) ? (int)min((int64_t)L - 1, row % ep.S + ep.q_off) : L - 1;
        auto val = [&](int i) -> float {
            if (!ATTN) return ir[i];
            return i > last ? -1e9f : div_by(ir[i], ep.scale, rscale);
        };
        float m = -1e30f;
        for (int i = threadIdx.x; i < L; i += kGeneralCTA) m = fmaxf(m, val(i));
        m = block_max(m, red[0]);
        float s = 0.0f;
        for (int i = threadIdx.x; i < L; i += kGeneralCTA) {
            const float e = expf(val(i) - m);
            orow[i] = e;
            s += e;
        }
        s = block_sum(s, red[1]);
        const float r = 1.0f / s;
        const int wend = (PAIR_OUT && ATTN && ep.causal && ep.q_off == 0) ? min(L, ((last + 256) >> 8) << 8) : L;
        for (int i = threadIdx.x; i < wend; i += kGeneralCTA) {
            const float q = div_by(orow[i], s, r);
            if constexpr (PAIR_OUT) {
                float hv, lv;
                split_value(q, hv, lv);
                orow[i] = hv;
                out_lo[row * L + i] = lv;
            } else {
                orow[i] = q;
            }
        }
        __syncthreads();
    }
}

static bool is_pow2(float x)
{
    int e;
    return x > 0.0f && frexpf(x, &e) == 0.5f;
}

template <int TPR, int V4, bool ATTN, bool PAIR_OUT>
static int launch_softmax_vec(const float* in, float* out, float* out_lo, int64_t rows, int L, ScoreEpilogue ep,
                              cudaStream_t stream)
{
    const int64_t grid256 = row_grid<TPR, 256>(rows);
    auto go = [&](auto ct) -> int {
        constexpr int CT = decltype(ct)::value;
        const int64_t g = row_grid<TPR, CT>(rows);
        if (g < 0) return GBX_ERANGE;
        const dim3 grid((unsigned)g), block(RowCTA<TPR, CT>::threads);
        if (ATTN && is_pow2(ep.scale))
            launch_row_kernel(softmax_vec_kernel<TPR, V4, ATTN, true, PAIR_OUT, CT>, grid, block, 0, stream, in, out,
                              out_lo, rows, L, ep);
        else
            launch_row_kernel(softmax_vec_kernel<TPR, V4, ATTN, false, PAIR_OUT, CT>, grid, block, 0, stream, in, out,
                              out_lo, rows, L, ep);
        return GBX_OK;
    };
    if constexpr (ATTN)
        return go(std::integral_constant<int, 128>());
    else if (grid256 >= 0 && small_row_grid(grid256))
        return go(std::integral_constant<int, 128>());
    else
        return go(std::integral_constant<int, 256>());
}

template <bool ATTN, bool PAIR_OUT>
static int launch_softmax(const char* what, const float* in, float* out, float* out_lo, int64_t rows, int L,
                          ScoreEpilogue ep, cudaStream_t s)
{
    RowShape shape;
    int rc;
    // the vector path numbers rows in 32 bits for the causal position
    if (L % 4 == 0 && aligned16(in) && aligned16(out) && (!PAIR_OUT || aligned16(out_lo)) &&
        row_shape(L / 4, &shape) && rows <= 0xffffffffLL) {
#define GBX_SM_CALL(T, V) launch_softmax_vec<T, V, ATTN, PAIR_OUT>(in, out, out_lo, rows, L, ep, s)
        rc = GBX_ROW_DISPATCH(shape, GBX_SM_CALL, GBX_ERANGE);
#undef GBX_SM_CALL
        if (rc != GBX_OK) return set_error(rc, "%s: rows=%lld L=%d out of range", what, (long long)rows, L);
    } else {
        const int grid = persistent_grid(softmax_general_kernel<ATTN, PAIR_OUT>, kGeneralCTA, 0, rows, 4);
        if (grid < 1) return GBX_ECUDA;
        softmax_general_kernel<ATTN, PAIR_OUT><<<grid, kGeneralCTA, 0, s>>>(in, out, out_lo, rows, L, ep);
    }
    return check_launch(what);
}

}  // namespace gbx

using namespace gbx;

extern "C" int gbx_softmax_rows(const float* in, float* out, int64_t rows, int L, gbx_stream_t stream)
{
    if (rows < 0 || L <= 0) return set_error(GBX_EINVAL, "gbx_softmax_rows: rows=%lld L=%d", (long long)rows, L);
    if (rows == 0) return GBX_OK;
    if (!in || !out) return set_error(GBX_EINVAL, "gbx_softmax_rows: null pointer");
    ScoreEpilogue ep{1, 0, 1.0f, false, make_fastdiv(1)};
    return launch_softmax<false, false>("gbx_softmax_rows", in, out, nullptr, rows, L, ep,
                                        reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gbx_attn_softmax_rows(const float* scores, float* probs, int64_t rows, int L, int S, int q_off,
                                     float scale, int causal, gbx_stream_t stream)
{
    if (rows < 0 || L <= 0 || S <= 0 || q_off < 0)
        return set_error(GBX_EINVAL, "gbx_attn_softmax_rows: rows=%lld L=%d S=%d q_off=%d", (long long)rows, L, S,
                         q_off);
    if (!(scale >= 1.17549435e-38f) || scale == INFINITY)   // a normal, finite, positive float
        return set_error(GBX_EINVAL, "gbx_attn_softmax_rows: scale=%g must be a normal positive float",
                         (double)scale);
    if (rows == 0) return GBX_OK;
    if (!scores || !probs) return set_error(GBX_EINVAL, "gbx_attn_softmax_rows: null pointer");
    ScoreEpilogue ep{S, q_off, scale, causal != 0, make_fastdiv((uint32_t)S)};
    return launch_softmax<true, false>("gbx_attn_softmax_rows", scores, probs, nullptr, rows, L, ep,
                                       reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gbx_attn_softmax_rows_pair(const float* scores, float* probs_hi, float* probs_lo, int64_t rows, int L,
                                          int S, int q_off, float scale, int causal, gbx_stream_t stream)
{
    if (rows < 0 || L <= 0 || S <= 0 || q_off < 0)
        return set_error(GBX_EINVAL, "gbx_attn_softmax_rows_pair: rows=%lld L=%d S=%d q_off=%d", (long long)rows, L, S,
                         q_off);
    if (!(scale >= 1.17549435e-38f) || scale == INFINITY)
        return set_error(GBX_EINVAL, "gbx_attn_softmax_rows_pair: scale=%g must be a normal positive float",
                         (double)scale);
    if (rows == 0) return GBX_OK;
    if (!scores || !probs_hi || !probs_lo) return set_error(GBX_EINVAL, "gbx_attn_softmax_rows_pair: null pointer");
    if ((const float*)probs_lo == scores || probs_lo == probs_hi)
        return set_error(GBX_EINVAL, "gbx_attn_softmax_rows_pair: probs_lo aliases scores or probs_hi");
    ScoreEpilogue ep{S, q_off, scale, causal != 0, make_fastdiv((uint32_t)S)};
    return launch_softmax<true, true>("gbx_attn_softmax_rows_pair", scores, probs_hi, probs_lo, rows, L, ep,
                                      reinterpret_cast<cudaStream_t>(stream));
}
