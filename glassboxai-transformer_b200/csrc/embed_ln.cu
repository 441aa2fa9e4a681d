// embed_ln.cu -- the token + position embedding fused with the first
// LayerNorm: embedTokensKernel (transformer.cu:175-185) followed by the
// layer-0 layerNormKernel launch of attentionBlock (:828), in one pass.
//
// A row group of TPR threads owns one token: it reads the token's id, loads
// its wte and wpe rows in their GGUF encoding (4 elements per load), forms
// h = dec(wte) + dec(wpe) in registers with the embedding's exact fp32 add,
// stores h once and, from the same registers, the LayerNorm of h (mean, the
// two-pass variance and the affine map, with layernorm.cu's arithmetic).
// h is never re-read from HBM: against gbx_embed + gbx_layernorm the pass
// saves one read of the [n_tok, d] fp32 rows and one launch.
//
// Shapes: one warp per token for d 516..2048 (up to 16 float4s per lane),
// otherwise the row groups of the LayerNorm kernels (rows.cuh: the smallest
// power-of-two group, 1 to 1024 threads, holding at most 4 float4s per
// thread; d up to 16384).  Mixed table dtypes or unaligned operands run
// gbx_embed then gbx_layernorm (h identical; y within the LayerNorm
// tolerance, the sums being taken in another order).
#include "decode.cuh"
#include "rows.cuh"
#include "tf32.cuh"

namespace gbx {

// Resident CTAs per SM the one-warp-per-token form is compiled for (its
// register budget: 65536 / (256 x this)).  4 (64 registers, a few bytes of
// spill) measured on B200 against the compiler's free choice (80 registers,
// 3 CTAs): 49.5 vs 53.7 us at d 768 (f32 tables), 94.6 vs 96.0 us at d 1600
// (bf16), equal at d 1024 (f16), 32,768 tokens each.
#ifndef GBX_EMBED_LN_WARP_MIN_CTAS
#define GBX_EMBED_LN_WARP_MIN_CTAS 4
#endif

// CTAs of 128 threads (rows.cuh): the same time as 256 for the XL prefill's
// 32,768 tokens (88.4 us), and twice the CTAs for a decode batch.
constexpr int kElnCTA = 128;
template <int TPR>
using ElnCTA = RowCTA<TPR, kElnCTA>;

template <int T, int TPR, int V4>
__global__ void __launch_bounds__(ElnCTA<TPR>::threads,
                                  TPR == 32 && V4 > 4 ? ElnCTA<TPR>::per256(GBX_EMBED_LN_WARP_MIN_CTAS) : 1)
embed_ln_kernel(const int32_t* __restrict__ ids, const void* __restrict__ wte, const void* __restrict__ wpe,
                const int32_t* __restrict__ pos_ids, float* __restrict__ h_out, float* __restrict__ y,
                float* __restrict__ y_lo, const float* __restrict__ gamma, const float* __restrict__ beta,
                int64_t n_tok, int seq, int pos_off, int d, int vocab, int n_ctx, float eps,
                int32_t* __restrict__ err)
{
    grid_dependency_wait();   // see launch_row_kernel
    allow_dependents();
    __shared__ float red[2][ElnCTA<TPR>::warps];
    const int n4 = d >> 2;
    const int lane = threadIdx.x & (TPR - 1);
    const int64_t t = (int64_t)blockIdx.x * ElnCTA<TPR>::rows + threadIdx.x / TPR;
    const bool valid = t < n_tok;
    const int64_t tt = valid ? t : 0;
    const int32_t id = __ldg(ids + tt);
    const int32_t pos = pos_ids ? __ldg(pos_ids + tt) : pos_off + (int32_t)(tt % seq);
    const int bad = ((uint32_t)id >= (uint32_t)vocab ? GBX_EMBED_BAD_ID : 0) |
                    ((uint32_t)pos >= (uint32_t)n_ctx ? GBX_EMBED_BAD_POS : 0);
    const bool live = valid && !bad;

    // Every lane walks its row through base pointers with compile-time
    // offsets (k * TPR units), and "float4 k * TPR + lane exists" is one
    // compare against lim: the loops below carry no per-element index math.
    using R = typename Raw4<T>::type;
    const int lim = n4 - lane;
    const R* const wrow = reinterpret_cast<const R*>(wte) + (int64_t)(live ? id : 0) * n4 + lane;
    const R* const prow = reinterpret_cast<const R*>(wpe) + (int64_t)(live ? pos : 0) * n4 + lane;
    R a[V4], b[V4];
#pragma unroll
    for (int k = 0; k < V4; ++k) {
        if (live && k * TPR < lim) {
            a[k] = __ldg(wrow + k * TPR);
            b[k] = __ldg(prow + k * TPR);
        } else {
            a[k] = zero_raw4<T>();
            b[k] = zero_raw4<T>();
        }
    }
    if (valid && bad && lane == 0 && err) atomicOr(err, bad);

    // h: one fp32 add per element and the f16 -0 rule, as gbx_embed; a
    // rejected token's row is zeros (its LayerNorm is then beta, as
    // gbx_layernorm of a zero row)
    const int64_t off = t * d;
    float4 v[V4];
#pragma unroll
    for (int k = 0; k < V4; ++k) {
        float4 o = add4(decode4_arith<T>(a[k]), decode4_arith<T>(b[k]));
        if constexpr (T == TF16) o = add4(o, make_float4(0.0f, 0.0f, 0.0f, 0.0f));
        v[k] = o;
    }
    if (h_out && valid) {
        float* const hrow = h_out + off + 4 * lane;
#pragma unroll
        for (int k = 0; k < V4; ++k)
            if (k * TPR < lim) st_stream(hrow + 4 * k * TPR, v[k]);
    }

    // LayerNorm of h, the arithmetic of ln_vec_kernel (layernorm.cu)
    const float fd = (float)d;
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < V4; ++k) s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    s = row_sum<TPR>(s, red[0]);
    const float mean = s / fd;
    float qs = 0.0f;
#pragma unroll
    for (int k = 0; k < V4; ++k) {
        if (k * TPR < lim) {
            const float4 dv = sub4s(v[k], mean);
            qs = fmaf(dv.x, dv.x, qs);
            qs = fmaf(dv.y, dv.y, qs);
            qs = fmaf(dv.z, dv.z, qs);
            qs = fmaf(dv.w, dv.w, qs);
        }
    }
    qs = row_sum<TPR>(qs, red[1]);
    const float inv = rsqrtf(qs / fd + eps);
    if (!valid) return;
    float* const yrow = y + off + 4 * lane;
    if (gamma && beta && !y_lo) {
        // the common case, with no per-element pointer tests
        const float* const grow = gamma + 4 * lane;
        const float* const brow = beta + 4 * lane;
#pragma unroll
        for (int k = 0; k < V4; ++k) {
            if (k * TPR < lim) {
                const float4 g = ld_param4(grow + 4 * k * TPR), bb = ld_param4(brow + 4 * k * TPR);
                st_stream(yrow + 4 * k * TPR, ln_affine4(v[k], mean, inv, g, bb));
            }
        }
        return;
    }
#pragma unroll
    for (int k = 0; k < V4; ++k) {
        const int c = k * TPR + lane;
        if (k * TPR < lim) {
            const float4 g = gamma ? ld_param4(gamma + 4 * c) : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
            const float4 bb = beta ? ld_param4(beta + 4 * c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            const float4 o = ln_affine4(v[k], mean, inv, g, bb);
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

template <int T, int TPR, int V4>
static int launch_embed_ln_v(const int32_t* ids, const void* wte, const void* wpe, const int32_t* pos_ids,
                             float* h_out, float* y, float* y_lo, const float* g, const float* b, int64_t n_tok,
                             int seq, int pos_off, int d, int vocab, int n_ctx, float eps, int32_t* err,
                             cudaStream_t s)
{
    const int64_t grid = row_grid<TPR, kElnCTA>(n_tok);
    if (grid < 0) return GBX_ERANGE;
    launch_row_kernel(embed_ln_kernel<T, TPR, V4>, dim3((unsigned)grid), dim3(ElnCTA<TPR>::threads), 0, s, ids, wte,
                      wpe, pos_ids, h_out, y, y_lo, g, b, n_tok, seq, pos_off, d, vocab, n_ctx, eps, err);
    return GBX_OK;
}

// Token rows of 5..16 float4s per lane run one warp per token (no barrier;
// the id -> row gather chain of many independent warps hides its latency):
// measured on B200 for 32,768 bf16 tokens at d 1600, 88.5 us against 94.7 us
// for the 128-thread row group (ncu: 2.6 times the instructions per token).
// Other widths take the row groups of the LayerNorm kernels (rows.cuh).
constexpr int kEmbedLnWarpMaxV4 = 16;

template <int T>
static int launch_embed_ln(const RowShape& shape, int n4, const int32_t* ids, const void* wte, const void* wpe,
                           const int32_t* pos_ids, float* h_out, float* y, float* y_lo, const float* g,
                           const float* b, int64_t n_tok, int seq, int pos_off, int d, int vocab, int n_ctx,
                           float eps, int32_t* err, cudaStream_t s)
{
#define GBX_ELN(TP, V) \
    launch_embed_ln_v<T, TP, V>(ids, wte, wpe, pos_ids, h_out, y, y_lo, g, b, n_tok, seq, pos_off, d, vocab, n_ctx, \
                                eps, err, s)
    if (n4 > 32 * kRowMaxV4 && n4 <= 32 * kEmbedLnWarpMaxV4) {
        switch ((n4 + 31) / 32) {
        case 5: return GBX_ELN(32, 5);
        case 6: return GBX_ELN(32, 6);
        case 7: return GBX_ELN(32, 7);
        case 8: return GBX_ELN(32, 8);
        case 9: return GBX_ELN(32, 9);
        case 10: return GBX_ELN(32, 10);
        case 11: return GBX_ELN(32, 11);
        case 12: return GBX_ELN(32, 12);
        case 13: return GBX_ELN(32, 13);
        case 14: return GBX_ELN(32, 14);
        case 15: return GBX_ELN(32, 15);
        case 16: return GBX_ELN(32, 16);
        }
        return GBX_ERANGE;
    }
    return GBX_ROW_DISPATCH(shape, GBX_ELN, GBX_ERANGE);
#undef GBX_ELN
}

}  // namespace gbx

using namespace gbx;

extern "C" int gbx_embed_layernorm(const int32_t* ids, const void* wte, int wte_dtype, const void* wpe,
                                   int wpe_dtype, const int32_t* pos_ids, float* h_out, float* y, float* y_lo,
                                   const float* gamma, const float* beta, int64_t n_tok, int seq, int pos_off, int d,
                                   int vocab, int n_ctx, float eps, int32_t* err_flag, gbx_stream_t stream)
{
    const int wt = dtype_index(wte_dtype), pt = dtype_index(wpe_dtype);
    if (wt < 0 || pt < 0)
        return set_error(GBX_EDTYPE, "gbx_embed_layernorm: unsupported GGUF dtype (wte %d, wpe %d)", wte_dtype,
                         wpe_dtype);
    if (n_tok < 0 || d <= 0 || vocab <= 0 || n_ctx <= 0)
        return set_error(GBX_EINVAL, "gbx_embed_layernorm: n_tok=%lld d=%d vocab=%d n_ctx=%d", (long long)n_tok, d,
                         vocab, n_ctx);
    if (n_tok == 0) return GBX_OK;
    if (!ids || !wte || !wpe || !y) return set_error(GBX_EINVAL, "gbx_embed_layernorm: null pointer");
    if ((h_out && (y == h_out || y_lo == h_out)) || (y_lo && y_lo == y))
        return set_error(GBX_EINVAL, "gbx_embed_layernorm: h_out, y and y_lo must differ");
    if (!pos_ids) {
        if (seq <= 0) return set_error(GBX_EINVAL, "gbx_embed_layernorm: seq=%d", seq);
        const int64_t span = n_tok < seq ? n_tok : seq;
        if (pos_off < 0 || (int64_t)pos_off + span > n_ctx)
            return set_error(GBX_ERANGE, "gbx_embed_layernorm: positions [%d, %lld) exceed n_ctx=%d", pos_off,
                             (long long)pos_off + span, n_ctx);
    } else if (seq <= 0) {
        seq = 1;
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int es = wt == TF32 ? 4 : 2;
    RowShape shape;
    const bool fused = wt == pt && d % 4 == 0 && row_shape(d / 4, &shape) && aligned16(y) &&
                       (!h_out || aligned16(h_out)) && (!y_lo || aligned16(y_lo)) &&
                       ((uintptr_t)wte % (4 * es)) == 0 && ((uintptr_t)wpe % (4 * es)) == 0 &&
                       (!gamma || aligned16(gamma)) && (!beta || aligned16(beta));
    if (!fused) {
        // the unfused pair: h into h_out (or into y, then normalised in place)
        float* h = h_out ? h_out : y;
        int rc = gbx_embed(ids, wte, wte_dtype, wpe, wpe_dtype, pos_ids, h, n_tok, seq, pos_off, d, vocab, n_ctx,
                           err_flag, stream);
        if (rc != GBX_OK) return rc;
        return y_lo ? gbx_layernorm_pair(h, y, y_lo, gamma, beta, n_tok, d, eps, stream)
                    : gbx_layernorm(h, y, gamma, beta, n_tok, d, eps, stream);
    }
    int rc;
    switch (wt) {
    case TF32:
        rc = launch_embed_ln<TF32>(shape, d / 4, ids, wte, wpe, pos_ids, h_out, y, y_lo, gamma, beta, n_tok, seq, pos_off,
                                   d, vocab, n_ctx, eps, err_flag, s);
        break;
    case TF16:
        rc = launch_embed_ln<TF16>(shape, d / 4, ids, wte, wpe, pos_ids, h_out, y, y_lo, gamma, beta, n_tok, seq, pos_off,
                                   d, vocab, n_ctx, eps, err_flag, s);
        break;
    default:
        rc = launch_embed_ln<TBF16>(shape, d / 4, ids, wte, wpe, pos_ids, h_out, y, y_lo, gamma, beta, n_tok, seq,
                                    pos_off, d, vocab, n_ctx, eps, err_flag, s);
        break;
    }
    if (rc != GBX_OK) return set_error(rc, "gbx_embed_layernorm: n_tok=%lld d=%d out of range", (long long)n_tok, d);
    return check_launch("gbx_embed_layernorm");
}
