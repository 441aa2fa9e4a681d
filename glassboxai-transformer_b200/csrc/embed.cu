// embed.cu -- GGUF f32/f16/bf16 decode and the token+position embedding
// gather/add (replaces GGUFLoader's host dequant, transformer.cu:508-534 and
// :635-650, and embedTokensKernel, transformer.cu:175-185).
//
// The tables stay in their GGUF encoding in HBM; each load brings 4 elements
// (8 bytes of f16/bf16, 16 bytes of f32), which are decoded in registers with
// the reference's exact rules and added in fp32.  Output rows are written
// with streaming 16-byte stores.
#include "gbx_common.cuh"
#include "decode.cuh"
#include "tcgen05.cuh"

namespace gbx {

// ---------------------------------------------------------------------------
// Embedding, vector path.  Work item = (token t, 4-element chunk c), numbered
// t*n4 + c, so the 32 lanes of a warp read 32 consecutive 8- or 16-byte pieces
// of table rows and write 512 consecutive bytes of output.  A full grid of
// CTAs, each thread taking kEmbedU items spaced one CTA width apart: all
// table loads are issued before any arithmetic, the loaded words stay raw
// (2 registers per f16/bf16 item) and are decoded only at the store.  (On
// B200, 8-element items written as two half-coalesced stores per lane, in a
// persistent grid, reached 68% of the copy bandwidth on a bf16 gather; the
// same items decoded right after their loads, 54%; this form 82-90%.)
constexpr int kEmbedThreads = 256;
constexpr int kEmbedU = 4;

template <int WT, int PT>
__global__ void __launch_bounds__(kEmbedThreads)
embed_vec4_kernel(const int32_t* __restrict__ ids, const void* __restrict__ wte,
                  const void* __restrict__ wpe, const int32_t* __restrict__ pos_ids,
                  float* __restrict__ out, uint32_t total, FastDiv div_n4, FastDiv div_seq,
                  int pos_off, int d, int vocab, int n_ctx, int32_t* __restrict__ err)
{
    grid_dependency_wait();   // see launch_row_kernel
    allow_dependents();
    const uint32_t n4 = div_n4.d;
    const uint32_t seq = div_seq.d;
    const uint32_t base = blockIdx.x * (uint32_t)(kEmbedThreads * kEmbedU) + threadIdx.x;
    typename Raw4<WT>::type a[kEmbedU];
    typename Raw4<PT>::type b[kEmbedU];
    uint32_t tok[kEmbedU], col[kEmbedU];
    int bad[kEmbedU];
#pragma unroll
    for (int u = 0; u < kEmbedU; ++u) {
        const uint32_t i = base + u * kEmbedThreads;
        const uint32_t ii = i < total ? i : 0;
        const uint32_t t = fast_div(ii, div_n4);
        tok[u] = t;
        col[u] = ii - t * n4;
        const int32_t id = __ldg(ids + t);
        const int32_t pos = pos_ids ? __ldg(pos_ids + t) : pos_off + (int32_t)(t - fast_div(t, div_seq) * seq);
        bad[u] = ((uint32_t)id >= (uint32_t)vocab ? GBX_EMBED_BAD_ID : 0) |
                 ((uint32_t)pos >= (uint32_t)n_ctx ? GBX_EMBED_BAD_POS : 0);
        if (i < total && !bad[u]) {
            a[u] = load_raw4<WT>(wte, (int64_t)id * d + 4 * col[u]);
            b[u] = load_raw4<PT>(wpe, (int64_t)pos * d + 4 * col[u]);
        } else {
            a[u] = zero_raw4<WT>();
            b[u] = zero_raw4<PT>();
        }
    }
#pragma unroll
    for (int u = 0; u < kEmbedU; ++u) {
        if (base + u * kEmbedThreads >= total) continue;
        if (bad[u] && col[u] == 0 && err) atomicOr(err, bad[u]);
        // one fp32 add per element, as embedTokensKernel (transformer.cu:183);
        // a rejected token's row is zeros (0 + 0).  f16 words are converted
        // by the hardware; the reference's decode turns an f16 -0 into +0,
        // so with an f16 table the reference's sum is never -0: adding +0
        // maps a -0 sum (-0 + -0) to +0 and leaves every other value as it
        // is.  A NaN element gives the GPU's canonical NaN either way.
        constexpr bool kF16 = WT == TF16 || PT == TF16;
        const float4 x = decode4_arith<WT>(a[u]), y = decode4_arith<PT>(b[u]);
        float4 o = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
        if (kF16) o = make_float4(__fadd_rn(o.x, 0.0f), __fadd_rn(o.y, 0.0f), __fadd_rn(o.z, 0.0f), __fadd_rn(o.w, 0.0f));
        st_stream(out + (int64_t)tok[u] * d + 4 * col[u], o);
    }
}

// ---------------------------------------------------------------------------
// Embedding, staged path: table rows of a multiple of 16 bytes in 16-byte
// aligned tables (every GPT-2 width in f32, f16 and bf16).  Each CTA owns
// `tpc` consecutive tokens, about 32 KB of table rows.  Lane j of warp 0
// bulk-copies token j's position row into shared memory (the position needs
// no load), then reads the token's id and bulk-copies its table row; all
// copies complete on one mbarrier as transaction bytes.  The CTA then
// decodes, adds and stores the rows out of shared memory, a warp writing 512
// consecutive bytes per store.  The copy engine keeps ~200 KB of table reads
// in flight per SM without holding registers; the register path above is
// limited by its two dependent loads per item (the id, then the table word)
// and the registers that hold the words in flight.  Measured on B200 against
// the register path, bit-identical: 32,768 bf16 tokens at d 1600, 64.5 ->
// 55.3 us (0.75 -> 0.88 of the copy bandwidth); 131,072 f16 tokens at
// d 4096, 567 -> 514 us (0.87 -> 0.96).
constexpr int kStageThreads = 256;
constexpr int kStageMaxTok = 32;          // tokens per CTA: one copying lane each
constexpr uint32_t kStageBytes = 32768;   // shared-memory bytes per CTA aimed at
constexpr uint64_t kStageWaitNs = kDeviceWaitNs;
constexpr int64_t kStageMinElems = 1 << 20;   // smaller launches take the register path

template <int WT, int PT>
__global__ void __launch_bounds__(kStageThreads)
embed_staged_kernel(const int32_t* __restrict__ ids, const void* __restrict__ wte, const void* __restrict__ wpe,
                    const int32_t* __restrict__ pos_ids, float* __restrict__ out, int64_t n_tok, int tpc,
                    FastDiv div_n4, int seq, int pos_off, int d, int vocab, int n_ctx, int32_t* __restrict__ err,
                    uint64_t first_wait_ns)
{
    extern __shared__ __align__(128) unsigned char stage[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ int bad_s[kStageMaxTok];
    constexpr uint32_t ew = WT == TF32 ? 4 : 2, ep = PT == TF32 ? 4 : 2;
    const uint32_t row_w = (uint32_t)d * ew, row_p = (uint32_t)d * ep;
    const int64_t t0 = (int64_t)blockIdx.x * tpc;
    const int nt = (int)(n_tok - t0 < tpc ? n_tok - t0 : tpc);
    const uint32_t bar_a = tc::smem_u32(&bar);
    const uint32_t sw = tc::smem_u32(stage), sp = sw + (uint32_t)tpc * row_w;

    if (threadIdx.x == 0) {
        tc::mbar_init(bar_a, (uint32_t)nt);
        tc::fence_mbar_init();
    }
    __syncthreads();
    grid_dependency_wait();   // see launch_row_kernel
    allow_dependents();
    if ((int)threadIdx.x < nt) {
        const int j = threadIdx.x;
        const int64_t t = t0 + j;
        const int32_t pos = pos_ids ? __ldg(pos_ids + t) : pos_off + (int32_t)(t % seq);
        int bad = (uint32_t)pos >= (uint32_t)n_ctx ? GBX_EMBED_BAD_POS : 0;
        if (!bad) {
            tc::mbar_expect_tx(bar_a, row_p);
            tc::bulk_load(sp + j * row_p, static_cast<const unsigned char*>(wpe) + (int64_t)pos * row_p, row_p, bar_a);
        }
        const int32_t id = __ldg(ids + t);
        if ((uint32_t)id >= (uint32_t)vocab) bad |= GBX_EMBED_BAD_ID;
        if (!bad) {
            tc::mbar_arrive_expect_tx(bar_a, row_w);
            tc::bulk_load(sw + j * row_w, static_cast<const unsigned char*>(wte) + (int64_t)id * row_w, row_w, bar_a);
        } else {
            tc::mbar_arrive(bar_a);
            if (err) atomicOr(err, bad);
        }
        bad_s[j] = bad;
    }
    __syncthreads();
    // first_wait_ns is kStageWaitNs unless a test shortens it (0: give up at once)
    if (!(first_wait_ns && tc::mbar_wait(bar_a, 0, nullptr, first_wait_ns))) {
        // the copies did not land within the limit: flag it, give the copies
        // in flight one more limit before the shared memory is released, and
        // leave this CTA's rows unwritten
        if (err) atomicOr(err, GBX_EMBED_TIMEOUT);
        tc::mbar_wait(bar_a, 0, nullptr, kStageWaitNs);
        return;
    }
    const uint32_t n4 = div_n4.d;
    const uint32_t items = (uint32_t)nt * n4;
    float* const out0 = out + t0 * d;
#pragma unroll 4
    for (uint32_t i = threadIdx.x; i < items; i += kStageThreads) {
        const uint32_t j = fast_div(i, div_n4), c = i - j * n4;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (!bad_s[j]) {
            // one fp32 add per element and the f16 -0 rule, as embed_vec4_kernel
            const auto a = *reinterpret_cast<const typename Raw4<WT>::type*>(stage + j * row_w + c * 4 * ew);
            const auto b = *reinterpret_cast<const typename Raw4<PT>::type*>(stage + tpc * row_w + j * row_p + c * 4 * ep);
            const float4 x = decode4_arith<WT>(a), y = decode4_arith<PT>(b);
            o = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
            if constexpr (WT == TF16 || PT == TF16)
                o = make_float4(__fadd_rn(o.x, 0.0f), __fadd_rn(o.y, 0.0f), __fadd_rn(o.z, 0.0f), __fadd_rn(o.w, 0.0f));
        }
        st_stream(out0 + (int64_t)j * d + 4 * c, o);
    }
}

// General path: any d, any alignment, 64-bit indexing; one element per item.
template <int WT, int PT>
__global__ void __launch_bounds__(256)
embed_scalar_kernel(const int32_t* __restrict__ ids, const void* __restrict__ wte,
                    const void* __restrict__ wpe, const int32_t* __restrict__ pos_ids,
                    float* __restrict__ out, int64_t n_tok, int seq, int pos_off, int d, int vocab,
                    int n_ctx, int32_t* __restrict__ err)
{
    const int64_t total = n_tok * d;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / d;
        const int c = (int)(i - t * d);
        const int32_t id = __ldg(ids + t);
        const int64_t pos = pos_ids ? (int64_t)__ldg(pos_ids + t) : (int64_t)pos_off + t % seq;
        const bool bad_id = (uint32_t)id >= (uint32_t)vocab;
        const bool bad_pos = pos < 0 || pos >= n_ctx;
        float v = 0.0f;
        if (!bad_id && !bad_pos) v = load1<WT>(wte, (int64_t)id * d + c) + load1<PT>(wpe, pos * d + c);
        else if (c == 0 && err)
            atomicOr(err, (bad_id ? GBX_EMBED_BAD_ID : 0) | (bad_pos ? GBX_EMBED_BAD_POS : 0));
        out[i] = v;
    }
}

// ---------------------------------------------------------------------------
// Dequant: full grid of 4-element items on the vector path, scalar tail.
template <int T>
__global__ void __launch_bounds__(256)
dequant_vec4_kernel(const void* __restrict__ src, float* __restrict__ dst, int64_t n4)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n4) st_stream(dst + i * 4, decode4<T>(load_raw4<T>(src, i * 4)));
}

template <int T>
__global__ void __launch_bounds__(256)
dequant_scalar_kernel(const void* __restrict__ src, float* __restrict__ dst, int64_t begin, int64_t n)
{
    for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = load1<T>(src, i);
}

template <int WT, int PT>
static int launch_embed(const int32_t* ids, const void* wte, const void* wpe, const int32_t* pos_ids,
                        float* out, int64_t n_tok, int seq, int pos_off, int d, int vocab, int n_ctx,
                        int32_t* err, cudaStream_t stream)
{
    const int n4 = d / 4;
    const int64_t total = n_tok * (int64_t)n4;
    const int es_w = WT == TF32 ? 4 : 2, es_p = PT == TF32 ? 4 : 2;
    // 32-bit item numbers (total < 2^31) and table rows aligned for the
    // 16-byte (f32) or 8-byte (f16/bf16) loads
    const bool vec = (d % 4 == 0) && total < 0x7fffffffLL && aligned16(out) &&
                     ((uintptr_t)wte % (4 * es_w)) == 0 && ((uintptr_t)wpe % (4 * es_p)) == 0;
    const int64_t row_w = (int64_t)d * es_w, row_p = (int64_t)d * es_p;
    int tpc = (int)(kStageBytes / (row_w + row_p));
    tpc = tpc < 1 ? 1 : (tpc > kStageMaxTok ? kStageMaxTok : tpc);
    const int64_t smem = tpc * (row_w + row_p);
    const int64_t grid_s = (n_tok + tpc - 1) / tpc;
    DeviceInfo di;
    // below ~1M elements a launch is latency-bound, and the register path's
    // shorter chain (no barrier set-up) measured 0.5 us faster on B200
    const bool staged = vec && n_tok * d >= kStageMinElems && row_w % 16 == 0 && row_p % 16 == 0 &&
                        aligned16(wte) && aligned16(wpe) &&
                        grid_s <= 0x7fffffffLL && device_info(&di) == GBX_OK && smem <= di.max_smem_optin;
    if (staged) {
        auto k = embed_staged_kernel<WT, PT>;
        if (smem > 48 * 1024 && cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return check_launch("gbx_embed");
        launch_row_kernel(k, dim3((unsigned)grid_s), dim3(kStageThreads), (size_t)smem, stream, ids, wte, wpe, pos_ids,
                          out, n_tok, tpc, make_fastdiv((uint32_t)n4), seq, pos_off, d, vocab, n_ctx, err,
                          first_wait_limit_ns());
    } else if (vec) {
        const int64_t per_cta = (int64_t)kEmbedThreads * kEmbedU;
        const int64_t grid = (total + per_cta - 1) / per_cta;
        launch_row_kernel(embed_vec4_kernel<WT, PT>, dim3((unsigned)grid), dim3(kEmbedThreads), 0, stream, ids, wte,
                          wpe, pos_ids, out, (uint32_t)total, make_fastdiv((uint32_t)n4),
                          make_fastdiv((uint32_t)seq), pos_off, d, vocab, n_ctx, err);
    } else {
        auto k = embed_scalar_kernel<WT, PT>;
        const int64_t total_e = n_tok * (int64_t)d;
        const int grid = persistent_grid(k, 256, 0, (total_e + 255) / 256, 4);
        if (grid < 1) return GBX_ECUDA;
        k<<<grid, 256, 0, stream>>>(ids, wte, wpe, pos_ids, out, n_tok, seq, pos_off, d, vocab, n_ctx, err);
    }
    return check_launch("gbx_embed");
}

template <int WT>
static int launch_embed_p(int pt, const int32_t* ids, const void* wte, const void* wpe,
                          const int32_t* pos_ids, float* out, int64_t n_tok, int seq, int pos_off,
                          int d, int vocab, int n_ctx, int32_t* err, cudaStream_t s)
{
    switch (pt) {
    case TF32: return launch_embed<WT, TF32>(ids, wte, wpe, pos_ids, out, n_tok, seq, pos_off, d, vocab, n_ctx, err, s);
    case TF16: return launch_embed<WT, TF16>(ids, wte, wpe, pos_ids, out, n_tok, seq, pos_off, d, vocab, n_ctx, err, s);
    default: return launch_embed<WT, TBF16>(ids, wte, wpe, pos_ids, out, n_tok, seq, pos_off, d, vocab, n_ctx, err, s);
    }
}

template <int T>
static int launch_dequant(const void* src, float* dst, int64_t n, cudaStream_t stream)
{
    int64_t done = 0;
    const int es = T == TF32 ? 4 : 2;
    if (((uintptr_t)src % (4 * es)) == 0 && aligned16(dst) && n >= 4) {
        const int64_t n4 = n / 4;
        const int64_t grid = (n4 + 255) / 256;
        if (grid <= 0x7fffffffLL) {
            dequant_vec4_kernel<T><<<(unsigned)grid, 256, 0, stream>>>(src, dst, n4);
            done = n4 * 4;
        }
    }
    if (done < n) {
        auto k = dequant_scalar_kernel<T>;
        const int grid = persistent_grid(k, 256, 0, (n - done + 255) / 256, 4);
        if (grid < 1) return GBX_ECUDA;
        k<<<grid, 256, 0, stream>>>(src, dst, done, n);
    }
    return check_launch("gbx_dequant");
}

}  // namespace gbx

using namespace gbx;

extern "C" int gbx_dequant(const void* src, int dtype, float* dst, int64_t n, gbx_stream_t stream)
{
    const int t = dtype_index(dtype);
    if (t < 0) return set_error(GBX_EDTYPE, "gbx_dequant: unsupported GGUF dtype %d", dtype);
    if (n < 0) return set_error(GBX_EINVAL, "gbx_dequant: n=%lld", (long long)n);
    if (n == 0) return GBX_OK;
    if (!src || !dst) return set_error(GBX_EINVAL, "gbx_dequant: null pointer");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (t) {
    case TF32: return launch_dequant<TF32>(src, dst, n, s);
    case TF16: return launch_dequant<TF16>(src, dst, n, s);
    default: return launch_dequant<TBF16>(src, dst, n, s);
    }
}

extern "C" int gbx_embed(const int32_t* ids, const void* wte, int wte_dtype, const void* wpe,
                         int wpe_dtype, const int32_t* pos_ids, float* out, int64_t n_tok, int seq,
                         int pos_off, int d, int vocab, int n_ctx, int32_t* err_flag,
                         gbx_stream_t stream)
{
    const int wt = dtype_index(wte_dtype), pt = dtype_index(wpe_dtype);
    if (wt < 0 || pt < 0)
        return set_error(GBX_EDTYPE, "gbx_embed: unsupported GGUF dtype (wte %d, wpe %d)", wte_dtype, wpe_dtype);
    if (n_tok < 0 || d <= 0 || vocab <= 0 || n_ctx <= 0)
        return set_error(GBX_EINVAL, "gbx_embed: n_tok=%lld d=%d vocab=%d n_ctx=%d", (long long)n_tok, d, vocab, n_ctx);
    if (n_tok == 0) return GBX_OK;
    if (!ids || !wte || !wpe || !out) return set_error(GBX_EINVAL, "gbx_embed: null pointer");
    if (!pos_ids) {
        if (seq <= 0) return set_error(GBX_EINVAL, "gbx_embed: seq=%d", seq);
        const int64_t span = n_tok < seq ? n_tok : seq;
        if (pos_off < 0 || (int64_t)pos_off + span > n_ctx)
            return set_error(GBX_ERANGE, "gbx_embed: positions [%d, %lld) exceed n_ctx=%d", pos_off,
                             (long long)pos_off + span, n_ctx);
    } else if (seq <= 0) {
        seq = 1;
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (wt) {
    case TF32: return launch_embed_p<TF32>(pt, ids, wte, wpe, pos_ids, out, n_tok, seq, pos_off, d, vocab, n_ctx, err_flag, s);
    case TF16: return launch_embed_p<TF16>(pt, ids, wte, wpe, pos_ids, out, n_tok, seq, pos_off, d, vocab, n_ctx, err_flag, s);
    default: return launch_embed_p<TBF16>(pt, ids, wte, wpe, pos_ids, out, n_tok, seq, pos_off, d, vocab, n_ctx, err_flag, s);
    }
}
