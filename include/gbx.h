/*
 * gbx.h -- C ABI of the B200 (sm_100a) layer-kernel hot path for
 * GlassBoxAI-Transformer: token+position embedding gather/add from GGUF
 * f32/f16/bf16 tables, residual-add + LayerNorm, bias + GELU(tanh), and the
 * row softmax.
 *
 * Conventions (all entry points):
 *   - Every pointer argument is a DEVICE pointer unless its name ends in
 *     `_host`.  Callers own every buffer; nothing here allocates per call.
 *   - Work is enqueued asynchronously on `stream` (NULL = the legacy default
 *     stream, which is what the reference uses).  Entry points are stateless
 *     and safe to call from several host threads at once.  Three process-wide
 *     settings exist, none needed for correct results: gbx_set_pdl,
 *     gbx_linear_set_tiles and (for tests) gbx_set_first_wait_limit; change
 *     them while no other host thread is launching.
 *   - Return GBX_OK (0) or a GBX_E* code; they never exit the process
 *     (the reference's CUDA_CHECK prints and calls exit(1),
 *     transformer.cu:24-32).  gbx_last_error() gives a one-line reason,
 *     per host thread.
 *   - dtype codes are GGUF's: 0 = f32, 1 = f16, 30 = bf16
 *     (transformer.cu:635-650 accepts exactly these three).
 *   - Rows are contiguous (row stride = row length).  Outputs may alias the
 *     matching input where stated; rows are processed whole, so aliasing is
 *     safe exactly as stated.
 *   - Fast paths need 16-byte aligned activation pointers and a row length
 *     that is a multiple of 4 (embed: d a multiple of 4 and tables aligned
 *     to 4 elements); other shapes run a slower general kernel on the GPU
 *     with the same results.
 */
#ifndef GBX_H
#define GBX_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct CUstream_st;
typedef struct CUstream_st* gbx_stream_t; /* identical to cudaStream_t */

enum {
    GBX_OK = 0,
    GBX_EINVAL = 1,    /* bad argument: null pointer, negative size, forbidden alias */
    GBX_EDTYPE = 2,    /* dtype code other than 0 / 1 / 30 */
    GBX_ERANGE = 3,    /* a size or position beyond what the call supports */
    GBX_ECUDA = 4,     /* the CUDA runtime reported an error (launch or copy) */
    GBX_EIO = 5,       /* file could not be opened / read / parsed */
    GBX_ENOTFOUND = 6, /* no tensor under any of the given names */
    GBX_ENOMEM = 7     /* device or host allocation failed (model set-up only) */
};

enum { GBX_DT_F32 = 0, GBX_DT_F16 = 1, GBX_DT_BF16 = 30 };

/* Bits set in *err_flag by gbx_embed (device int32, OR-ed in).
 * GBX_EMBED_TIMEOUT: a staged copy of table rows did not complete within one
 * second; the rows it fed are left unwritten (the kernel returns without
 * faulting). */
enum { GBX_EMBED_BAD_ID = 1, GBX_EMBED_BAD_POS = 2, GBX_EMBED_TIMEOUT = 4 };

/* Library version, major*10000 + minor*100 + patch. */
int gbx_version(void);
/* Static name of a status code. */
const char* gbx_status_string(int status);
/* Detail of the last failing call made by this host thread ("" if none). */
const char* gbx_last_error(void);

/*
 * Programmatic dependent launch for the row kernels (embed, LayerNorm,
 * residual + LayerNorm, bias + GELU, softmax), process-wide, off by default.
 * When on, each of these kernels may be scheduled while the previous kernel
 * on its stream drains, and waits on the device for that kernel's
 * completion before touching memory: results are unchanged, launch gaps
 * shrink (most visible in chains of small launches and in CUDA graphs).
 * Returns the previous setting.
 */
int gbx_set_pdl(int enable);

/*
 * Limit of the first consumer wait of the staged embedding (the CTA waiting
 * for its table rows' bulk copies) and of the tensor-core contractions (the
 * MMA thread waiting for its first tile loads), process-wide, in ns of
 * %globaltimer time; 1 s by default, like every other device wait here.  0
 * makes that wait give up at once, so a test can drive the timeout path:
 * the kernel sets GBX_EMBED_TIMEOUT / GBX_LINEAR_TIMEOUT in *err_flag, waits
 * (with the full 1 s limit) for the copies or MMAs it already started,
 * frees what it holds and returns, leaving its outputs unwritten.  No
 * counterpart in the reference (whose CUDA_CHECK exits the process,
 * transformer.cu:24-32).  Returns the previous limit.  For tests only.
 */
uint64_t gbx_set_first_wait_limit(uint64_t ns);

/*
 * GGUF tensor decode to fp32 on the device, bit-identical to the reference's
 * host dequant GGUFLoader::loadTensorByIndex (transformer.cu:635-650) with
 * float16ToFloat32 (:508-527: -0 -> +0, every NaN -> 0x7fc00000, subnormals
 * exact) and bfloat16ToFloat32 (:529-534: bits << 16).  n elements.
 * Replaces the host loop behind GGUFLoader::getTensorGPU (:676-695).
 */
int gbx_dequant(const void* src, int dtype, float* dst, int64_t n, gbx_stream_t stream);

/*
 * Token + position embedding, replacing embedTokensKernel / embedTokens
 * (transformer.cu:175-185, 805-815):
 *   out[t*d + i] = dec(wte[ids[t]*d + i]) + dec(wpe[pos(t)*d + i])
 * with dec() the reference decode above and one fp32 add (bit-exact with the
 * reference).  The tables stay in their GGUF dtype on the device (no fp32
 * copy).  pos(t) = pos_ids ? pos_ids[t] : pos_off + (t % seq); `seq` is the
 * sequence length of a batch of n_tok/seq sequences (the reference has one
 * sequence, pos = t).  Tokens whose id is outside [0, vocab) or whose
 * position is outside [0, n_ctx) get an all-zero row, and the matching
 * GBX_EMBED_* bit is OR-ed into *err_flag (a device int32; may be NULL).
 * The reference reads out of bounds in that case.  Without pos_ids the
 * position range is checked on the host (GBX_ERANGE).
 * out: [n_tok, d] fp32; wte: [vocab, d]; wpe: [n_ctx, d].
 */
int gbx_embed(const int32_t* ids, const void* wte, int wte_dtype, const void* wpe, int wpe_dtype,
              const int32_t* pos_ids, float* out, int64_t n_tok, int seq, int pos_off, int d,
              int vocab, int n_ctx, int32_t* err_flag, gbx_stream_t stream);

/*
 * Embedding fused with the first LayerNorm: gbx_embed followed by
 * gbx_layernorm (or gbx_layernorm_pair when y_lo is given) in one pass,
 * replacing embedTokensKernel (transformer.cu:175-185) and the layer-0
 * layerNormKernel launch of attentionBlock (:828):
 *   h = gbx_embed(ids, wte, wpe, ...)         into h_out (may be NULL: not stored)
 *   y = LayerNorm(h) with gamma, beta, eps   (y_lo non-NULL: y, y_lo its tf32 pair)
 * h is bit-identical to gbx_embed's, err_flag receives the same GBX_EMBED_*
 * bits, and a rejected token's h row is zeros (its y row is then beta, as
 * gbx_layernorm of a zero row).  y is within the LayerNorm tolerance of
 * gbx_layernorm(h) (the row sums are taken in another order).  h is never
 * re-read from memory.  Fused for wte_dtype == wpe_dtype, d a multiple of 4
 * up to 16384 and 16-byte aligned rows; other cases run the two calls.
 * h_out, y and y_lo must be distinct, non-overlapping [n_tok, d] buffers.
 */
int gbx_embed_layernorm(const int32_t* ids, const void* wte, int wte_dtype, const void* wpe, int wpe_dtype,
                        const int32_t* pos_ids, float* h_out, float* y, float* y_lo, const float* gamma,
                        const float* beta, int64_t n_tok, int seq, int pos_off, int d, int vocab, int n_ctx, float eps,
                        int32_t* err_flag, gbx_stream_t stream);

/*
 * LayerNorm over rows of length d, replacing layerNormKernel
 * (transformer.cu:77-124, launched at :828, :868, :896):
 *   mean = sum(x)/d; var = sum((x-mean)^2)/d; inv = rsqrtf(var + eps);
 *   y = ((x - mean) * inv) * gamma + beta
 * gamma / beta may be NULL (treated as 1 / 0, as at :120-121).  y may alias x.
 */
int gbx_layernorm(const float* x, float* y, const float* gamma, const float* beta, int64_t rows,
                  int d, float eps, gbx_stream_t stream);

/*
 * gbx_layernorm with the output as the tf32 pair gbx_linear reads as its x
 * operand: y_hi, y_lo are exactly gbx_split_tf32 of gbx_layernorm's y, in
 * one pass (no fp32 copy of y).  No counterpart in the reference: it feeds
 * the QKV and FFN-up contractions.  y_hi may alias x; y_lo may not.
 */
int gbx_layernorm_pair(const float* x, float* y_hi, float* y_lo, const float* gamma, const float* beta,
                       int64_t rows, int d, float eps, gbx_stream_t stream);

/*
 * Fused residual add + LayerNorm.  Replaces the residual epilogue of
 * projectionKernel / ffnDownKernel (transformer.cu:262, :292:
 * out = residual + (bias + sum)) followed by the next layerNormKernel:
 *   h = r + (x + xbias)      (xbias: optional per-column bias of the
 *                             sublayer output, may be NULL)
 *   y = LayerNorm(h) as in gbx_layernorm
 * h_out may be NULL (h not stored) and may alias r or x; y may alias x or r;
 * h_out and y must differ.  Each row is read once and written once.
 */
int gbx_residual_layernorm(const float* x, const float* r, const float* xbias, float* h_out,
                           float* y, const float* gamma, const float* beta, int64_t rows, int d,
                           float eps, gbx_stream_t stream);

/*
 * Final LayerNorm of each sequence's last row, replacing the last-row copy
 * and layerNormKernel launch of TransformerModel::computeLogits
 * (transformer.cu:883-896) together with the residual epilogue of the last
 * ffnDownKernel (:292), for n_seq sequences of seq rows in one launch:
 *   t = b*seq + seq - 1
 *   y[b*d + i] = LayerNorm(r[t*d + .] + x[t*d + .])[i]    (b < n_seq)
 * with gbx_layernorm's arithmetic (the add is one fp32 add, as
 * gbx_residual_layernorm's).  x may be NULL: y = LayerNorm of r's last rows.
 * x, r: [n_seq*seq, d]; y: [n_seq, d], overlapping neither input when
 * seq > 1 (GBX_EINVAL).  No row other than each sequence's last is read.
 */
int gbx_final_layernorm(const float* x, const float* r, float* y, const float* gamma, const float* beta,
                        int64_t n_seq, int seq, int d, float eps, gbx_stream_t stream);

/*
 * Bias + GELU(tanh), replacing the ffnUpKernel epilogue
 * (transformer.cu:272, 276-277) and geluKernel (:68-75):
 *   u = in + bias[col]        (bias may be NULL: u = in)
 *   out = u * (0.5f * (1.0f + tanhf(0.7978845608f * (u + 0.044715f*u*u*u))))
 * in/out: [rows, F]; out may alias in.
 */
int gbx_bias_gelu(const float* in, float* out, const float* bias, int64_t rows, int F,
                  gbx_stream_t stream);

/*
 * Row softmax over rows of length L, replacing softmaxKernel
 * (transformer.cu:126-166; the reference launches it once per head,
 * :839-842; here all rows of all heads and sequences go in one call):
 *   m = max(-1e30f, row); e = expf(x - m); out = e / sum(e)
 * Entries masked with -1e9f (the reference's causal-mask value,
 * transformer.cu:221) come out as exactly 0.  out may alias in.
 */
int gbx_softmax_rows(const float* in, float* out, int64_t rows, int L, gbx_stream_t stream);

/*
 * Attention-score epilogue fused with the row softmax.  Replaces the
 * epilogue of attentionScoresKernel (transformer.cu:213-232: scores =
 * dot / scale with scale = sqrtf(headDim) (:836), -1e9f where the key comes
 * after the query (:220-221)) followed by softmaxKernel (:126-166):
 *   row r is query position p = r % S of one [S, L] score matrix;
 *   x[c] = c > p + q_off (and causal) ? -1e9f : dot[r, c] / scale
 *   out  = softmax(x) exactly as gbx_softmax_rows
 * `scores` holds the raw dot products q.k; entries past the causal limit
 * are never read (they may hold anything).  q_off shifts the diagonal:
 * 0 for prefill (L == S), L - S when S new queries follow L - S cached keys.
 * rows = matrices * S; probs may alias scores.  scale must be a normal,
 * finite, positive float (GBX_EINVAL otherwise).
 */
int gbx_attn_softmax_rows(const float* scores, float* probs, int64_t rows, int L, int S, int q_off,
                          float scale, int causal, gbx_stream_t stream);

/*
 * gbx_attn_softmax_rows with the probabilities written as the tf32 pair
 * gbx_attn_values reads: probs_hi, probs_lo are exactly gbx_split_tf32 of
 * gbx_attn_softmax_rows' output, in one pass.  No counterpart in the
 * reference: it feeds the attention-output contraction.  With causal and
 * q_off 0, only the columns below round_up(p + 1, 256) of row p (p = row % S)
 * are written: the others are zero, and gbx_attn_values never reads them.
 * probs_hi may alias scores; probs_lo may alias neither.
 */
int gbx_attn_softmax_rows_pair(const float* scores, float* probs_hi, float* probs_lo, int64_t rows, int L, int S,
                               int q_off, float scale, int causal, gbx_stream_t stream);

/*
 * Tied-weight logits, replacing computeLogitsKernel (transformer.cu:296-307,
 * launched at :898-900 on the final-LayerNorm row):
 *   logits[r*vocab + v] = sum_j h[r*d + j] * dec(wte[v*d + j])
 * for `rows` hidden rows (the reference has one), reading the token table in
 * its GGUF dtype (dec() as in gbx_embed; no fp32 copy of the table).  The
 * table crosses HBM once per 8 rows.  fp32 accumulation in a different order
 * from the reference's sequential sum.
 */
int gbx_logits(const float* h, int64_t rows, const void* wte, int wte_dtype, float* logits, int vocab, int d,
               gbx_stream_t stream);

/*
 * Next-token selection over `rows` logits rows of length vocab, replacing the
 * host loop of TransformerModel::generate (transformer.cu:994-1028):
 *   out_best[r]       first index of the row maximum (the reference's strict
 *                     `>` scan from index 0; a NaN in entry 0 gives 0)
 *   out_best_logit[r] that maximum
 *   out_ids[r]        out_best[r] when temperature <= 0.01; otherwise, with
 *                     l = (float)(logit / temperature) (a double division),
 *                     p = expf(l - max l) / (fp32 sum), the first j with
 *                     uniforms[r] <= sum_{i<=j} p_i accumulated in double,
 *                     or 0 when none qualifies
 * uniforms: device doubles in [0, 1), one per row: the caller's draws (the
 * reference draws uniform_real_distribution<double>(0, 1) from an mt19937);
 * may be NULL when temperature <= 0.01.  out_best and out_best_logit may be
 * NULL.  All outputs are device arrays of `rows` entries.  The fp32 sum
 * runs in a different order from the reference's, so a draw within ~1e-7
 * of a cumulative boundary may select the neighbouring token.
 */
int gbx_select_tokens(const float* logits, int64_t rows, int vocab, double temperature, const double* uniforms,
                      int32_t* out_ids, int32_t* out_best, float* out_best_logit, gbx_stream_t stream);

/* ------------------------------------------------------------------------
 * The contractions either side of the path, on the tcgen05 tensor cores.
 *
 * An fp32 operand enters as a tf32 pair: hi = x rounded to tf32 (10
 * mantissa bits) and lo = (x - hi) rounded to tf32, so hi + lo carries
 * 21 of x's 24 significant bits.  gbx_linear forms
 *   x.w = hi_x.hi_w + hi_x.lo_w + lo_x.hi_w
 * with f32 accumulation (the lo_x.lo_w term, below 2^-22 of |x w|, is
 * dropped): each product is within ~2^-21 of fp32's, the sums are fp32.
 * ------------------------------------------------------------------------ */

/* Bit set in *err_flag by gbx_linear when a wait of its pipeline ran past
 * one second (the output is then incomplete; the kernel returns without
 * faulting). */
enum { GBX_LINEAR_TIMEOUT = 4 };
enum { GBX_ACT_NONE = 0, GBX_ACT_GELU = 1 };

/* hi[i] = tf32(x[i]); lo[i] = tf32(x[i] - hi[i]) for n elements (0 when hi
 * is not finite).  No counterpart in the reference: it prepares operands
 * for gbx_linear (weights once at load, activations per step).  hi may
 * alias x. */
int gbx_split_tf32(const float* x, float* hi, float* lo, int64_t n, gbx_stream_t stream);

/*
 * y[m, n] = act(sum_k x[m, k] w[n, k] + bias[n]) + resid[m, n]
 * for m < M, n < N, k < K: x [M, K] and w [N, K] row-major (the
 * reference's weight layout, w[i * K + j]), given as tf32 pairs
 * (x_hi, x_lo) and (w_hi, w_lo).  Replaces the GEMVs of computeQKVKernel
 * (transformer.cu:187-210, bias only), projectionKernel (:251-264) and
 * ffnDownKernel (:281-294) (bias + residual), and ffnUpKernel (:266-279)
 * (bias + GELU, act = GBX_ACT_GELU), in one launch per call.
 *   x_lo / w_lo  may be NULL when that operand is exact in tf32 (weights
 *                decoded from f16 or bf16 are): one product term less
 *   bias, resid  may be NULL; resid may alias y (read, then written, by
 *                the same thread)
 *   y_lo         NULL: y receives the fp32 result.  Otherwise y and y_lo
 *                receive its tf32 pair (gbx_split_tf32 of it), ready to be
 *                the x operand of the next gbx_linear
 *   err_flag     device int32 (may be NULL): GBX_LINEAR_TIMEOUT
 * The tensor-core path needs K a multiple of 4 and x_hi, x_lo, w_hi, w_lo
 * 16-byte aligned (the TMA row and base rules); other shapes run a general
 * CUDA-core kernel with the same three product terms.  M < 2^31.  y must
 * not overlap x or w.
 */
int gbx_linear(const float* x_hi, const float* x_lo, const float* w_hi, const float* w_lo, const float* bias,
               const float* resid, float* y, float* y_lo, int64_t M, int N, int K, int act, int* err_flag,
               gbx_stream_t stream);

/*
 * Tile configuration of the tensor-core contractions (gbx_linear, its split-K
 * forms and the attention products), process-wide; no counterpart in the
 * reference.  k_block: 16 (default; 64-byte swizzled rows) or 32 (128-byte
 * rows).  pair_mode: -1 (default) CTA pairs (cta_group::2, an M 256 tile on
 * two SMs) for M >= 1024, 0 never, 1 for every shape.  Every form computes
 * the same three product terms with fp32 accumulation (results within the
 * bound stated below, not necessarily bit-identical); it exists so that tests
 * can run every tile form on any shape, and for tuning.  The previous values
 * go to prev_* (may be NULL).  Not to be changed while another host thread
 * launches contractions.
 */
int gbx_linear_set_tiles(int k_block, int pair_mode, int* prev_k_block, int* prev_pair_mode);

/*
 * gbx_linear with K cut into ksplit slices of K / ksplit (1 <= ksplit <= 16),
 * for contractions with too few output tiles to fill the GPU (one sequence
 * of 1024 tokens against a d x d projection: 16 CTA-pair tiles for 74 SM
 * pairs).  No counterpart in the reference: the same result as gbx_linear
 * (same epilogue, same operands) from ksplit times the tiles.  Each slice's
 * fp32 partial sums go to `workspace` (device, at least ksplit * M * N
 * floats, overlapping no operand), then one pass adds the slices in order
 * (s = 0, 1, ...: deterministic) and applies bias, act, resid and the
 * optional tf32 split.  Rounding differs from gbx_linear's by ksplit - 1 fp32
 * additions per output.  When ksplit is 1, or K / ksplit is not a multiple
 * of 4, or an operand is off 16-byte alignment, it runs gbx_linear instead
 * and leaves the workspace untouched.
 */
int gbx_linear_splitk(const float* x_hi, const float* x_lo, const float* w_hi, const float* w_lo, const float* bias,
                      const float* resid, float* y, float* y_lo, int64_t M, int N, int K, int act, int ksplit,
                      float* workspace, int64_t workspace_floats, int* err_flag, gbx_stream_t stream);

/*
 * gbx_linear_splitk for callers that cannot allocate device memory: a binding
 * or plugin host that owns every device buffer and gives the library only
 * the inputs and outputs, or a latency-critical caller for which
 * cudaMalloc's implicit synchronization is not acceptable.  No counterpart
 * in the reference.  The partial sums go to a scratch array inside the
 * library (16 MiB, held on every GPU that loads the library until the
 * process exits), so ksplit * M * N may be at most 4,194,304 (GBX_ERANGE
 * otherwise; gbx_linear_splitk takes any size).  Nothing is allocated,
 * freed or cleared per call: every call writes each scratch element it later
 * reads.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current) and caches it; make that
 * first call before any stream capture.  All calls share the one array:
 * calls that can overlap on the GPU (other streams, other host threads)
 * race on it and must be serialised by the caller.  Results are those of
 * gbx_linear_splitk; ksplit 1 or an unsliceable shape runs gbx_linear, which
 * needs no scratch, so the size limit applies only to calls that split K.
 * The cached address assumes the device's primary context (the one the CUDA
 * runtime uses) and does not survive cudaDeviceReset.
 */
int gbx_linear_splitk_noalloc(const float* x_hi, const float* x_lo, const float* w_hi, const float* w_lo,
                              const float* bias, const float* resid, float* y, float* y_lo, int64_t M, int N, int K,
                              int act, int ksplit, int* err_flag, gbx_stream_t stream);

/* ------------------------------------------------------------------------
 * The per-head attention products on the tcgen05 tensor cores, for B
 * sequences of S tokens, H heads of width hd, every operand a tf32 pair (the
 * *_lo planes may be NULL: one product term less).  Head z = b*H + h.
 * ------------------------------------------------------------------------ */

/*
 * Raw attention dot products, replacing the sums of attentionScoresKernel
 * (transformer.cu:213-232) for every head of every sequence in one launch:
 *   dots[(z*S + p)*S + s] = sum_i q[(b*S + p)*ld + h*hd + i] * k[(b*S + s)*ld + h*hd + i]
 * q and k are row-major with row stride ld (>= H*hd; the Q and K column
 * blocks of the [tokens, 3*d] QKV output: ld = 3*d).  causal != 0: only
 * s <= p is required, and tiles of the [S, S] matrix lying wholly past the
 * diagonal are neither computed nor written (gbx_attn_softmax_rows reads
 * no entry past the diagonal).  The scale and the -1e9f mask are applied by
 * the softmax.  dots must not overlap the operands.  err_flag: as
 * gbx_linear (GBX_LINEAR_TIMEOUT).
 */
int gbx_attn_scores(const float* q_hi, const float* q_lo, const float* k_hi, const float* k_lo, int64_t ld,
                    float* dots, int B, int S, int H, int hd, int causal, int* err_flag, gbx_stream_t stream);

/*
 * V of each head transposed for gbx_attn_values (no counterpart in the
 * reference; one plane, call it for hi and for lo):
 *   vt[((b*H + h)*hd + i)*S + s] = v[(b*S + s)*ld + h*hd + i]
 */
int gbx_transpose_heads(const float* v, int64_t ld, float* vt, int B, int S, int H, int hd, gbx_stream_t stream);

/*
 * Attention output, replacing attentionOutputKernel (transformer.cu:234-249)
 * for every head of every sequence in one launch:
 *   out[(b*S + p)*ld_out + h*hd + i] = sum_s P[(z*S + p)*S + s] * vt[(z*hd + i)*S + s]
 * P: the probabilities [B*H*S, S] as a tf32 pair (gbx_attn_softmax_rows_pair);
 * vt: gbx_transpose_heads of V.  causal != 0: P is zero past the diagonal
 * (as the causal softmax writes it) and the sum stops there.  out_lo NULL:
 * out receives the fp32 result; otherwise out and out_lo its tf32 pair,
 * the x operand of the output projection.  out must not overlap the
 * operands.  err_flag: as gbx_linear.
 */
int gbx_attn_values(const float* p_hi, const float* p_lo, const float* vt_hi, const float* vt_lo, float* out,
                    float* out_lo, int64_t ld_out, int B, int S, int H, int hd, int causal, int* err_flag,
                    gbx_stream_t stream);

/*
 * Self-attention of every head of every sequence in one launch, fused on the
 * tensor cores, replacing attentionScoresKernel, the per-head softmaxKernel
 * launches and attentionOutputKernel (transformer.cu:213-249, launched at
 * :834-846), with no [S, S] score or probability matrix in memory:
 *   out[(b*S + p)*ld_out + h*64 + i] = sum_s w_ps v[b, s, h*64 + i],
 *   w_p = softmax over s of q_p . k_s / scale (s <= p when causal)
 * q, k: tf32 pairs with row stride ld, as gbx_attn_scores takes them (the Q
 * and K column blocks of the QKV output); v_hi, v_lo: V's two planes with the
 * same row stride (the QKV output's V column block, read as it lies: no
 * transpose).  out_lo NULL: out receives the fp32 result; otherwise
 * out and out_lo its tf32 pair (the projection's x operand).  The softmax is
 * the online form (running maximum and sum per row, the running output
 * rescaled when the maximum grows), so the weights differ from the
 * reference's single-pass softmax only in rounding; keys past the diagonal
 * weigh exactly 0.  hd must be 64 (every GPT-2 size); ld and ld_out
 * multiples of 4; operands 16-byte aligned; any S >= 1.  Other shapes return
 * GBX_EINVAL: use gbx_attn_scores, gbx_attn_softmax_rows_pair and
 * gbx_attn_values.  out and out_lo must overlap neither each other nor any
 * of q, k, v (GBX_EINVAL): no in-place attention over the QKV block.
 * err_flag: as gbx_linear (GBX_LINEAR_TIMEOUT).
 */
int gbx_attn_fused(const float* q_hi, const float* q_lo, const float* k_hi, const float* k_lo, int64_t ld,
                   const float* v_hi, const float* v_lo, float* out, float* out_lo, int64_t ld_out, int B, int S,
                   int H, int hd, float scale, int causal, int* err_flag, gbx_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GBX_H */
