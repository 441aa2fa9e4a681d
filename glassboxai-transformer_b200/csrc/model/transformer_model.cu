// transformer_model.cu -- TransformerModel::forward (the reference's
// transformer.cu:913-927 and the launch sites it calls, :805-911) on the
// sm_100a hot-path kernels.
//
// Per forward of B sequences of S tokens (N = B*S rows, hidden d, H heads of
// hd = d/H, feed-forward F, vocab V):
//
//   gbx_embed_layernorm                    h = wte[ids] + wpe[pos]          (:805-815)
//                                          and layer 0's ln = LN1(h) as a tf32 pair,
//                                          one pass                        (:827-828)
//   for each layer l:
//     gbx_layernorm_pair (l > 0)           ln = LN1(h), as a tf32 pair     (:827-828)
//     gbx_linear                           qkv = ln . Wqkv^T + b_qkv, as a tf32 pair (:830-832)
//     head width 64 (every GPT-2 size):
//       gbx_attn_fused                     attn = softmax(mask(Q K^T / sqrt(hd))) V, every
//                                          head of every sequence in one launch, Q, K and V
//                                          read from the QKV rows as they lie, no [S, S]
//                                          matrix in memory (:834-846)
//     other widths, per group of sequences, every head in one launch each:
//       gbx_attn_scores                    raw[b][h] = Q_bh . K_bh^T, causal tiles only
//                                                                          (:834-837, without
//                                                                          the scale and mask)
//       gbx_attn_softmax_rows_pair         P = softmax(mask(raw / sqrt(hd))), as a tf32 pair
//                                                                          (:220-229, :839-842)
//       gbx_transpose_heads (hi, lo)       Vt[b][h] = V_bh^T
//       gbx_attn_values                    attn_bh = P_bh . V_bh, as a tf32 pair (:844-846)
//     gbx_linear                           h += attn . Wproj^T + b_proj    (:848-852, the
//                                                                          residual in the epilogue)
//     gbx_layernorm_pair                   ln = LN2(h), as a tf32 pair     (:866-868)
//     gbx_linear                           up = GELU(ln . Wup^T + b_up), as a tf32 pair
//                                                                          (:870-872)
//     gbx_linear                           h += up . Wdown^T + b_down      (:874-878)
//   gbx_final_layernorm                    last = LN_f(h) of each sequence's last row
//                                                                          (:883-896)
//   gbx_logits                             logits = last . wte^T           (:898-900)
//   (nextToken) gbx_select_tokens          argmax / temperature sampling   (:994-1028)
//
// Every contraction, the weight products (gbx_linear) and the per-head
// attention products (gbx_attn_scores, gbx_attn_values), runs on the tcgen05
// tensor cores with every operand as a tf32 pair: each product within
// ~2^-21 of fp32's, fp32 sums, so they differ from the reference's
// sequential GEMV sums by rounding of the same order as a change of
// summation order.  Weights are split once at load; a weight read from an
// f16 or bf16 tensor is exact in tf32 and needs no low part.  Activation
// buffers grow to the largest call (like allocateBuffers, :770-787) and are
// reused; the attention scores of at most kScoreGroupFloats floats are held
// at a time (sequences are taken in groups that fit).
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>

#include <cuda_runtime.h>

#include "gbx_model.hpp"

namespace gbx {

namespace {

// attention scores held at once: 2^28 floats (1 GiB), and as much again for
// the low half of the probabilities
constexpr int64_t kScoreGroupFloats = (int64_t)1 << 28;

// K slices for a contraction of M rows x N outputs over K: a contraction with
// fewer output tiles than half the GPU's tile slots (one 1024-token sequence
// against a d x d matrix) is cut into slices, ksplit doubling while the
// tiles still fit in the slots and each slice keeps at least 256 of K.
int splitk_of(int64_t M, int N, int K, int sm_count)
{
    const bool pair_tiles = M >= 1024;   // gbx_linear's CTA-pair threshold
    const int64_t slots = pair_tiles ? sm_count / 2 : sm_count;
    const int64_t tiles = ((M + (pair_tiles ? 255 : 127)) / (pair_tiles ? 256 : 128)) * ((N + 255) / 256);
    int ks = 1;
    while (ks < 8 && tiles * ks * 2 <= slots && K % (8 * ks) == 0 && K / (2 * ks) >= 256) ks *= 2;
    return ks;
}

struct DevBuf {
    float* p = nullptr;
    size_t n = 0;
    bool ensure(size_t want)
    {
        if (want <= n) return true;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        if (cudaMalloc(&p, want * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        n = want;
        return true;
    }
    void release()
    {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
};

}  // namespace

struct TransformerModel::Impl {
    cudaStream_t stream = nullptr;
    int device = -1;
    // activations (ln, qkv, scores (as probabilities), vt, attn and up hold
    // the hi half of a tf32 pair, *_lo the low half)
    DevBuf h, ln, ln_lo, qkv, qkv_lo, scores, probs_lo, vt, vt_lo, attn, attn_lo, up, up_lo, last_y, logits;
    DevBuf splitk_ws;      // partial sums of the K-split contractions
    int score_group = 1;   // sequences per attention launch (unfused path)
    bool fused = false;    // attention in one gbx_attn_fused launch (head width 64)
    bool want_fused = true;   // setFusedAttention
    int sm_count = 148;
    int32_t* ids = nullptr;
    size_t ids_n = 0;
    int32_t* err = nullptr;
    // next-token selection: [selected, best], best logit, the uniform draw
    int32_t* sel_ids = nullptr;
    float* sel_logit = nullptr;
    double* sel_u = nullptr;
    // weights (device pointers owned by the loader)
    struct Layer {
        const float *ln1_g, *ln1_b, *qkv_w, *qkv_b, *proj_w, *proj_b, *ln2_g, *ln2_b, *up_w, *up_b, *down_w,
            *down_b;
    };
    std::vector<Layer> layers;
    // tf32 pairs of the four weight matrices per layer: hi is the loader's
    // fp32 tensor itself when that is exact in tf32 (decoded from f16 or
    // bf16; lo NULL), else a split copy owned here
    struct Pair {
        const float* hi = nullptr;
        const float* lo = nullptr;
    };
    struct LayerW {
        Pair qkv, proj, up, down;
    };
    std::vector<LayerW> wpairs;
    std::vector<float*> owned;
    const float *lnf_g = nullptr, *lnf_b = nullptr;
    const void *wte = nullptr, *wpe = nullptr;
    int wte_dt = 0, wpe_dt = 0;

    ~Impl()
    {
        for (DevBuf* b : {&h, &ln, &ln_lo, &qkv, &qkv_lo, &scores, &probs_lo, &vt, &vt_lo, &attn, &attn_lo, &up, &up_lo,
                          &last_y, &logits, &splitk_ws})
            b->release();
        for (float* p : owned) cudaFree(p);
        if (ids) cudaFree(ids);
        if (err) cudaFree(err);
        if (sel_ids) cudaFree(sel_ids);
        if (sel_logit) cudaFree(sel_logit);
        if (sel_u) cudaFree(sel_u);
        if (stream) cudaStreamDestroy(stream);
    }
};

TransformerModel::TransformerModel() : impl_(new Impl) {}

TransformerModel::~TransformerModel()
{
    if (impl_ && impl_->device >= 0) cudaSetDevice(impl_->device);
    impl_.reset();
    loader_.freeGPUMemory();
}

bool TransformerModel::fail(const std::string& msg)
{
    err_ = msg;
    return false;
}

bool TransformerModel::loadModel(const std::string& ggufPath)
{
    if (!loader_.loadFromFile(ggufPath)) return fail(loader_.lastError());
    Impl& m = *impl_;
    if (cudaGetDevice(&m.device) != cudaSuccess) return fail("no CUDA device");
    if (cudaStreamCreateWithFlags(&m.stream, cudaStreamNonBlocking) != cudaSuccess) return fail("stream");
    if (cudaDeviceGetAttribute(&m.sm_count, cudaDevAttrMultiProcessorCount, m.device) != cudaSuccess || m.sm_count < 1)
        return fail("no CUDA device properties");
    if (cudaMalloc(&m.err, sizeof(int32_t)) != cudaSuccess || cudaMalloc(&m.sel_ids, 2 * sizeof(int32_t)) != cudaSuccess ||
        cudaMalloc(&m.sel_logit, sizeof(float)) != cudaSuccess || cudaMalloc(&m.sel_u, sizeof(double)) != cudaSuccess)
        return fail("cudaMalloc");

    embedDim_ = loader_.getEmbedDim();
    numLayers_ = loader_.getNumLayers();
    numHeads_ = loader_.getNumHeads();
    ffnDim_ = loader_.getFFNDim();
    if (embedDim_ <= 0 || numHeads_ <= 0 || embedDim_ % numHeads_ || numLayers_ < 0 || ffnDim_ <= 0)
        return fail("inconsistent model dimensions in the GGUF header");
    headDim_ = embedDim_ / numHeads_;

    int64_t n_wte = 0, n_wpe = 0;
    m.wte = loader_.getTensorGPURaw({"token_embd.weight", "wte.weight"}, &m.wte_dt, &n_wte);
    m.wpe = loader_.getTensorGPURaw({"position_embd.weight", "wpe.weight"}, &m.wpe_dt, &n_wpe);
    if (!m.wte || !m.wpe) return fail("token / position embedding: " + loader_.lastError());
    if (n_wte % embedDim_ || n_wpe % embedDim_) return fail("embedding tables are not [rows, embed_dim]");
    vocab_ = (int)(n_wte / embedDim_);
    nCtx_ = (int)(n_wpe / embedDim_);

    auto get = [&](const std::string& name, int64_t want) -> const float* {
        const GGUFTensor* t = loader_.findTensor({name});
        if (!t) {
            fail("missing tensor " + name);
            return nullptr;
        }
        if (t->numElements != want) {
            fail("tensor " + name + " has " + std::to_string(t->numElements) + " elements, expected " +
                 std::to_string(want));
            return nullptr;
        }
        const float* p = loader_.getTensorGPU({name});
        if (!p) fail(name + ": " + loader_.lastError());
        return p;
    };
    const int64_t d = embedDim_, F = ffnDim_;
    m.layers.resize(numLayers_);
    for (int l = 0; l < numLayers_; ++l) {
        const std::string pre = "blk." + std::to_string(l) + ".";
        Impl::Layer& L = m.layers[l];
        if (!(L.ln1_g = get(pre + "attn_norm.weight", d)) || !(L.ln1_b = get(pre + "attn_norm.bias", d)) ||
            !(L.qkv_w = get(pre + "attn_qkv.weight", 3 * d * d)) || !(L.qkv_b = get(pre + "attn_qkv.bias", 3 * d)) ||
            !(L.proj_w = get(pre + "attn_output.weight", d * d)) ||
            !(L.proj_b = get(pre + "attn_output.bias", d)) || !(L.ln2_g = get(pre + "ffn_norm.weight", d)) ||
            !(L.ln2_b = get(pre + "ffn_norm.bias", d)) || !(L.up_w = get(pre + "ffn_up.weight", F * d)) ||
            !(L.up_b = get(pre + "ffn_up.bias", F)) || !(L.down_w = get(pre + "ffn_down.weight", d * F)) ||
            !(L.down_b = get(pre + "ffn_down.bias", d)))
            return false;
    }
    // tf32 pairs of the weight matrices
    auto pair = [&](const std::string& name, const float* w, int64_t n, Impl::Pair* out) -> bool {
        const GGUFTensor* t = loader_.findTensor({name});
        if (t->dtype == GBX_DT_F16 || t->dtype == GBX_DT_BF16) {
            out->hi = w;   // at most 11 significant bits: exact in tf32
            out->lo = nullptr;
            return true;
        }
        float *hi = nullptr, *lo = nullptr;
        if (cudaMalloc(&hi, n * sizeof(float)) != cudaSuccess) return fail("cudaMalloc of weight pairs failed");
        m.owned.push_back(hi);
        if (cudaMalloc(&lo, n * sizeof(float)) != cudaSuccess) return fail("cudaMalloc of weight pairs failed");
        m.owned.push_back(lo);
        if (gbx_split_tf32(w, hi, lo, n, reinterpret_cast<gbx_stream_t>(m.stream)) != GBX_OK)
            return fail(std::string("weight split: ") + gbx_last_error());
        out->hi = hi;
        out->lo = lo;
        return true;
    };
    m.wpairs.resize(numLayers_);
    for (int l = 0; l < numLayers_; ++l) {
        const std::string pre = "blk." + std::to_string(l) + ".";
        const Impl::Layer& L = m.layers[l];
        Impl::LayerW& W = m.wpairs[l];
        if (!pair(pre + "attn_qkv.weight", L.qkv_w, 3 * d * d, &W.qkv) ||
            !pair(pre + "attn_output.weight", L.proj_w, d * d, &W.proj) ||
            !pair(pre + "ffn_up.weight", L.up_w, F * d, &W.up) || !pair(pre + "ffn_down.weight", L.down_w, d * F, &W.down))
            return false;
    }
    if (cudaStreamSynchronize(m.stream) != cudaSuccess) return fail("weight split failed");

    const GGUFTensor* g = loader_.findTensor({"output_norm.weight", "ln_f.weight"});
    const GGUFTensor* b = loader_.findTensor({"output_norm.bias", "ln_f.bias"});
    if (!g || !b) return fail("missing output_norm / ln_f");
    if (!(m.lnf_g = get(g->name, d)) || !(m.lnf_b = get(b->name, d))) return false;
    return true;
}

bool TransformerModel::ensureBuffers(int64_t tokens, int seq)
{
    Impl& m = *impl_;
    const int64_t d = embedDim_, F = ffnDim_, B = tokens / seq;
    const int64_t per_seq = (int64_t)numHeads_ * seq * seq;
    int64_t G = kScoreGroupFloats / per_seq;
    G = G < 1 ? 1 : (G > B ? B : G);
    m.score_group = (int)G;
    // the fused attention needs no score buffers
    m.fused = m.want_fused && headDim_ == 64 && d % 4 == 0;
    const int64_t score_floats = m.fused ? 1 : G * per_seq;
    const int64_t vt_floats = m.fused ? 1 : G * seq * d;
    // the largest split-K workspace of the four contractions
    size_t ws = 1;
    const int64_t shapes[4][2] = {{3 * d, d}, {d, d}, {F, d}, {d, F}};
    for (const auto& nk : shapes) {
        const int ks = splitk_of(tokens, (int)nk[0], (int)nk[1], m.sm_count);
        if (ks > 1 && (size_t)(ks * tokens * nk[0]) > ws) ws = (size_t)(ks * tokens * nk[0]);
    }
    const bool ok = m.h.ensure(tokens * d) && m.ln.ensure(tokens * d) && m.ln_lo.ensure(tokens * d) &&
                    m.qkv.ensure(tokens * 3 * d) && m.qkv_lo.ensure(tokens * 3 * d) &&
                    m.scores.ensure((size_t)score_floats) && m.probs_lo.ensure((size_t)score_floats) &&
                    m.vt.ensure((size_t)vt_floats) && m.vt_lo.ensure((size_t)vt_floats) &&
                    m.attn.ensure(tokens * d) && m.attn_lo.ensure(tokens * d) && m.up.ensure(tokens * F) &&
                    m.up_lo.ensure(tokens * F) && m.splitk_ws.ensure(ws) &&
                    m.last_y.ensure(B * d) &&
                    m.logits.ensure((size_t)B * vocab_);
    if (!ok) return fail("cudaMalloc of activation buffers failed");
    if ((size_t)tokens > m.ids_n) {
        if (m.ids) cudaFree(m.ids);
        m.ids = nullptr;
        m.ids_n = 0;
        if (cudaMalloc(&m.ids, tokens * sizeof(int32_t)) != cudaSuccess) return fail("cudaMalloc of ids failed");
        m.ids_n = (size_t)tokens;
    }
    return true;
}

std::vector<float> TransformerModel::forward(const std::vector<int>& tokenIDs) { return forwardBatch(tokenIDs, 1); }

std::vector<float> TransformerModel::forwardBatch(const std::vector<int>& tokenIDs, int batch)
{
    Impl& m = *impl_;
    int cur = -1;
    cudaGetDevice(&cur);
    std::vector<float> out;
    if (runForward(tokenIDs, batch)) {
        out.resize((size_t)batch * vocab_);
        if (cudaMemcpyAsync(out.data(), m.logits.p, out.size() * sizeof(float), cudaMemcpyDeviceToHost, m.stream) !=
                cudaSuccess ||
            cudaStreamSynchronize(m.stream) != cudaSuccess) {
            fail("device-to-host copy of the logits failed");
            out.clear();
        }
    }
    if (cur >= 0 && cur != m.device) cudaSetDevice(cur);
    return out;
}

int TransformerModel::nextToken(const std::vector<int>& tokenIDs, double temperature, std::mt19937& rng, int* bestID,
                                float* bestLogit)
{
    // the reference draws only when it samples (transformer.cu:1017-1018),
    // after its forward; the draw does not depend on the logits
    double u = 0.0;
    if (temperature > 0.01) u = std::uniform_real_distribution<double>(0.0, 1.0)(rng);
    return nextTokenWithDraw(tokenIDs, temperature, u, bestID, bestLogit);
}

int TransformerModel::nextTokenWithDraw(const std::vector<int>& tokenIDs, double temperature, double u, int* bestID,
                                        float* bestLogit)
{
    Impl& m = *impl_;
    int cur = -1;
    cudaGetDevice(&cur);
    int selected = -1;
    if (runForward(tokenIDs, 1)) {
        int32_t host[2] = {0, 0};
        float blog = 0.0f;
        int rc = GBX_OK;
        if (cudaMemcpyAsync(m.sel_u, &u, sizeof(double), cudaMemcpyHostToDevice, m.stream) != cudaSuccess)
            rc = GBX_ECUDA;
        if (rc == GBX_OK)
            rc = gbx_select_tokens(m.logits.p, 1, vocab_, temperature, m.sel_u, m.sel_ids, m.sel_ids + 1, m.sel_logit,
                                   reinterpret_cast<gbx_stream_t>(m.stream));
        if (rc == GBX_OK &&
            (cudaMemcpyAsync(host, m.sel_ids, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost, m.stream) != cudaSuccess ||
             cudaMemcpyAsync(&blog, m.sel_logit, sizeof(float), cudaMemcpyDeviceToHost, m.stream) != cudaSuccess ||
             cudaStreamSynchronize(m.stream) != cudaSuccess))
            rc = GBX_ECUDA;
        if (rc == GBX_OK) {
            selected = host[0];
            if (bestID) *bestID = host[1];
            if (bestLogit) *bestLogit = blog;
        } else {
            fail(std::string("token selection failed: ") + gbx_last_error());
        }
    }
    if (cur >= 0 && cur != m.device) cudaSetDevice(cur);
    return selected;
}

void TransformerModel::setFusedAttention(bool on) { impl_->want_fused = on; }

bool TransformerModel::fusedAttention() const { return impl_->want_fused; }

std::vector<float> TransformerModel::forwardHidden(const std::vector<int>& tokenIDs, int batch)
{
    if (!loader_.isLoaded() || batch <= 0 || tokenIDs.empty()) {
        fail("forwardHidden: model not loaded or empty input");
        return {};
    }
    std::vector<float> hidden((size_t)(numLayers_ + 1) * tokenIDs.size() * embedDim_);
    int cur = -1;
    cudaGetDevice(&cur);
    const bool ok = runForward(tokenIDs, batch, hidden.data());
    if (cur >= 0 && cur != impl_->device) cudaSetDevice(cur);
    if (!ok) return {};
    return hidden;
}

bool TransformerModel::runForward(const std::vector<int>& tokenIDs, int batch, float* hidden_host)
{
    Impl& m = *impl_;
    err_.clear();
    if (!loader_.isLoaded() || !m.stream) return fail("model not loaded");
    if (batch <= 0 || tokenIDs.empty() || tokenIDs.size() % (size_t)batch)
        return fail("forward: need batch > 0 sequences of equal, non-zero length");
    const int64_t N = (int64_t)tokenIDs.size();
    const int S = (int)(N / batch);
    if (S > nCtx_)
        return fail("forward: " + std::to_string(S) + " tokens exceed the " + std::to_string(nCtx_) +
                    " position rows");
    for (int id : tokenIDs)
        if (id < 0 || id >= vocab_) return fail("forward: token id " + std::to_string(id) + " outside the token table");
    cudaSetDevice(m.device);
    if (!ensureBuffers(N, S)) return false;

    const int d = embedDim_, H = numHeads_, hd = headDim_, F = ffnDim_, V = vocab_;
    cudaStream_t st = m.stream;
    gbx_stream_t gs = reinterpret_cast<gbx_stream_t>(st);
    int rc = GBX_OK;
    auto check = [&](int r) {
        if (rc == GBX_OK && r != GBX_OK) rc = r;
    };
    // y[M, Nout] = act(x . W^T + bias) + resid on the tensor cores, x and W as
    // tf32 pairs; K-split (splitk_of) when the output tiles are few
    auto linear = [&](const float* xh, const float* xl, const Impl::Pair& W, const float* bias, const float* resid,
                      float* y, float* y_lo, int64_t M, int Nout, int K, int act) {
        const int ks = splitk_of(M, Nout, K, m.sm_count);
        if (ks > 1) {
            check(gbx_linear_splitk(xh, xl, W.hi, W.lo, bias, resid, y, y_lo, M, Nout, K, act, ks, m.splitk_ws.p,
                                    (int64_t)m.splitk_ws.n, m.err, gs));
        } else {
            check(gbx_linear(xh, xl, W.hi, W.lo, bias, resid, y, y_lo, M, Nout, K, act, m.err, gs));
        }
    };

    if (cudaMemcpyAsync(m.ids, tokenIDs.data(), N * sizeof(int32_t), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemsetAsync(m.err, 0, sizeof(int32_t), st) != cudaSuccess)
        return fail("host-to-device copy of token ids failed");
    // the embedding and layer 0's attention LayerNorm in one pass (h written once, not re-read)
    check(gbx_embed_layernorm(m.ids, m.wte, m.wte_dt, m.wpe, m.wpe_dt, nullptr, m.h.p, m.ln.p, m.ln_lo.p,
                              numLayers_ > 0 ? m.layers[0].ln1_g : nullptr, numLayers_ > 0 ? m.layers[0].ln1_b : nullptr,
                              N, S, 0, d, V, nCtx_, 1e-5f, m.err, gs));
    // forwardHidden: the residual stream after the embedding and after each layer
    auto keep_hidden = [&](int slot) {
        if (hidden_host && rc == GBX_OK &&
            cudaMemcpyAsync(hidden_host + (size_t)slot * N * d, m.h.p, (size_t)N * d * sizeof(float),
                            cudaMemcpyDeviceToHost, st) != cudaSuccess)
            check(GBX_ECUDA);
    };
    keep_hidden(0);

    const float scale = sqrtf((float)hd);   // transformer.cu:836
    for (int l = 0; l < numLayers_ && rc == GBX_OK; ++l) {
        const Impl::Layer& L = m.layers[l];
        const Impl::LayerW& W = m.wpairs[l];
        if (l > 0) check(gbx_layernorm_pair(m.h.p, m.ln.p, m.ln_lo.p, L.ln1_g, L.ln1_b, N, d, 1e-5f, gs));
        linear(m.ln.p, m.ln_lo.p, W.qkv, L.qkv_b, nullptr, m.qkv.p, m.qkv_lo.p, N, 3 * d, d, GBX_ACT_NONE);
        if (m.fused) {
            // attn = softmax(mask(Q K^T / sqrt(hd))) V for every head of every
            // sequence in one launch, as a tf32 pair
            check(gbx_attn_fused(m.qkv.p, m.qkv_lo.p, m.qkv.p + d, m.qkv_lo.p + d, 3 * d, m.qkv.p + 2 * d,
                                 m.qkv_lo.p + 2 * d, m.attn.p, m.attn_lo.p, d, batch, S, H, hd, scale, 1, m.err, gs));
        }
        for (int b0 = 0; !m.fused && b0 < batch; b0 += m.score_group) {
            const int g = batch - b0 < m.score_group ? batch - b0 : m.score_group;
            const float* qh = m.qkv.p + (int64_t)b0 * S * 3 * d;
            const float* ql = m.qkv_lo.p + (int64_t)b0 * S * 3 * d;
            // raw[b][h][p][s] = sum_i Q[b, p, h*hd+i] K[b, s, h*hd+i] (s <= p)
            check(gbx_attn_scores(qh, ql, qh + d, ql + d, 3 * d, m.scores.p, g, S, H, hd, 1, m.err, gs));
            check(gbx_attn_softmax_rows_pair(m.scores.p, m.scores.p, m.probs_lo.p, (int64_t)g * H * S, S, S, 0, scale,
                                             1, gs));
            check(gbx_transpose_heads(qh + 2 * d, 3 * d, m.vt.p, g, S, H, hd, gs));
            check(gbx_transpose_heads(ql + 2 * d, 3 * d, m.vt_lo.p, g, S, H, hd, gs));
            // attn[b, p, h*hd+i] = sum_s P[b][h][p][s] V[b, s, h*hd+i]
            check(gbx_attn_values(m.scores.p, m.probs_lo.p, m.vt.p, m.vt_lo.p, m.attn.p + (int64_t)b0 * S * d,
                                  m.attn_lo.p + (int64_t)b0 * S * d, d, g, S, H, hd, 1, m.err, gs));
        }
        linear(m.attn.p, m.attn_lo.p, W.proj, L.proj_b, m.h.p, m.h.p, nullptr, N, d, d, GBX_ACT_NONE);
        check(gbx_layernorm_pair(m.h.p, m.ln.p, m.ln_lo.p, L.ln2_g, L.ln2_b, N, d, 1e-5f, gs));
        linear(m.ln.p, m.ln_lo.p, W.up, L.up_b, nullptr, m.up.p, m.up_lo.p, N, F, d, GBX_ACT_GELU);
        linear(m.up.p, m.up_lo.p, W.down, L.down_b, m.h.p, m.h.p, nullptr, N, d, F, GBX_ACT_NONE);
        keep_hidden(l + 1);
    }
    if (rc == GBX_OK) {
        // ln_f of each sequence's last row of h (transformer.cu:883-896)
        check(gbx_final_layernorm(nullptr, m.h.p, m.last_y.p, m.lnf_g, m.lnf_b, batch, S, d, 1e-5f, gs));
        check(gbx_logits(m.last_y.p, batch, m.wte, m.wte_dt, m.logits.p, V, d, gs));
    }
    int32_t err_host = 0;
    if (rc == GBX_OK && cudaMemcpyAsync(&err_host, m.err, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess)
        rc = GBX_ECUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess && rc == GBX_OK) rc = GBX_ECUDA;
    if (rc != GBX_OK) return fail(std::string(gbx_status_string(rc)) + ": " + gbx_last_error());
    // GBX_LINEAR_TIMEOUT and GBX_EMBED_TIMEOUT are the same bit of the shared flag
    if (err_host & GBX_LINEAR_TIMEOUT)
        return fail("a device wait timed out (a tensor-core contraction or the staged embedding): the forward's "
                    "outputs are incomplete");
    if (err_host) return fail("embedding reported out-of-range ids or positions");
    return true;
}

}  // namespace gbx
