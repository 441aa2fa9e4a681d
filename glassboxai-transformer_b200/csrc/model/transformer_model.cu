// transformer_model.cu -- TransformerModel::forward (the reference's
// transformer.cu:913-927 and the launch sites it calls, :805-911) on the
// sm_100a hot-path kernels.
//
// Per forward of B sequences of S tokens (N = B*S rows, hidden d, H heads of
// hd = d/H, feed-forward F, vocab V):
//
//   gbx_embed                              h = wte[ids] + wpe[pos]          (:805-815)
//   for each layer l:
//     gbx_layernorm / gbx_residual_layernorm
//                                          ln = LN1(h)   (l = 0)
//                                          h += down + b_down(l-1); ln = LN1(h)   (l > 0: the
//                                          residual of :874-878 fused with the LN of :868)
//     cuBLAS                               qkv = ln . Wqkv^T + b_qkv       (:830-832)
//     cuBLAS (per sequence, batched over heads)
//                                          raw[h] = Q_h . K_h^T            (:834-837, without
//                                                                          the scale and mask)
//     gbx_attn_softmax_rows                P = softmax(mask(raw / sqrt(hd)))  (:220-229, :839-842)
//     cuBLAS (per sequence, batched over heads)
//                                          attn_h = P_h . V_h              (:844-846)
//     cuBLAS                               proj = attn . Wproj^T           (:848-850, bias below)
//     gbx_residual_layernorm               h += proj + b_proj; ln = LN2(h) (:850-852 fused with :868)
//     cuBLAS                               up = ln . Wup^T                 (:870-872, bias below)
//     gbx_bias_gelu                        up = GELU(up + b_up)            (:272, 276-277)
//     cuBLAS                               down = up . Wdown^T             (:874-876, bias and
//                                                                          residual deferred)
//   gbx_residual_layernorm on each sequence's last row
//                                          last = LN_f(h + down + b_down)  (:890-896)
//   gbx_logits                             logits = last . wte^T           (:898-900)
//   (nextToken) gbx_select_tokens          argmax / temperature sampling   (:994-1028)
//
// The GEMMs are fp32 cuBLAS (CUBLAS_COMPUTE_32F, no TF32), the reference's
// precision; their outputs differ from the reference's sequential GEMV sums
// in summation order only.  Activation buffers grow to the largest call
// (like allocateBuffers, :770-787) and are reused.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>

#include <cublas_v2.h>
#include <cuda_runtime.h>

#include "gbx_model.hpp"

namespace gbx {

namespace {

// dst[r * ld + c] = src[c] for r < rows, c < cols (QKV bias seeds the GEMM
// accumulator, as the reference seeds its sum with the bias, :195-197).
__global__ void broadcast_rows_kernel(float* __restrict__ dst, int64_t ld, const float* __restrict__ src,
                                      int64_t rows, int cols)
{
    const int64_t total = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols;
        const int c = (int)(i - r * cols);
        dst[r * ld + c] = src[c];
    }
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
    cublasHandle_t blas = nullptr;
    cudaStream_t stream = nullptr;
    int device = -1;
    // activations
    DevBuf h, ln, qkv, scores, attn, proj, up, down, last_h, last_x, last_y, logits;
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
    const float *lnf_g = nullptr, *lnf_b = nullptr;
    const void *wte = nullptr, *wpe = nullptr;
    int wte_dt = 0, wpe_dt = 0;

    ~Impl()
    {
        for (DevBuf* b : {&h, &ln, &qkv, &scores, &attn, &proj, &up, &down, &last_h, &last_x, &last_y, &logits})
            b->release();
        if (ids) cudaFree(ids);
        if (err) cudaFree(err);
        if (sel_ids) cudaFree(sel_ids);
        if (sel_logit) cudaFree(sel_logit);
        if (sel_u) cudaFree(sel_u);
        if (blas) cublasDestroy(blas);
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
    if (cublasCreate(&m.blas) != CUBLAS_STATUS_SUCCESS) return fail("cublasCreate failed");
    cublasSetStream(m.blas, m.stream);
    cublasSetMathMode(m.blas, CUBLAS_DEFAULT_MATH);   // fp32 SGEMM; TF32 is never enabled
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
    const bool ok = m.h.ensure(tokens * d) && m.ln.ensure(tokens * d) && m.qkv.ensure(tokens * 3 * d) &&
                    m.scores.ensure((size_t)numHeads_ * seq * seq) && m.attn.ensure(tokens * d) &&
                    m.proj.ensure(tokens * d) && m.up.ensure(tokens * F) && m.down.ensure(tokens * d) &&
                    m.last_h.ensure(B * d) && m.last_x.ensure(B * d) && m.last_y.ensure(B * d) &&
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

bool TransformerModel::runForward(const std::vector<int>& tokenIDs, int batch)
{
    Impl& m = *impl_;
    err_.clear();
    if (!loader_.isLoaded() || !m.blas) return fail("model not loaded");
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
    const float one = 1.0f, zero = 0.0f;
    cudaStream_t st = m.stream;
    gbx_stream_t gs = reinterpret_cast<gbx_stream_t>(st);
    int rc = GBX_OK;
    bool blas_ok = true;
    auto check = [&](int r) {
        if (rc == GBX_OK && r != GBX_OK) rc = r;
    };
    auto blas = [&](cublasStatus_t s) {
        if (s != CUBLAS_STATUS_SUCCESS) blas_ok = false;
    };
    // row-major Y[M, Nout] (ld ldy) = X[M, K] (ld ldx) . W[Nout, K]^T (ld K)
    auto linear = [&](const float* X, int64_t ldx, const float* W, float* Y, int64_t ldy, int64_t M, int Nout, int K,
                      float beta) {
        blas(cublasSgemm(m.blas, CUBLAS_OP_T, CUBLAS_OP_N, Nout, (int)M, K, &one, W, K, X, (int)ldx, &beta, Y,
                         (int)ldy));
    };

    if (cudaMemcpyAsync(m.ids, tokenIDs.data(), N * sizeof(int32_t), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemsetAsync(m.err, 0, sizeof(int32_t), st) != cudaSuccess)
        return fail("host-to-device copy of token ids failed");
    check(gbx_embed(m.ids, m.wte, m.wte_dt, m.wpe, m.wpe_dt, nullptr, m.h.p, N, S, 0, d, V, nCtx_, m.err, gs));

    const float scale = sqrtf((float)hd);   // transformer.cu:836
    for (int l = 0; l < numLayers_ && rc == GBX_OK && blas_ok; ++l) {
        const Impl::Layer& L = m.layers[l];
        if (l == 0)
            check(gbx_layernorm(m.h.p, m.ln.p, L.ln1_g, L.ln1_b, N, d, 1e-5f, gs));
        else
            check(gbx_residual_layernorm(m.down.p, m.h.p, m.layers[l - 1].down_b, m.h.p, m.ln.p, L.ln1_g, L.ln1_b, N,
                                         d, 1e-5f, gs));
        // qkv = b_qkv + ln . Wqkv^T
        {
            const int64_t total = N * 3 * d;
            const int grid = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
            broadcast_rows_kernel<<<grid, 256, 0, st>>>(m.qkv.p, 3 * d, L.qkv_b, N, 3 * d);
            if (cudaGetLastError() != cudaSuccess) check(GBX_ECUDA);
        }
        linear(m.ln.p, d, L.qkv_w, m.qkv.p, 3 * d, N, 3 * d, d, 1.0f);
        for (int b = 0; b < batch; ++b) {
            const float* q = m.qkv.p + (int64_t)b * S * 3 * d;
            const float* k = q + d;
            const float* v = q + 2 * d;
            // raw[h][p][s] = sum_i Q[p, h*hd+i] K[s, h*hd+i]
            blas(cublasSgemmStridedBatched(m.blas, CUBLAS_OP_T, CUBLAS_OP_N, S, S, hd, &one, k, 3 * d, hd, q, 3 * d,
                                           hd, &zero, m.scores.p, S, (int64_t)S * S, H));
            check(gbx_attn_softmax_rows(m.scores.p, m.scores.p, (int64_t)H * S, S, S, 0, scale, 1, gs));
            // attn[p, h*hd+i] = sum_s P[h][p][s] V[s, h*hd+i]
            blas(cublasSgemmStridedBatched(m.blas, CUBLAS_OP_N, CUBLAS_OP_N, hd, S, S, &one, v, 3 * d, hd, m.scores.p,
                                           S, (int64_t)S * S, &zero, m.attn.p + (int64_t)b * S * d, d, hd, H));
        }
        linear(m.attn.p, d, L.proj_w, m.proj.p, d, N, d, d, 0.0f);
        check(gbx_residual_layernorm(m.proj.p, m.h.p, L.proj_b, m.h.p, m.ln.p, L.ln2_g, L.ln2_b, N, d, 1e-5f, gs));
        linear(m.ln.p, d, L.up_w, m.up.p, F, N, F, d, 0.0f);
        check(gbx_bias_gelu(m.up.p, m.up.p, L.up_b, N, F, gs));
        linear(m.up.p, F, L.down_w, m.down.p, d, N, d, F, 0.0f);
    }
    if (rc == GBX_OK && blas_ok) {
        // each sequence's last row: h + (down + b_down), then ln_f
        const size_t pitch = (size_t)S * d * sizeof(float);
        const size_t row = (size_t)d * sizeof(float);
        if (cudaMemcpy2DAsync(m.last_h.p, row, m.h.p + (int64_t)(S - 1) * d, pitch, row, batch,
                              cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            check(GBX_ECUDA);
        if (numLayers_ > 0) {
            if (cudaMemcpy2DAsync(m.last_x.p, row, m.down.p + (int64_t)(S - 1) * d, pitch, row, batch,
                                  cudaMemcpyDeviceToDevice, st) != cudaSuccess)
                check(GBX_ECUDA);
            check(gbx_residual_layernorm(m.last_x.p, m.last_h.p, m.layers[numLayers_ - 1].down_b, nullptr, m.last_y.p,
                                         m.lnf_g, m.lnf_b, batch, d, 1e-5f, gs));
        } else {
            check(gbx_layernorm(m.last_h.p, m.last_y.p, m.lnf_g, m.lnf_b, batch, d, 1e-5f, gs));
        }
        check(gbx_logits(m.last_y.p, batch, m.wte, m.wte_dt, m.logits.p, V, d, gs));
    }
    int32_t err_host = 0;
    if (rc == GBX_OK && blas_ok &&
        cudaMemcpyAsync(&err_host, m.err, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess)
        rc = GBX_ECUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess && rc == GBX_OK) rc = GBX_ECUDA;
    if (!blas_ok) return fail("cuBLAS call failed");
    if (rc != GBX_OK) return fail(std::string(gbx_status_string(rc)) + ": " + gbx_last_error());
    if (err_host) return fail("embedding reported out-of-range ids or positions");
    return true;
}

}  // namespace gbx
