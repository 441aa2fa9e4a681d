// ref_shim.cu -- TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference's own transformer.cu, unmodified, from where it lies
// (the include path is given by oracle/Makefile) and exports a C ABI over the
// pieces of it that the hot path covers, so the tests and the reference arm
// of the benchmark can run the reference's *own* code:
//
//   ref_gguf_*            GGUFLoader::loadFromFile / getTensor / getters
//                         (transformer.cu:657-674, 697-706, 733-738): the
//                         reference's host-side f16/bf16 -> f32 dequant.
//   ref_launch_embed      embedTokensKernel with its launch shape
//                         (grid seqLen, block embedDim; transformer.cu:811-813)
//   ref_launch_layernorm  layerNormKernel (grid rows, block 256, 1 KB smem;
//                         transformer.cu:827-828)
//   ref_launch_softmax    softmaxKernel (grid rows, block 256, 1 KB smem;
//                         transformer.cu:839-842, one launch per head there)
//   ref_launch_gelu       geluKernel (1 thread per element, block 256)
//   ref_launch_add        addResidualKernel (1 thread per element, block 256)
//   ref_model_*           TransformerModel::loadModel / forward (transformer.cu:
//                         913-949): the reference's whole GPU forward, for the
//                         end-to-end parity test of the drop-in TransformerModel;
//                         ref_model_forward_hidden runs the same steps and also
//                         returns the residual stream after every layer.
//                         forward is a private member there, so the reference's
//                         source is compiled with `private` spelled `public`;
//                         that changes access checking only, not code.
//
// The only deviation from the reference's launches is the stream argument:
// the reference uses the legacy default stream; these take one.
// Nothing in the product library links this file.
#include <iostream>
#include <fstream>
#include <sstream>
#include <vector>
#include <string>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <algorithm>
#include <random>
#include <chrono>
#include <limits>
#include <iomanip>

#include <cuda_runtime.h>
#include <device_launch_parameters.h>

#define main glassbox_reference_main
#define private public
#include "transformer.cu"
#undef private
#undef main

extern "C" {

void* ref_gguf_open(const char* path)
{
    GGUFLoader* l = new GGUFLoader();
    if (!l->loadFromFile(path)) { delete l; return nullptr; }
    return l;
}

void ref_gguf_close(void* h) { delete static_cast<GGUFLoader*>(h); }

// GGUFLoader::getTensor({name}) copied into dst (capacity `cap` floats).
// Returns the element count (0 when the reference returns an empty vector,
// -1 when dst is too small).
int64_t ref_gguf_get_tensor(void* h, const char* name, float* dst, int64_t cap)
{
    std::vector<float> v = static_cast<GGUFLoader*>(h)->getTensor({std::string(name)});
    if ((int64_t)v.size() > cap) return -1;
    if (!v.empty()) std::memcpy(dst, v.data(), v.size() * sizeof(float));
    return (int64_t)v.size();
}

int ref_gguf_has_tensor(void* h, const char* name)
{
    return static_cast<GGUFLoader*>(h)->hasTensor(std::string(name)) ? 1 : 0;
}

// embedDim, numLayers, numHeads, ffnDim, vocabSize, maxSeqLen
void ref_gguf_config(void* h, int* out6)
{
    GGUFLoader* l = static_cast<GGUFLoader*>(h);
    out6[0] = l->getEmbedDim(); out6[1] = l->getNumLayers(); out6[2] = l->getNumHeads();
    out6[3] = l->getFFNDim(); out6[4] = l->getVocabSize(); out6[5] = l->getMaxSeqLen();
}

int ref_launch_embed(const int* ids, const float* wte, const float* wpe, float* out,
                     int seqLen, int embedDim, void* stream)
{
    embedTokensKernel<<<dim3(seqLen), dim3(embedDim), 0, (cudaStream_t)stream>>>(
        ids, wte, wpe, out, seqLen, embedDim);
    return (int)cudaGetLastError();
}

int ref_launch_layernorm(const float* in, float* out, const float* g, const float* b,
                         int rows, int dim, void* stream)
{
    layerNormKernel<<<rows, BLOCK_SIZE, BLOCK_SIZE * sizeof(float), (cudaStream_t)stream>>>(
        in, out, g, b, rows, dim);
    return (int)cudaGetLastError();
}

int ref_launch_softmax(float* data, int rows, int cols, void* stream)
{
    softmaxKernel<<<rows, BLOCK_SIZE, BLOCK_SIZE * sizeof(float), (cudaStream_t)stream>>>(
        data, rows, cols);
    return (int)cudaGetLastError();
}

int ref_launch_gelu(float* data, int size, void* stream)
{
    geluKernel<<<(size + BLOCK_SIZE - 1) / BLOCK_SIZE, BLOCK_SIZE, 0, (cudaStream_t)stream>>>(
        data, size);
    return (int)cudaGetLastError();
}

int ref_launch_add(float* out, const float* residual, int size, void* stream)
{
    addResidualKernel<<<(size + BLOCK_SIZE - 1) / BLOCK_SIZE, BLOCK_SIZE, 0, (cudaStream_t)stream>>>(
        out, residual, size);
    return (int)cudaGetLastError();
}

int ref_block_size(void) { return BLOCK_SIZE; }

void* ref_model_open(const char* path)
{
    TransformerModel* m = new TransformerModel();
    if (!m->loadModel(path)) { delete m; return nullptr; }
    return m;
}

void ref_model_close(void* m) { delete static_cast<TransformerModel*>(m); }

// TransformerModel::forward(tokenIDs): the last token's logits
// (vocabSize = 50257 of them, transformer.cu:492).  Returns the count, or -1
// when `cap` is too small.
int64_t ref_model_forward(void* m, const int* ids, int n, float* logits, int64_t cap)
{
    std::vector<int> v(ids, ids + n);
    std::vector<float> out = static_cast<TransformerModel*>(m)->forward(v);
    if ((int64_t)out.size() > cap) return -1;
    std::memcpy(logits, out.data(), out.size() * sizeof(float));
    return (int64_t)out.size();
}

// TransformerModel::forward (transformer.cu:913-927) step by step through the
// reference's own member functions, in forward's order (embedTokens, then
// attentionBlock and ffnBlock per layer, then computeLogits; only the progress
// print is left out), copying its residual stream d_hidden to the host after
// the embedding and after each layer: hidden receives (numLayers + 1) blocks
// of n x embedDim floats, logits the last token's logits.  Returns the block
// count, or -1 when a capacity is too small.
int64_t ref_model_forward_hidden(void* mp, const int* ids, int n, float* hidden, int64_t cap, float* logits,
                                 int64_t lcap)
{
    TransformerModel* m = static_cast<TransformerModel*>(mp);
    const int64_t per = (int64_t)n * m->embedDim;
    if (cap < per * (m->numLayers + 1) || lcap < m->vocabSize) return -1;
    std::vector<int> v(ids, ids + n);
    m->allocateBuffers(n);
    m->embedTokens(v, n);
    cudaMemcpy(hidden, m->d_hidden, per * sizeof(float), cudaMemcpyDeviceToHost);
    for (int l = 0; l < m->numLayers; l++) {
        m->attentionBlock(n, l);
        m->ffnBlock(n, l);
        cudaMemcpy(hidden + (l + 1) * per, m->d_hidden, per * sizeof(float), cudaMemcpyDeviceToHost);
    }
    std::vector<float> out = m->computeLogits(n);
    std::memcpy(logits, out.data(), out.size() * sizeof(float));
    return m->numLayers + 1;
}

}  // extern "C"
