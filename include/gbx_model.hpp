// gbx_model.hpp -- C++ surface of the B200 hot path, mirroring the classes
// GlassBoxAI-Transformer's callers use: GGUFLoader (transformer.cu:480-740)
// and TransformerModel (transformer.cu:744-1051).  A caller of the reference
// switches by including this header, using namespace gbx, and linking
// libgbx_model.so; the method names, argument meaning and return conventions
// are the reference's:
//
//   GGUFLoader::loadFromFile(path) -> bool                (transformer.cu:657-674)
//   GGUFLoader::getTensorGPU({names...}) -> float*        (:676-695, fp32 device copy, cached)
//   GGUFLoader::getTensor({names...}) -> std::vector<float> (:697-706, host fp32 copy)
//   GGUFLoader::hasTensor(name) -> bool                   (:708-710)
//   GGUFLoader::printAllTensorNames()                     (:712-722)
//   GGUFLoader::freeGPUMemory()                           (:724-731)
//   GGUFLoader::getEmbedDim/NumLayers/NumHeads/FFNDim/VocabSize/MaxSeqLen/isLoaded (:733-739)
//   TransformerModel::loadModel(path) -> bool             (:937-949)
//   TransformerModel::forward(tokenIDs) -> last-row logits (:913-927; public here, as README.md:107-108
//                                                           documents it)
//
// Differences, each deliberate:
//   - No call ever exits the process.  Where the reference's CUDA_CHECK would
//     print and exit(1) (transformer.cu:24-32), methods return their failure
//     value (false / nullptr / empty vector) and lastError() says why.
//   - The header is parsed from a read-only memory map with every read
//     bounds-checked; a truncated or malformed file fails loadFromFile (the
//     reference reads past the end of its stream).  general.alignment is
//     honoured (the reference always aligns tensor data to 32 bytes, which is
//     GGUF's default).
//   - getTensorGPU decodes f16/bf16 on the device (gbx_dequant, bit-identical
//     to the reference's host loop) instead of on the host.
//   - getTensor after getTensorGPU still returns the data (the reference's
//     returns an empty vector then: its host copy was released).
//   - getTensorGPURaw (new) gives the tensor's GGUF bytes on the device; the
//     embedding and logits kernels read wte/wpe that way, so f16/bf16 tables
//     are never widened to fp32 in HBM.
//   - forward checks its input: an empty sequence, an id outside the token
//     table or more tokens than position rows return an empty vector (the
//     reference launches an invalid grid or reads out of bounds).  The vocab
//     size of the logits is the token table's row count (the reference's
//     getVocabSize() is the constant 50257, transformer.cu:492).
//   - forwardBatch (new) runs `batch` equal-length sequences in one pass.
//   - nextToken (new) is one step of generate without the tokenizer: the
//     argmax / temperature sampling of transformer.cu:994-1028 runs on the
//     device (gbx_select_tokens), so the logits never cross to the host.
//   - The weight contractions (QKV, projection, FFN up/down) run on the
//     tcgen05 tensor cores (gbx_linear, gbx_linear_splitk when the output
//     tiles are few) with fp32 operands carried as tf32 pairs, their bias,
//     GELU and residual fused into the epilogue; the per-head score and
//     P.V products run on the same kernel (gbx_attn_scores,
//     gbx_attn_values), every head of every sequence in one launch.  The hot path
//     itself (embed, LayerNorm, score epilogue + softmax, logits) runs on the
//     sm_100a kernels behind gbx.h.  Loading keeps a tf32 pair of every f32
//     weight matrix on the device (two extra fp32 copies); f16 / bf16
//     weights need none.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "gbx.h"

namespace gbx {

struct GGUFTensor {
    std::string name;
    std::vector<int64_t> shape;   // GGUF ne[] order, innermost first (as the reference stores it)
    int numDims = 0;
    int dtype = 0;                // GGUF type code
    int64_t dataOffset = 0;       // from the start of the tensor-data section
    int64_t numElements = 0;
    void* d_raw = nullptr;        // device copy of the GGUF bytes (getTensorGPURaw)
    float* d_data = nullptr;      // device fp32 copy (getTensorGPU)
};

struct GGUFConfig {
    int embedDim = 768;     // defaults of transformer.cu:488-493
    int numLayers = 12;
    int numHeads = 12;
    int ffnDim = 3072;
    int vocabSize = 50257;
    int maxSeqLen = 1024;
};

class GGUFLoader {
public:
    GGUFLoader();
    ~GGUFLoader();
    GGUFLoader(const GGUFLoader&) = delete;
    GGUFLoader& operator=(const GGUFLoader&) = delete;

    bool loadFromFile(const std::string& fname);
    float* getTensorGPU(const std::vector<std::string>& names);
    std::vector<float> getTensor(const std::vector<std::string>& names);
    bool hasTensor(const std::string& name) const;
    void printAllTensorNames() const;
    void freeGPUMemory();

    // New: the tensor's GGUF bytes on the device (cached); dtype and element
    // count through the optional out-pointers.  nullptr if no name matches,
    // the dtype is not f32/f16/bf16, or an upload fails.
    const void* getTensorGPURaw(const std::vector<std::string>& names, int* dtype = nullptr,
                                int64_t* numElements = nullptr);
    // New: metadata of the first tensor found under `names` (nullptr if none).
    const GGUFTensor* findTensor(const std::vector<std::string>& names) const;

    int getEmbedDim() const { return cfg_.embedDim; }
    int getNumLayers() const { return cfg_.numLayers; }
    int getNumHeads() const { return cfg_.numHeads; }
    int getFFNDim() const { return cfg_.ffnDim; }
    int getVocabSize() const { return cfg_.vocabSize; }
    int getMaxSeqLen() const { return cfg_.maxSeqLen; }
    bool isLoaded() const { return loaded_; }
    const GGUFConfig& config() const { return cfg_; }
    size_t tensorCount() const { return tensors_.size(); }
    const std::string& lastError() const { return err_; }

private:
    bool parse();
    bool tensorBytes(const GGUFTensor& t, const uint8_t** p, int64_t* nbytes);
    bool upload(const void* host, int64_t nbytes, void** dev);
    bool fail(const std::string& msg);

    std::string filename_;
    const uint8_t* map_ = nullptr;
    size_t mapSize_ = 0;
    int fd_ = -1;
    std::vector<GGUFTensor> tensors_;
    std::map<std::string, size_t> tensorMap_;
    int64_t tensorDataStart_ = 0;
    GGUFConfig cfg_;
    bool loaded_ = false;
    int device_ = -1;
    std::string err_;
};

class TransformerModel {
public:
    TransformerModel();
    ~TransformerModel();
    TransformerModel(const TransformerModel&) = delete;
    TransformerModel& operator=(const TransformerModel&) = delete;

    bool loadModel(const std::string& ggufPath);
    // Logits of the last token (one row of vocab floats), as the reference.
    std::vector<float> forward(const std::vector<int>& tokenIDs);
    // `batch` sequences of tokenIDs.size()/batch tokens each, concatenated;
    // returns batch rows of logits (each sequence's last token).
    std::vector<float> forwardBatch(const std::vector<int>& tokenIDs, int batch);
    // One step of generate's loop (transformer.cu:986-1036) without the
    // tokenizer: forward, then the reference's argmax / temperature sampling
    // (:994-1028) on the device, drawing from `rng` exactly when the
    // reference draws (temperature > 0.01).  Returns the selected id (-1 on
    // failure, see lastError()); bestID / bestLogit as the reference prints.
    int nextToken(const std::vector<int>& tokenIDs, double temperature, std::mt19937& rng, int* bestID = nullptr,
                  float* bestLogit = nullptr);
    // The same with the uniform draw in [0, 1) supplied by the caller.
    int nextTokenWithDraw(const std::vector<int>& tokenIDs, double temperature, double u, int* bestID = nullptr,
                          float* bestLogit = nullptr);

    // New (inspection): the residual stream h after the embedding and after
    // each layer of forwardBatch(tokenIDs, batch): (layers + 1) blocks of
    // tokens x embedDim floats, layer by layer; empty on failure.
    std::vector<float> forwardHidden(const std::vector<int>& tokenIDs, int batch = 1);
    // New: the attention of head width 64 as one fused launch (gbx_attn_fused,
    // the default) or as the per-head products (gbx_attn_scores, the score
    // softmax, gbx_attn_values); the results differ only in rounding.
    void setFusedAttention(bool on);
    bool fusedAttention() const;

    bool isModelLoaded() const { return loader_.isLoaded(); }
    void printTensorNames() { loader_.printAllTensorNames(); }
    GGUFLoader& getLoader() { return loader_; }
    int getEmbedDim() const { return embedDim_; }
    int getNumLayers() const { return numLayers_; }
    int getNumHeads() const { return numHeads_; }
    int getFFNDim() const { return ffnDim_; }
    int getVocabSize() const { return vocab_; }     // token-table rows
    int getMaxSeqLen() const { return nCtx_; }      // position-table rows
    const std::string& lastError() const { return err_; }

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
    GGUFLoader loader_;
    int embedDim_ = 0, numHeads_ = 0, headDim_ = 0, numLayers_ = 0, ffnDim_ = 0, vocab_ = 0, nCtx_ = 0;
    std::string err_;
    bool fail(const std::string& msg);
    bool ensureBuffers(int64_t tokens, int seq);
    // logits stay on the device; hidden_host (optional) receives forwardHidden's blocks
    bool runForward(const std::vector<int>& tokenIDs, int batch, float* hidden_host = nullptr);
};

// Row sharding across GPUs with one host thread per device: a replica of
// the model on each listed device, a batch of sequences split into
// contiguous whole-sequence shards (shares within one of each other), each
// shard run on its device's thread, the logits gathered in order on the
// host.  No collective and no peer memory: the only exchange is the final
// device-to-host copy of each shard's logits.  A device may be listed twice
// (two replicas on one GPU).
class ShardedModel {
public:
    ShardedModel();
    ~ShardedModel();
    ShardedModel(const ShardedModel&) = delete;
    ShardedModel& operator=(const ShardedModel&) = delete;

    bool loadModel(const std::string& ggufPath, const std::vector<int>& devices);
    // As TransformerModel::forwardBatch: `batch` equal-length sequences,
    // batch rows of logits.  Fails as a whole if any shard fails.
    std::vector<float> forwardBatch(const std::vector<int>& tokenIDs, int batch);
    int replicas() const { return (int)models_.size(); }
    int getVocabSize() const { return models_.empty() ? 0 : models_[0]->getVocabSize(); }
    const std::string& lastError() const { return err_; }

private:
    std::vector<std::unique_ptr<TransformerModel>> models_;
    std::vector<int> devices_;
    std::string err_;
};

}  // namespace gbx
