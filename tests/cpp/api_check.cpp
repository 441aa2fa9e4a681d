// api_check.cpp -- a C++ caller of gbx_model.hpp, written the way the
// reference's own code calls its GGUFLoader / TransformerModel
// (transformer.cu:937-1046).  Built by the test suite with g++ against the
// installed headers and libraries:
//   api_check loader <file.gguf> <tensor>   -> config, hasTensor, getTensor checksum
//   api_check model  <file.gguf> <id...>    -> forward logits checksum, argmax,
//                                              nextToken at T=0 and T=0.8 (mt19937 seed 1234),
//                                              forwardHidden (block count, last block's checksum),
//                                              the argmax with the per-head attention products
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <string>
#include <vector>

#include "gbx_model.hpp"

static double checksum(const std::vector<float>& v)
{
    double s = 0.0;
    for (size_t i = 0; i < v.size(); ++i) s += (double)v[i] * (double)((i % 7) + 1);
    return s;
}

int main(int argc, char** argv)
{
    if (argc < 4) {
        std::fprintf(stderr, "usage: api_check loader|model file.gguf ...\n");
        return 2;
    }
    const std::string mode = argv[1], path = argv[2];
    if (mode == "loader") {
        gbx::GGUFLoader loader;
        if (!loader.loadFromFile(path)) {
            std::printf("error %s\n", loader.lastError().c_str());
            return 1;
        }
        std::vector<float> t = loader.getTensor({"missing.weight", argv[3]});   // alias list, first match wins
        std::printf("config %d %d %d %d %d %d\n", loader.getEmbedDim(), loader.getNumLayers(), loader.getNumHeads(),
                    loader.getFFNDim(), loader.getVocabSize(), loader.getMaxSeqLen());
        std::printf("has %d %d\n", (int)loader.hasTensor(argv[3]), (int)loader.hasTensor("missing.weight"));
        std::printf("tensor %zu %.17g\n", t.size(), checksum(t));
        return 0;
    }
    gbx::TransformerModel model;
    if (!model.loadModel(path)) {
        std::printf("error %s\n", model.lastError().c_str());
        return 1;
    }
    std::vector<int> ids;
    for (int i = 3; i < argc; ++i) ids.push_back(std::atoi(argv[i]));
    std::vector<float> logits = model.forward(ids);
    if (logits.empty()) {
        std::printf("error %s\n", model.lastError().c_str());
        return 1;
    }
    int best = 0;
    for (size_t j = 1; j < logits.size(); ++j)
        if (logits[j] > logits[best]) best = (int)j;
    std::printf("logits %zu %.17g %d\n", logits.size(), checksum(logits), best);
    std::mt19937 rng(1234);
    int b0 = -1, b1 = -1;
    float l0 = 0, l1 = 0;
    const int greedy = model.nextToken(ids, 0.0, rng, &b0, &l0);
    const int sampled = model.nextToken(ids, 0.8, rng, &b1, &l1);
    std::printf("next %d %d %d %d\n", greedy, b0, sampled, b1);
    // inspection: the residual stream after the embedding and after every layer
    const std::vector<float> hidden = model.forwardHidden(ids);
    const size_t block = ids.size() * (size_t)model.getEmbedDim();
    if (hidden.size() != (size_t)(model.getNumLayers() + 1) * block) {
        std::printf("error forwardHidden returned %zu floats\n", hidden.size());
        return 1;
    }
    const std::vector<float> last(hidden.end() - block, hidden.end());
    std::printf("hidden %d %.17g\n", model.getNumLayers() + 1, checksum(last));
    // the same forward on the per-head attention products
    model.setFusedAttention(false);
    const std::vector<float> unfused = model.forward(ids);
    model.setFusedAttention(true);
    int ubest = 0;
    for (size_t j = 1; j < unfused.size(); ++j)
        if (unfused[j] > unfused[ubest]) ubest = (int)j;
    std::printf("unfused %zu %d %d\n", unfused.size(), ubest, (int)model.fusedAttention());
    return greedy < 0 || sampled < 0 || unfused.empty() ? 1 : 0;
}
