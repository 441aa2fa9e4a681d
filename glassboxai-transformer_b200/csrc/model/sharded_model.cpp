// sharded_model.cpp -- ShardedModel: the row-sharded forward over several
// GPUs, one host thread per device (see gbx_model.hpp).
#include <cuda_runtime.h>

#include <cstring>
#include <thread>

#include "gbx_model.hpp"

namespace gbx {

ShardedModel::ShardedModel() = default;
ShardedModel::~ShardedModel() = default;

bool ShardedModel::loadModel(const std::string& ggufPath, const std::vector<int>& devices)
{
    err_.clear();
    if (devices.empty()) {
        err_ = "ShardedModel: no devices";
        return false;
    }
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess) {
        err_ = "ShardedModel: cudaGetDeviceCount failed";
        return false;
    }
    for (int d : devices)
        if (d < 0 || d >= count) {
            err_ = "ShardedModel: no device " + std::to_string(d);
            return false;
        }
    models_.clear();
    devices_ = devices;
    int cur = 0;
    cudaGetDevice(&cur);
    // load the replicas in parallel: each thread binds its device first
    std::vector<std::unique_ptr<TransformerModel>> models(devices.size());
    std::vector<std::string> errs(devices.size());
    std::vector<std::thread> th;
    for (size_t i = 0; i < devices.size(); ++i)
        th.emplace_back([&, i] {
            if (cudaSetDevice(devices[i]) != cudaSuccess) {
                errs[i] = "cudaSetDevice failed";
                return;
            }
            models[i].reset(new TransformerModel());
            if (!models[i]->loadModel(ggufPath)) errs[i] = models[i]->lastError();
        });
    for (auto& t : th) t.join();
    cudaSetDevice(cur);
    for (size_t i = 0; i < devices.size(); ++i)
        if (!errs[i].empty()) {
            err_ = "device " + std::to_string(devices[i]) + ": " + errs[i];
            return false;
        }
    models_ = std::move(models);
    return true;
}

std::vector<float> ShardedModel::forwardBatch(const std::vector<int>& tokenIDs, int batch)
{
    err_.clear();
    const int n = (int)models_.size();
    if (!n) return err_ = "ShardedModel: not loaded", std::vector<float>();
    if (batch <= 0 || tokenIDs.empty() || tokenIDs.size() % (size_t)batch)
        return err_ = "forward: need batch > 0 sequences of equal, non-zero length", std::vector<float>();
    const size_t S = tokenIDs.size() / (size_t)batch;
    const size_t V = (size_t)models_[0]->getVocabSize();
    std::vector<float> out((size_t)batch * V);
    std::vector<std::string> errs(n);
    std::vector<std::thread> th;
    const int base = batch / n, extra = batch % n;
    for (int r = 0; r < n; ++r) {
        const int first = r * base + (r < extra ? r : extra);
        const int count = base + (r < extra ? 1 : 0);
        if (!count) continue;
        th.emplace_back([&, r, first, count] {
            if (cudaSetDevice(devices_[r]) != cudaSuccess) {
                errs[r] = "cudaSetDevice failed";
                return;
            }
            std::vector<int> ids(tokenIDs.begin() + (ptrdiff_t)(first * S),
                                 tokenIDs.begin() + (ptrdiff_t)((first + count) * S));
            std::vector<float> part = models_[r]->forwardBatch(ids, count);
            if (part.empty()) {
                errs[r] = models_[r]->lastError();
                return;
            }
            std::memcpy(out.data() + (size_t)first * V, part.data(), part.size() * sizeof(float));
        });
    }
    for (auto& t : th) t.join();
    for (int r = 0; r < n; ++r)
        if (!errs[r].empty()) return err_ = "device " + std::to_string(devices_[r]) + ": " + errs[r], std::vector<float>();
    return out;
}

}  // namespace gbx
