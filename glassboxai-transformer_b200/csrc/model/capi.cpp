// capi.cpp -- the C ABI of gbx_model.h over the C++ classes.
#include <cstring>
#include <new>

#include "gbx_model.h"
#include "gbx_model.hpp"

namespace gbx {
int set_error(int code, const char* fmt, ...);
}

struct gbx_gguf {
    gbx::GGUFLoader loader;
};

struct gbx_model {
    gbx::TransformerModel model;
};

struct gbx_sharded {
    gbx::ShardedModel model;
};

extern "C" {

gbx_gguf* gbx_gguf_open(const char* path)
{
    if (!path) {
        gbx::set_error(GBX_EINVAL, "gbx_gguf_open: null path");
        return nullptr;
    }
    gbx_gguf* g = new (std::nothrow) gbx_gguf;
    if (!g) {
        gbx::set_error(GBX_ENOMEM, "gbx_gguf_open: out of memory");
        return nullptr;
    }
    if (!g->loader.loadFromFile(path)) {
        gbx::set_error(GBX_EIO, "%s", g->loader.lastError().c_str());
        delete g;
        return nullptr;
    }
    return g;
}

void gbx_gguf_close(gbx_gguf* g) { delete g; }

int64_t gbx_gguf_get_tensor(gbx_gguf* g, const char* name, float* dst_host, int64_t cap)
{
    if (!g || !name) return gbx::set_error(GBX_EINVAL, "gbx_gguf_get_tensor: null argument"), -1;
    const gbx::GGUFTensor* t = g->loader.findTensor({name});
    if (t && t->numElements > cap) return gbx::set_error(GBX_ERANGE, "gbx_gguf_get_tensor: capacity"), -1;
    std::vector<float> v = g->loader.getTensor({name});
    if (!v.empty()) std::memcpy(dst_host, v.data(), v.size() * sizeof(float));
    return (int64_t)v.size();
}

int gbx_gguf_has_tensor(gbx_gguf* g, const char* name) { return g && name && g->loader.hasTensor(name) ? 1 : 0; }

int gbx_gguf_config(gbx_gguf* g, int32_t out6[6])
{
    if (!g || !out6) return gbx::set_error(GBX_EINVAL, "gbx_gguf_config: null argument");
    const gbx::GGUFConfig& c = g->loader.config();
    out6[0] = c.embedDim;
    out6[1] = c.numLayers;
    out6[2] = c.numHeads;
    out6[3] = c.ffnDim;
    out6[4] = c.vocabSize;
    out6[5] = c.maxSeqLen;
    return GBX_OK;
}

const float* gbx_gguf_tensor_gpu(gbx_gguf* g, const char* name)
{
    if (!g || !name) return gbx::set_error(GBX_EINVAL, "gbx_gguf_tensor_gpu: null argument"), nullptr;
    const float* p = g->loader.getTensorGPU({name});
    if (!p) gbx::set_error(GBX_ENOTFOUND, "%s", g->loader.lastError().c_str());
    return p;
}

const void* gbx_gguf_tensor_gpu_raw(gbx_gguf* g, const char* name, int* dtype, int64_t* n)
{
    if (!g || !name) return gbx::set_error(GBX_EINVAL, "gbx_gguf_tensor_gpu_raw: null argument"), nullptr;
    const void* p = g->loader.getTensorGPURaw({name}, dtype, n);
    if (!p) gbx::set_error(GBX_ENOTFOUND, "%s", g->loader.lastError().c_str());
    return p;
}

gbx_model* gbx_model_open(const char* gguf_path)
{
    if (!gguf_path) {
        gbx::set_error(GBX_EINVAL, "gbx_model_open: null path");
        return nullptr;
    }
    gbx_model* m = new (std::nothrow) gbx_model;
    if (!m) {
        gbx::set_error(GBX_ENOMEM, "gbx_model_open: out of memory");
        return nullptr;
    }
    if (!m->model.loadModel(gguf_path)) {
        gbx::set_error(GBX_EIO, "%s", m->model.lastError().c_str());
        delete m;
        return nullptr;
    }
    return m;
}

void gbx_model_close(gbx_model* m) { delete m; }

int gbx_model_config(gbx_model* m, int32_t out6[6])
{
    if (!m || !out6) return gbx::set_error(GBX_EINVAL, "gbx_model_config: null argument");
    out6[0] = m->model.getEmbedDim();
    out6[1] = m->model.getNumLayers();
    out6[2] = m->model.getNumHeads();
    out6[3] = m->model.getFFNDim();
    out6[4] = m->model.getVocabSize();
    out6[5] = m->model.getMaxSeqLen();
    return GBX_OK;
}

int gbx_model_forward(gbx_model* m, const int32_t* ids_host, int64_t n_ids, int batch, float* logits_host)
{
    if (!m || !ids_host || !logits_host || n_ids <= 0 || batch <= 0)
        return gbx::set_error(GBX_EINVAL, "gbx_model_forward: bad argument");
    std::vector<int> ids(ids_host, ids_host + n_ids);
    std::vector<float> out = m->model.forwardBatch(ids, batch);
    if (out.empty()) return gbx::set_error(GBX_EINVAL, "%s", m->model.lastError().c_str());
    std::memcpy(logits_host, out.data(), out.size() * sizeof(float));
    return GBX_OK;
}

int gbx_model_forward_hidden(gbx_model* m, const int32_t* ids_host, int64_t n_ids, int batch, float* hidden_host,
                             int64_t cap)
{
    if (!m || !ids_host || !hidden_host || n_ids <= 0 || batch <= 0)
        return gbx::set_error(GBX_EINVAL, "gbx_model_forward_hidden: bad argument");
    const int64_t need = (int64_t)(m->model.getNumLayers() + 1) * n_ids * m->model.getEmbedDim();
    if (cap < need)
        return gbx::set_error(GBX_ERANGE, "gbx_model_forward_hidden: %lld floats needed, %lld given", (long long)need,
                              (long long)cap);
    std::vector<int> ids(ids_host, ids_host + n_ids);
    std::vector<float> out = m->model.forwardHidden(ids, batch);
    if (out.empty()) return gbx::set_error(GBX_EINVAL, "%s", m->model.lastError().c_str());
    std::memcpy(hidden_host, out.data(), out.size() * sizeof(float));
    return GBX_OK;
}

int gbx_model_set_fused_attention(gbx_model* m, int on)
{
    if (!m) return gbx::set_error(GBX_EINVAL, "gbx_model_set_fused_attention: null model");
    const int prev = m->model.fusedAttention() ? 1 : 0;
    m->model.setFusedAttention(on != 0);
    return prev;
}

int gbx_model_next_token(gbx_model* m, const int32_t* ids_host, int64_t n_ids, double temperature, double u,
                         int32_t* out_id, int32_t* best, float* best_logit)
{
    if (!m || !ids_host || !out_id || n_ids <= 0) return gbx::set_error(GBX_EINVAL, "gbx_model_next_token: bad argument");
    std::vector<int> ids(ids_host, ids_host + n_ids);
    int b = 0;
    float bl = 0.0f;
    const int sel = m->model.nextTokenWithDraw(ids, temperature, u, &b, &bl);
    if (sel < 0) return gbx::set_error(GBX_EINVAL, "%s", m->model.lastError().c_str());
    *out_id = sel;
    if (best) *best = b;
    if (best_logit) *best_logit = bl;
    return GBX_OK;
}

gbx_sharded* gbx_sharded_open(const char* gguf_path, const int32_t* devices, int n)
{
    if (!gguf_path || !devices || n <= 0) {
        gbx::set_error(GBX_EINVAL, "gbx_sharded_open: bad argument");
        return nullptr;
    }
    gbx_sharded* s = new (std::nothrow) gbx_sharded;
    if (!s) {
        gbx::set_error(GBX_ENOMEM, "gbx_sharded_open: out of memory");
        return nullptr;
    }
    if (!s->model.loadModel(gguf_path, std::vector<int>(devices, devices + n))) {
        gbx::set_error(GBX_EIO, "%s", s->model.lastError().c_str());
        delete s;
        return nullptr;
    }
    return s;
}

void gbx_sharded_close(gbx_sharded* s) { delete s; }

int gbx_sharded_forward(gbx_sharded* s, const int32_t* ids_host, int64_t n_ids, int batch, float* logits_host)
{
    if (!s || !ids_host || !logits_host || n_ids <= 0 || batch <= 0)
        return gbx::set_error(GBX_EINVAL, "gbx_sharded_forward: bad argument");
    std::vector<int> ids(ids_host, ids_host + n_ids);
    std::vector<float> out = s->model.forwardBatch(ids, batch);
    if (out.empty()) return gbx::set_error(GBX_EINVAL, "%s", s->model.lastError().c_str());
    std::memcpy(logits_host, out.data(), out.size() * sizeof(float));
    return GBX_OK;
}

}  // extern "C"
