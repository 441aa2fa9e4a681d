/*
 * gbx_model.h -- C ABI over the C++ GGUFLoader / TransformerModel of
 * gbx_model.hpp, for callers that bind C (ctypes, cgo, JNI, N-API).
 * Host buffers only; every call is synchronous.  Failures return NULL / a
 * negative count / a GBX_E* code, with the reason in gbx_last_error()
 * (per host thread).  Nothing here exits the process.
 */
#ifndef GBX_MODEL_H
#define GBX_MODEL_H

#include <stdint.h>

#include "gbx.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct gbx_gguf gbx_gguf;
typedef struct gbx_model gbx_model;
typedef struct gbx_sharded gbx_sharded;

/* GGUFLoader::loadFromFile (transformer.cu:657-674). */
gbx_gguf* gbx_gguf_open(const char* path);
void gbx_gguf_close(gbx_gguf* g);
/* GGUFLoader::getTensor({name}) (transformer.cu:697-706): fp32 values
 * decoded with the reference's rules into dst (capacity cap floats).
 * Returns the element count, 0 when the reference would return an empty
 * vector (no such tensor, unsupported dtype), -1 when cap is too small. */
int64_t gbx_gguf_get_tensor(gbx_gguf* g, const char* name, float* dst_host, int64_t cap);
/* GGUFLoader::hasTensor (transformer.cu:708-710). */
int gbx_gguf_has_tensor(gbx_gguf* g, const char* name);
/* embed_dim, num_layers, num_heads, ffn_dim, vocab_size, max_seq_len: the
 * reference's getters (transformer.cu:733-738; vocab_size is its constant). */
int gbx_gguf_config(gbx_gguf* g, int32_t out6[6]);
/* GGUFLoader::getTensorGPU (transformer.cu:676-695): cached fp32 device copy. */
const float* gbx_gguf_tensor_gpu(gbx_gguf* g, const char* name);
/* The tensor's GGUF bytes on the device (cached), its dtype and element count. */
const void* gbx_gguf_tensor_gpu_raw(gbx_gguf* g, const char* name, int* dtype, int64_t* n);

/* TransformerModel::loadModel (transformer.cu:937-949) on the current device. */
gbx_model* gbx_model_open(const char* gguf_path);
void gbx_model_close(gbx_model* m);
/* embed_dim, num_layers, num_heads, ffn_dim, vocab (token-table rows),
 * n_ctx (position-table rows). */
int gbx_model_config(gbx_model* m, int32_t out6[6]);
/* TransformerModel::forward (transformer.cu:913-927) for `batch` sequences
 * of n_ids/batch tokens: logits_host receives batch x vocab floats, the
 * logits of each sequence's last token. */
int gbx_model_forward(gbx_model* m, const int32_t* ids_host, int64_t n_ids, int batch, float* logits_host);

/* The residual stream of gbx_model_forward's sequences after the embedding
 * and after each layer (no counterpart in the reference; for inspecting a
 * forward layer by layer): hidden_host receives (num_layers + 1) blocks of
 * n_ids x embed_dim floats; cap is its capacity in floats (GBX_ERANGE when
 * too small). */
int gbx_model_forward_hidden(gbx_model* m, const int32_t* ids_host, int64_t n_ids, int batch, float* hidden_host,
                             int64_t cap);

/* Attention of head width 64 in one fused launch (on != 0, the default) or as
 * the per-head products; returns the previous setting (or a GBX_E* code for
 * a NULL model).  The two differ only in rounding. */
int gbx_model_set_fused_attention(gbx_model* m, int on);

/* One step of generate's loop without the tokenizer (transformer.cu:986-1028):
 * forward, then the reference's argmax / temperature sampling on the device
 * with the caller's uniform draw u in [0, 1) (used when temperature > 0.01).
 * *out_id receives the selected token; best / best_logit (may be NULL) the
 * argmax and its logit, as the reference prints them. */
int gbx_model_next_token(gbx_model* m, const int32_t* ids_host, int64_t n_ids, double temperature, double u,
                         int32_t* out_id, int32_t* best, float* best_logit);

/* ShardedModel: a model replica on each of the n devices listed, one host
 * thread per device; gbx_sharded_forward splits `batch` sequences of
 * n_ids/batch tokens into contiguous shards, one per replica, and gathers
 * batch x vocab logits in order (no collective; per-shard D2H only). */
gbx_sharded* gbx_sharded_open(const char* gguf_path, const int32_t* devices, int n);
void gbx_sharded_close(gbx_sharded* s);
int gbx_sharded_forward(gbx_sharded* s, const int32_t* ids_host, int64_t n_ids, int batch, float* logits_host);

#ifdef __cplusplus
}
#endif

#endif /* GBX_MODEL_H */
