// gguf_loader.cpp -- GGUFLoader (the reference's GGUFLoader surface,
// transformer.cu:480-740) over a read-only memory map.
//
// File format (GGUF v2/v3, as the reference parses it at :567-621):
//   "GGUF" | u32 version | u64 tensor_count | u64 kv_count
//   kv_count x { string key | u32 type | value }
//   tensor_count x { string name | u32 n_dims | u64 ne[n_dims] | u32 type | u64 offset }
//   padding to the alignment (32, or general.alignment), then tensor data,
//   each tensor at data_start + offset.
// Strings are u64 length + bytes.  Value types 0..12 are u8, i8, u16, i16,
// u32, i32, f32, bool, string, array (u32 elem type, u64 count, elems), u64,
// i64, f64.  The five gpt2.* keys below are read when stored as u32, i32 or
// u64 (the reference's rule, :585-598); everything else is skipped.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <thread>

#include <cuda_runtime.h>

#include "gbx_model.hpp"

namespace gbx {

namespace {

constexpr int kDtF32 = 0, kDtF16 = 1, kDtBF16 = 30;

int elem_size(int dtype)
{
    switch (dtype) {
    case kDtF32: return 4;
    case kDtF16: return 2;
    case kDtBF16: return 2;
    default: return 0;   // quantised block types are not read (transformer.cu:647-650)
    }
}

struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;

    bool need(uint64_t n)
    {
        if (!ok || (uint64_t)(end - p) < n) ok = false;
        return ok;
    }
    template <class T>
    T get()
    {
        T v{};
        if (need(sizeof(T))) {
            std::memcpy(&v, p, sizeof(T));
            p += sizeof(T);
        }
        return v;
    }
    std::string str()
    {
        const uint64_t n = get<uint64_t>();
        if (!need(n)) return {};
        std::string s(reinterpret_cast<const char*>(p), (size_t)n);
        p += n;
        return s;
    }
    void skip(uint64_t n)
    {
        if (need(n)) p += n;
    }
};

int scalar_size(uint32_t type)
{
    switch (type) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
    }
}

bool skip_value(Reader& r, uint32_t type, int depth)
{
    if (depth > 4) return false;
    if (const int sz = scalar_size(type)) {
        r.skip(sz);
        return r.ok;
    }
    if (type == 8) {
        r.skip(r.get<uint64_t>());
        return r.ok;
    }
    if (type == 9) {
        const uint32_t et = r.get<uint32_t>();
        const uint64_t n = r.get<uint64_t>();
        if (!r.ok) return false;
        if (const int sz = scalar_size(et)) {
            if (n > (uint64_t)(r.end - r.p) / (uint64_t)sz) return false;
            r.skip(n * (uint64_t)sz);
            return r.ok;
        }
        for (uint64_t i = 0; i < n && r.ok; ++i)
            if (!skip_value(r, et, depth + 1)) return false;
        return r.ok;
    }
    return false;   // unknown type: the file cannot be walked further
}

// The reference's float16ToFloat32 (transformer.cu:508-527) as a bit
// construction: every finite half is exact in fp32; +-0 -> +0 (the sign is
// dropped, :514); any NaN -> the canonical quiet NaN 0x7fc00000 (:521).
float half_to_float_ref(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t ex = (h >> 10) & 0x1fu;
    const uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (ex == 0) {
        if (man == 0) return 0.0f;
        float v = (float)man * 5.9604644775390625e-8f;   // man * 2^-24, exact
        std::memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (ex == 31) {
        bits = man ? 0x7fc00000u : (sign | 0x7f800000u);
    } else {
        bits = sign | ((ex + 112u) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// Decode n GGUF elements to fp32 with the reference's rules, over several
// host threads for large tensors.
void decode_host(const uint8_t* src, int dtype, float* dst, int64_t n)
{
    auto part = [=](int64_t b, int64_t e) {
        if (dtype == kDtF32) {
            std::memcpy(dst + b, src + 4 * b, (size_t)(e - b) * 4);
        } else if (dtype == kDtF16) {
            for (int64_t i = b; i < e; ++i) {
                uint16_t h;
                std::memcpy(&h, src + 2 * i, 2);
                dst[i] = half_to_float_ref(h);
            }
        } else {
            for (int64_t i = b; i < e; ++i) {
                uint16_t h;
                std::memcpy(&h, src + 2 * i, 2);
                const uint32_t bits = (uint32_t)h << 16;
                std::memcpy(dst + i, &bits, 4);
            }
        }
    };
    const int64_t kPerThread = 1 << 22;
    unsigned nt = std::thread::hardware_concurrency();
    if (nt > 16) nt = 16;
    if (n < 2 * kPerThread || nt < 2) {
        part(0, n);
        return;
    }
    std::vector<std::thread> th;
    for (unsigned t = 0; t < nt; ++t) th.emplace_back(part, n * t / nt, n * (t + 1) / nt);
    for (auto& x : th) x.join();
}

}  // namespace

GGUFLoader::GGUFLoader() = default;

GGUFLoader::~GGUFLoader()
{
    freeGPUMemory();
    if (map_) munmap(const_cast<uint8_t*>(map_), mapSize_);
    if (fd_ >= 0) close(fd_);
}

bool GGUFLoader::fail(const std::string& msg)
{
    err_ = msg;
    return false;
}

bool GGUFLoader::loadFromFile(const std::string& fname)
{
    if (map_) return fail("loadFromFile: a file is already loaded");
    filename_ = fname;
    fd_ = open(fname.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd_ < 0) return fail("Failed to open GGUF file: " + fname);
    struct stat st;
    if (fstat(fd_, &st) != 0 || st.st_size < 24) return fail("GGUF file too short: " + fname);
    mapSize_ = (size_t)st.st_size;
    void* m = mmap(nullptr, mapSize_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (m == MAP_FAILED) {
        map_ = nullptr;
        return fail("mmap failed: " + fname);
    }
    map_ = static_cast<const uint8_t*>(m);
    if (!parse()) return false;
    loaded_ = true;
    return true;
}

bool GGUFLoader::parse()
{
    Reader r{map_, map_ + mapSize_};
    if (std::memcmp(map_, "GGUF", 4) != 0) return fail("Invalid GGUF magic");
    r.skip(4);
    const uint32_t version = r.get<uint32_t>();
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    if (!r.ok || version < 2) return fail("unsupported GGUF version " + std::to_string(version));
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv; ++i) {
        const std::string key = r.str();
        const uint32_t type = r.get<uint32_t>();
        if (!r.ok) return fail("truncated GGUF metadata");
        int* target = nullptr;
        if (key == "gpt2.embedding_length") target = &cfg_.embedDim;
        else if (key == "gpt2.block_count") target = &cfg_.numLayers;
        else if (key == "gpt2.attention.head_count") target = &cfg_.numHeads;
        else if (key == "gpt2.feed_forward_length") target = &cfg_.ffnDim;
        else if (key == "gpt2.context_length") target = &cfg_.maxSeqLen;
        if (target && (type == 4 || type == 5 || type == 10)) {
            *target = type == 10 ? (int)r.get<uint64_t>() : (int)r.get<uint32_t>();
        } else if (key == "general.alignment" && type == 4) {
            alignment = r.get<uint32_t>();
            if (alignment == 0 || (alignment & (alignment - 1))) return fail("bad general.alignment");
        } else if (!skip_value(r, type, 0)) {
            return fail("malformed GGUF metadata value for key '" + key + "'");
        }
    }
    if (n_tensors > (uint64_t)(r.end - r.p) / 24) return fail("GGUF tensor count exceeds the file");
    tensors_.resize((size_t)n_tensors);
    for (uint64_t i = 0; i < n_tensors; ++i) {
        GGUFTensor& t = tensors_[(size_t)i];
        t.name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (!r.ok || nd > 8) return fail("malformed GGUF tensor info");
        t.numDims = (int)nd;
        t.shape.resize(nd);
        int64_t ne = 1;
        for (uint32_t k = 0; k < nd; ++k) {
            const uint64_t v = r.get<uint64_t>();
            if (v > (uint64_t)INT64_MAX || (v && (uint64_t)ne > (uint64_t)INT64_MAX / v))
                return fail("GGUF tensor dimension overflow: " + t.name);
            t.shape[k] = (int64_t)v;
            ne *= (int64_t)v;
        }
        t.numElements = ne;
        t.dtype = (int)r.get<uint32_t>();
        t.dataOffset = (int64_t)r.get<uint64_t>();
        if (!r.ok) return fail("truncated GGUF tensor info");
        tensorMap_[t.name] = (size_t)i;
    }
    const uint64_t pos = (uint64_t)(r.p - map_);
    tensorDataStart_ = (int64_t)((pos + alignment - 1) / alignment * alignment);
    return true;
}

bool GGUFLoader::tensorBytes(const GGUFTensor& t, const uint8_t** p, int64_t* nbytes)
{
    const int es = elem_size(t.dtype);
    if (!es) return fail("Unsupported dtype " + std::to_string(t.dtype) + " for tensor " + t.name);
    if (t.numElements > INT64_MAX / es) return fail("tensor too large: " + t.name);
    const int64_t nb = t.numElements * es;
    const uint64_t start = (uint64_t)tensorDataStart_ + (uint64_t)t.dataOffset;
    if (t.dataOffset < 0 || start > mapSize_ || (uint64_t)nb > mapSize_ - start)
        return fail("tensor data outside the file: " + t.name);
    *p = map_ + start;
    *nbytes = nb;
    return true;
}

const GGUFTensor* GGUFLoader::findTensor(const std::vector<std::string>& names) const
{
    for (const auto& n : names) {
        auto it = tensorMap_.find(n);
        if (it != tensorMap_.end()) return &tensors_[it->second];
    }
    return nullptr;
}

bool GGUFLoader::hasTensor(const std::string& name) const { return tensorMap_.count(name) != 0; }

std::vector<float> GGUFLoader::getTensor(const std::vector<std::string>& names)
{
    // transformer.cu:697-706: the first name whose tensor loads wins; a
    // tensor that fails to load passes on to the next alias.
    for (const auto& n : names) {
        auto it = tensorMap_.find(n);
        if (it == tensorMap_.end()) continue;
        const GGUFTensor& t = tensors_[it->second];
        const uint8_t* p;
        int64_t nb;
        if (!tensorBytes(t, &p, &nb)) continue;
        std::vector<float> out((size_t)t.numElements);
        decode_host(p, t.dtype, out.data(), t.numElements);
        return out;
    }
    return {};
}

bool GGUFLoader::upload(const void* host, int64_t nbytes, void** dev)
{
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) return fail("cudaGetDevice failed");
    if (device_ < 0) device_ = d;
    if (d != device_) return fail("GGUFLoader: tensors already live on device " + std::to_string(device_));
    void* p = nullptr;
    if (cudaMalloc(&p, nbytes > 0 ? (size_t)nbytes : 16) != cudaSuccess) {
        cudaGetLastError();
        return fail("cudaMalloc of " + std::to_string(nbytes) + " bytes failed");
    }
    const int64_t kChunk = 32ll << 20;
    bool ok = true;
    if (nbytes <= kChunk) {
        ok = cudaMemcpy(p, host, (size_t)nbytes, cudaMemcpyHostToDevice) == cudaSuccess;
    } else {
        // Two pinned staging buffers: the copy out of the (page-faulting)
        // file map into one overlaps the DMA of the other.
        void* stage[2] = {nullptr, nullptr};
        cudaEvent_t done[2] = {nullptr, nullptr};
        cudaStream_t s = nullptr;
        ok = cudaHostAlloc(&stage[0], kChunk, cudaHostAllocDefault) == cudaSuccess &&
             cudaHostAlloc(&stage[1], kChunk, cudaHostAllocDefault) == cudaSuccess &&
             cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming) == cudaSuccess &&
             cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess;
        for (int64_t off = 0, i = 0; ok && off < nbytes; off += kChunk, ++i) {
            const int b = (int)(i & 1);
            const int64_t n = nbytes - off < kChunk ? nbytes - off : kChunk;
            if (i >= 2) ok = cudaEventSynchronize(done[b]) == cudaSuccess;
            if (!ok) break;
            std::memcpy(stage[b], static_cast<const uint8_t*>(host) + off, (size_t)n);
            ok = cudaMemcpyAsync(static_cast<uint8_t*>(p) + off, stage[b], (size_t)n, cudaMemcpyHostToDevice, s) ==
                     cudaSuccess &&
                 cudaEventRecord(done[b], s) == cudaSuccess;
        }
        if (s) ok = (cudaStreamSynchronize(s) == cudaSuccess) && ok;
        for (int b = 0; b < 2; ++b) {
            if (done[b]) cudaEventDestroy(done[b]);
            if (stage[b]) cudaFreeHost(stage[b]);
        }
        if (s) cudaStreamDestroy(s);
    }
    if (!ok) {
        cudaGetLastError();
        cudaFree(p);
        return fail("host-to-device copy failed");
    }
    *dev = p;
    return true;
}

const void* GGUFLoader::getTensorGPURaw(const std::vector<std::string>& names, int* dtype, int64_t* numElements)
{
    for (const auto& n : names) {
        auto it = tensorMap_.find(n);
        if (it == tensorMap_.end()) continue;
        GGUFTensor& t = tensors_[it->second];
        if (dtype) *dtype = t.dtype;
        if (numElements) *numElements = t.numElements;
        if (t.dtype == kDtF32 && t.d_data) return t.d_data;
        if (t.d_raw) return t.d_raw;
        const uint8_t* p;
        int64_t nb;
        if (!tensorBytes(t, &p, &nb)) return nullptr;
        void* dev = nullptr;
        if (!upload(p, nb, &dev)) return nullptr;
        if (t.dtype == kDtF32) t.d_data = static_cast<float*>(dev);
        else t.d_raw = dev;
        return dev;
    }
    fail("no tensor named " + (names.empty() ? std::string("<none>") : names[0]));
    return nullptr;
}

float* GGUFLoader::getTensorGPU(const std::vector<std::string>& names)
{
    // transformer.cu:676-695: the first name present decides (cached fp32 copy).
    for (const auto& n : names) {
        auto it = tensorMap_.find(n);
        if (it == tensorMap_.end()) continue;
        GGUFTensor& t = tensors_[it->second];
        if (t.d_data) return t.d_data;
        if (t.dtype == kDtF32) return static_cast<float*>(const_cast<void*>(getTensorGPURaw({n})));
        const uint8_t* p;
        int64_t nb;
        if (!tensorBytes(t, &p, &nb)) return nullptr;
        void* raw = t.d_raw;
        bool temp = false;
        if (!raw) {
            if (!upload(p, nb, &raw)) return nullptr;
            temp = true;
        }
        float* f = nullptr;
        if (cudaMalloc(&f, (size_t)t.numElements * sizeof(float) + 16) != cudaSuccess) {
            cudaGetLastError();
            if (temp) cudaFree(raw);
            fail("cudaMalloc failed for " + t.name);
            return nullptr;
        }
        int rc = gbx_dequant(raw, t.dtype, f, t.numElements, nullptr);
        if (rc == GBX_OK && cudaStreamSynchronize(nullptr) != cudaSuccess) rc = GBX_ECUDA;
        if (temp) cudaFree(raw);
        if (rc != GBX_OK) {
            cudaFree(f);
            fail(std::string("dequant failed: ") + gbx_last_error());
            return nullptr;
        }
        t.d_data = f;
        return f;
    }
    return nullptr;
}

void GGUFLoader::printAllTensorNames() const
{
    std::printf("\n=== All Tensor Names ===\n");
    for (const auto& t : tensors_) {
        std::printf("%s [", t.name.c_str());
        for (size_t i = 0; i < t.shape.size(); ++i) std::printf("%s%lld", i ? ", " : "", (long long)t.shape[i]);
        std::printf("] dtype=%d\n", t.dtype);
    }
}

void GGUFLoader::freeGPUMemory()
{
    int cur = -1;
    const bool switch_dev = device_ >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != device_;
    if (switch_dev) cudaSetDevice(device_);
    for (auto& t : tensors_) {
        if (t.d_data) cudaFree(t.d_data);
        if (t.d_raw) cudaFree(t.d_raw);
        t.d_data = nullptr;
        t.d_raw = nullptr;
    }
    if (switch_dev) cudaSetDevice(cur);
}

}  // namespace gbx
