// model_store.cuh — .qraf model files on the device: qraf_cuda_model_*.
//
// Included once, at the end of capi.cu (it uses that file's error reporting).
// A .qraf file (the reference's format, include/qraf/format.h) is mapped
// read-only, checked as the reference's loader checks it (validate_header,
// src/qraf/header.cpp:8-55, and the per-tensor bounds of
// QrafModel::parse_tensor_directory, src/qraf/loader.cpp:178-211) plus the
// bounds of every section and string this reader touches, all before any device
// work; then every Q8_0 / Q4_0 tensor is copied into ONE device allocation,
// each tensor at a 256-byte boundary, through two pinned staging buffers (the
// host fills one while the copy engine drains the other).  The mapping is
// dropped after the upload: weights are immutable model data, so the device
// copy is the only one the matvec needs.  F32 tensors (norms, embeddings,
// biases) stay with the caller's own loader, unless qraf_cuda_model_open_ex is
// given QRAF_MODEL_F32: then they join the same allocation (the decode engine's
// model).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <unordered_map>
#include <unordered_set>

namespace {

// The on-disk structures (include/qraf/format.h:26-131): plain little-endian PODs.
struct FileHeader {
    uint32_t magic, version;
    uint64_t file_size, config_offset, config_size, tokenizer_offset, tokenizer_size, tensor_dir_offset,
        tensor_dir_size, quant_dir_offset, quant_dir_size, string_table_offset, string_table_size, data_offset;
    uint32_t num_tensors, num_quant_schemes, flags, padding;
    uint8_t reserved[8];
};
struct FileTensorMeta {
    uint64_t name_hash;
    uint32_t name_offset, ndim, shape[8], dtype, quant_scheme_id;
    uint64_t data_offset, data_size;
    uint32_t layout_id, padding;
};
struct FileQuantScheme {
    uint32_t id, type, block_size, group_size;
    float scale, zero_point;
    uint32_t flags, padding;
};
struct FileConfigEntry {
    uint32_t key_offset, value_type, value;
};
static_assert(sizeof(FileHeader) == 128 && sizeof(FileTensorMeta) == 80 && sizeof(FileQuantScheme) == 32 &&
                  sizeof(FileConfigEntry) == 12,
              "the .qraf structures have fixed sizes");
constexpr uint32_t kQrafMagic = 0x46415251u;   // "QRAF"
constexpr uint32_t kNoQuant = 0xFFFFFFFFu;
constexpr uint64_t kStoreAlign = 256;
constexpr size_t kStagingBytes = size_t(32) << 20;

// The file mapped read-only for the duration of qraf_cuda_model_open.
struct Mapping {
    int fd = -1;
    void* base = nullptr;
    uint64_t size = 0;
    ~Mapping() {
        if (base) munmap(base, size);
        if (fd >= 0) close(fd);
    }
    const uint8_t* at(uint64_t off) const { return static_cast<const uint8_t*>(base) + off; }
};

bool in_file(uint64_t off, uint64_t len, uint64_t size) { return off <= size && len <= size - off; }

constexpr uint32_t kFileDtypeF32 = 0;   // DType::F32 (include/core/types.h)

// One tensor of the file and its place in the device allocation: a quantized
// weight, or (dtype F32) `count` floats.
struct StorePlace {
    std::string name;
    uint32_t dtype, bs, rows, cols;
    uint64_t file_off, bytes, dev_off, count;
};

// Copy every place's bytes from the mapping to base + dev_off through two
// pinned staging buffers on a stream of its own.
cudaError_t upload_places(const Mapping& mp, const std::vector<StorePlace>& places, uint8_t* base) {
    uint8_t* stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    bool used[2] = {false, false};
    cudaStream_t st = nullptr;
    cudaError_t e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
        e = cudaHostAlloc(reinterpret_cast<void**>(&stage[b]), kStagingBytes, cudaHostAllocDefault);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming);
    }
    int b = 0;
    for (size_t i = 0; i < places.size() && e == cudaSuccess; ++i) {
        const StorePlace& pl = places[i];
        for (uint64_t o = 0; o < pl.bytes && e == cudaSuccess; o += kStagingBytes) {
            const size_t n = static_cast<size_t>(std::min<uint64_t>(kStagingBytes, pl.bytes - o));
            if (used[b]) e = cudaEventSynchronize(done[b]);   // the copy that last read this buffer
            if (e != cudaSuccess) break;
            std::memcpy(stage[b], mp.at(pl.file_off + o), n);
            e = cudaMemcpyAsync(base + pl.dev_off + o, stage[b], n, cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess) e = cudaEventRecord(done[b], st);
            used[b] = true;
            b ^= 1;
        }
    }
    if (st) {
        const cudaError_t s = cudaStreamSynchronize(st);
        if (e == cudaSuccess) e = s;
    }
    for (int k = 0; k < 2; ++k) {
        if (stage[k]) cudaFreeHost(stage[k]);
        if (done[k]) cudaEventDestroy(done[k]);
    }
    if (st) cudaStreamDestroy(st);
    return e;
}

}  // namespace

struct qraf_model {
    int device = 0;
    void* base = nullptr;          // one device allocation holding every quantized tensor
    uint64_t device_bytes = 0;
    std::vector<std::string> names;                         // quantized tensors, directory order
    std::unordered_map<std::string, qraf_weight_t> weights;
    std::unordered_map<std::string, uint32_t> config;       // u32 and f32 (raw bits) entries
    std::unordered_map<std::string, std::string> config_str;   // string entries
    std::unordered_map<std::string, std::pair<const float*, uint64_t>> f32;   // QRAF_MODEL_F32: device floats
};

extern "C" {

int qraf_cuda_model_open_ex(const char* path, uint32_t flags, qraf_model_t* out) {
    if (!path || !out) return fail(QRAF_ERR_INVALID, "path or out is NULL");
    *out = nullptr;
    if (flags & ~static_cast<uint32_t>(QRAF_MODEL_F32)) return fail(QRAF_ERR_INVALID, "unknown flags 0x%x", flags);
    const bool want_f32 = (flags & QRAF_MODEL_F32) != 0;
    Mapping mp;
    mp.fd = open(path, O_RDONLY);
    if (mp.fd < 0) return fail(QRAF_ERR_INVALID, "cannot open %s", path);
    struct stat st;
    if (fstat(mp.fd, &st) != 0) return fail(QRAF_ERR_INVALID, "cannot stat %s", path);
    mp.size = static_cast<uint64_t>(st.st_size);
    if (mp.size < sizeof(FileHeader))
        return fail(QRAF_ERR_INVALID, "%s: %llu bytes, too small for a .qraf header", path,
                    static_cast<unsigned long long>(mp.size));
    mp.base = mmap(nullptr, mp.size, PROT_READ, MAP_PRIVATE, mp.fd, 0);
    if (mp.base == MAP_FAILED) {
        mp.base = nullptr;
        return fail(QRAF_ERR_INVALID, "cannot map %s", path);
    }
    FileHeader h;
    std::memcpy(&h, mp.base, sizeof(h));
    // validate_header (header.cpp:8-55), then the sections this reader reads
    if (h.magic != kQrafMagic) return fail(QRAF_ERR_INVALID, "%s: bad magic 0x%08x", path, h.magic);
    if (h.version != 1) return fail(QRAF_ERR_INVALID, "%s: unsupported version %u", path, h.version);
    if (h.file_size != mp.size)
        return fail(QRAF_ERR_INVALID, "%s: header says %llu bytes, the file has %llu", path,
                    static_cast<unsigned long long>(h.file_size), static_cast<unsigned long long>(mp.size));
    if (!in_file(h.config_offset, h.config_size, mp.size) ||
        !in_file(h.tensor_dir_offset, h.tensor_dir_size, mp.size) || h.data_offset > mp.size ||
        !in_file(h.quant_dir_offset, h.quant_dir_size, mp.size) ||
        !in_file(h.string_table_offset, h.string_table_size, mp.size))
        return fail(QRAF_ERR_INVALID, "%s: a section extends past the end of the file", path);
    if (h.tensor_dir_size != static_cast<uint64_t>(h.num_tensors) * sizeof(FileTensorMeta))
        return fail(QRAF_ERR_INVALID, "%s: tensor directory of %llu bytes for %u tensors", path,
                    static_cast<unsigned long long>(h.tensor_dir_size), h.num_tensors);
    if (h.quant_dir_size < static_cast<uint64_t>(h.num_quant_schemes) * sizeof(FileQuantScheme))
        return fail(QRAF_ERR_INVALID, "%s: quant directory too small for %u schemes", path, h.num_quant_schemes);
    // a string of the table, bounded by the table's end
    auto string_at = [&](uint32_t off, std::string* s) -> bool {
        if (off >= h.string_table_size) return false;
        const char* p = reinterpret_cast<const char*>(mp.at(h.string_table_offset + off));
        const size_t n = strnlen(p, h.string_table_size - off);
        if (n == h.string_table_size - off) return false;   // no terminator inside the table
        s->assign(p, n);
        return true;
    };

    std::unique_ptr<qraf_model> m(new qraf_model());
    if (h.config_size >= 4) {
        uint32_t n = 0;
        std::memcpy(&n, mp.at(h.config_offset), 4);
        if (4 + static_cast<uint64_t>(n) * sizeof(FileConfigEntry) > h.config_size)
            return fail(QRAF_ERR_INVALID, "%s: config block too small for %u entries", path, n);
        for (uint32_t i = 0; i < n; ++i) {
            FileConfigEntry e;
            std::memcpy(&e, mp.at(h.config_offset + 4 + static_cast<uint64_t>(i) * sizeof(e)), sizeof(e));
            std::string key;
            if (!string_at(e.key_offset, &key))
                return fail(QRAF_ERR_INVALID, "%s: config key %u out of range", path, i);
            if (e.value_type <= 1) {
                m->config[key] = e.value;
            } else if (e.value_type == 2) {
                std::string v;
                if (!string_at(e.value, &v))
                    return fail(QRAF_ERR_INVALID, "%s: config string '%s' out of range", path, key.c_str());
                m->config_str[key] = v;
            }
        }
    }

    std::vector<StorePlace> places;
    std::unordered_set<std::string> seen;
    uint64_t total = 0;
    for (uint32_t i = 0; i < h.num_tensors; ++i) {
        FileTensorMeta t;
        std::memcpy(&t, mp.at(h.tensor_dir_offset + static_cast<uint64_t>(i) * sizeof(t)), sizeof(t));
        std::string name;
        if (!string_at(t.name_offset, &name)) return fail(QRAF_ERR_INVALID, "%s: tensor %u has no name", path, i);
        if (!in_file(t.data_offset, t.data_size, mp.size))
            return fail(QRAF_ERR_INVALID, "%s: tensor '%s' data extends past the end of the file", path, name.c_str());
        const bool is_f32 = want_f32 && t.dtype == kFileDtypeF32;
        if (!known_dtype(t.dtype) && !is_f32) continue;
        if (t.ndim == 0 || t.ndim > 8)
            return fail(QRAF_ERR_INVALID, "%s: tensor '%s' has ndim %u", path, name.c_str(), t.ndim);
        if (is_f32) {
            uint64_t count = 1;
            for (uint32_t d = 0; d < t.ndim; ++d) count *= t.shape[d];
            if (count > (uint64_t(1) << 40) || t.data_size < count * 4)
                return fail(QRAF_ERR_INVALID, "%s: F32 tensor '%s' holds %llu bytes, its shape needs %llu", path,
                            name.c_str(), static_cast<unsigned long long>(t.data_size),
                            static_cast<unsigned long long>(count * 4));
            if (!seen.insert(name).second)
                return fail(QRAF_ERR_INVALID, "%s: tensor '%s' appears twice", path, name.c_str());
            StorePlace pl{name, kFileDtypeF32, 0, 0, 0, t.data_offset, count * 4, 0, count};
            total = (total + kStoreAlign - 1) / kStoreAlign * kStoreAlign;
            pl.dev_off = total;
            total += pl.bytes;
            places.push_back(pl);
            continue;
        }
        // rows = the product of the leading dimensions, cols = the last (row-major,
        // layout_id 0; a weight is [out_dim][in_dim])
        uint64_t rows = 1;
        for (uint32_t d = 0; d + 1 < t.ndim; ++d) rows *= t.shape[d];
        const uint32_t cols = t.shape[t.ndim - 1];
        // the scheme's block size; 32 without one, as the reference's dispatch
        // defaults a missing QuantScheme (backend.cpp:135)
        uint32_t bs = 32;
        if (t.quant_scheme_id != kNoQuant && t.quant_scheme_id < h.num_quant_schemes) {
            FileQuantScheme q;
            std::memcpy(&q, mp.at(h.quant_dir_offset + static_cast<uint64_t>(t.quant_scheme_id) * sizeof(q)),
                        sizeof(q));
            bs = q.block_size;
        }
        if (rows > 0xFFFFFFFFull) return fail(QRAF_ERR_INVALID, "%s: tensor '%s' has too many rows", path, name.c_str());
        if (bs == 0 || (t.dtype == QRAF_DTYPE_Q4_0 && bs < 2))
            return fail(QRAF_ERR_INVALID, "%s: tensor '%s' has block size %u", path, name.c_str(), bs);
        StorePlace pl{};
        pl.name = name;
        pl.dtype = t.dtype;
        pl.bs = bs;
        pl.rows = static_cast<uint32_t>(rows);
        pl.cols = cols;
        pl.bytes = qraf_row_bytes(t.dtype, bs, cols) * rows;
        if (t.data_size < pl.bytes)
            return fail(QRAF_ERR_INVALID, "%s: tensor '%s' holds %llu bytes, its shape needs %llu", path,
                        name.c_str(), static_cast<unsigned long long>(t.data_size),
                        static_cast<unsigned long long>(pl.bytes));
        if (!seen.insert(name).second)
            return fail(QRAF_ERR_INVALID, "%s: tensor '%s' appears twice", path, name.c_str());
        pl.file_off = t.data_offset;
        total = (total + kStoreAlign - 1) / kStoreAlign * kStoreAlign;
        pl.dev_off = total;
        total += pl.bytes;
        places.push_back(pl);
    }

    // device work from here on
    int rc = ensure_device(&m->device, nullptr);
    if (rc) return rc;
    if (total) {
        if (cudaMalloc(&m->base, total) != cudaSuccess) {
            cudaGetLastError();
            return fail(QRAF_ERR_NOMEM, "%s: cudaMalloc of %llu bytes for the weights failed", path,
                        static_cast<unsigned long long>(total));
        }
        m->device_bytes = total;
        const cudaError_t e = upload_places(mp, places, static_cast<uint8_t*>(m->base));
        if (e != cudaSuccess) {
            cudaGetLastError();
            cudaFree(m->base);
            return fail(QRAF_ERR_CUDA, "%s: weight upload: %s", path, cudaGetErrorString(e));
        }
    }
    for (const StorePlace& pl : places) {
        if (pl.dtype == kFileDtypeF32) {
            m->f32[pl.name] = {reinterpret_cast<const float*>(static_cast<uint8_t*>(m->base) + pl.dev_off), pl.count};
            continue;
        }
        qraf_weight_t w;
        rc = describe_weight(pl.bytes, pl.dtype, pl.bs, pl.rows, pl.cols, &w);
        if (rc) {
            cudaFree(m->base);
            return rc;
        }
        w.data = static_cast<uint8_t*>(m->base) + pl.dev_off;
        m->weights[pl.name] = w;
        m->names.push_back(pl.name);
    }
    *out = m.release();
    return QRAF_OK;
}

int qraf_cuda_model_open(const char* path, qraf_model_t* out) { return qraf_cuda_model_open_ex(path, 0, out); }

int qraf_cuda_model_tensor_f32(qraf_model_t m, const char* name, const float** data, uint64_t* count) {
    if (!m || !name || !data || !count) return fail(QRAF_ERR_INVALID, "model, name, data or count is NULL");
    auto it = m->f32.find(name);
    if (it == m->f32.end())
        return fail(QRAF_ERR_INVALID, "no F32 tensor named '%s' (open the model with QRAF_MODEL_F32)", name);
    *data = it->second.first;
    *count = it->second.second;
    return QRAF_OK;
}

int qraf_cuda_model_weight(qraf_model_t m, const char* name, qraf_weight_t* out) {
    if (!m || !name || !out) return fail(QRAF_ERR_INVALID, "model, name or out is NULL");
    auto it = m->weights.find(name);
    if (it == m->weights.end()) return fail(QRAF_ERR_INVALID, "no Q8_0 / Q4_0 tensor named '%s'", name);
    *out = it->second;
    return QRAF_OK;
}

int qraf_cuda_model_info(qraf_model_t m, uint32_t* num_weights, uint64_t* device_bytes, int* device) {
    if (!m) return fail(QRAF_ERR_INVALID, "model is NULL");
    if (num_weights) *num_weights = static_cast<uint32_t>(m->names.size());
    if (device_bytes) *device_bytes = m->device_bytes;
    if (device) *device = m->device;
    return QRAF_OK;
}

const char* qraf_cuda_model_weight_name(qraf_model_t m, uint32_t index) {
    if (!m || index >= m->names.size()) return nullptr;
    return m->names[index].c_str();
}

int qraf_cuda_model_config_u32(qraf_model_t m, const char* key, uint32_t* value) {
    if (!m || !key || !value) return fail(QRAF_ERR_INVALID, "model, key or value is NULL");
    auto it = m->config.find(key);
    if (it == m->config.end()) return fail(QRAF_ERR_INVALID, "no u32 / f32 config entry '%s'", key);
    *value = it->second;
    return QRAF_OK;
}

int qraf_cuda_model_close(qraf_model_t m) {
    if (!m) return QRAF_OK;
    cudaError_t e = cudaSuccess;
    if (m->base) {
        int cur = 0;
        cudaGetDevice(&cur);
        cudaSetDevice(m->device);
        e = cudaFree(m->base);
        cudaSetDevice(cur);
    }
    delete m;
    if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "freeing the model's weights: %s", cudaGetErrorString(e));
    return QRAF_OK;
}

}  // extern "C"
