// ref_shim.cpp — C entry points onto the reference's OWN compiled sources.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the unmodified reference sources (src/tensor/{quantize,dtype,tensor}.cpp,
// src/nn/{backend,ops,threading,attention,transformer}.cpp,
// src/core/{logging,error}.cpp, src/qraf/{loader,header,writer}.cpp, read in
// place from the reference tree) into oracle/_ref/libqraf_ref.so.  It is used
// to pin the C restatement (qraf_oracle.c), to generate the golden fixtures in
// tests/golden/, and as the timed CPU baseline.  No reference source is copied.
#include "core/types.h"
#include "nn/attention.h"
#include "nn/backend.h"
#include "nn/ops.h"
#include "nn/kv_cache_quant.h"
#include "nn/transformer.h"
#include "qraf/format.h"
#include "qraf/loader.h"
#include "qraf/writer.h"
#include "tensor/quantize.h"

#include <cstring>
#include <random>
#include <thread>
#include <vector>

using namespace qraf;

namespace qraf {
f32 fp16_to_fp32(f16 h);
f16 fp32_to_fp16(f32 f);
}

static QuantScheme make_scheme(int block_size) {
    QuantScheme qs;
    std::memset(&qs, 0, sizeof(qs));
    qs.block_size = static_cast<u32>(block_size);
    qs.flags = 1;
    return qs;
}

extern "C" {

// quantize_q8_0 / quantize_q4_0 (src/tensor/quantize.cpp:105-183).  Copies the
// returned byte vector into `out` (caller sizes it) and returns its length.
size_t qref_quantize(uint32_t dtype, const float* data, size_t count, int block_size, uint8_t* out) {
    std::vector<u8> v;
    if (dtype == static_cast<uint32_t>(DType::Q8_0)) v = quantize_q8_0(data, count, block_size);
    else if (dtype == static_cast<uint32_t>(DType::Q4_0)) v = quantize_q4_0(data, count, block_size);
    else return 0;
    if (out) std::memcpy(out, v.data(), v.size());
    return v.size();
}

// dot_q8_0_f32 / dot_q4_0_f32 (src/tensor/quantize.cpp:187-239).
float qref_dot(uint32_t dtype, const void* q, const float* x, size_t count, int block_size) {
    if (dtype == static_cast<uint32_t>(DType::Q8_0)) return dot_q8_0_f32(q, x, count, block_size);
    if (dtype == static_cast<uint32_t>(DType::Q4_0)) return dot_q4_0_f32(q, x, count, block_size);
    return 0.0f;
}

// dequantize_block_q8_0 / _q4_0 (src/tensor/quantize.cpp:17-51).
void qref_dequantize_block(uint32_t dtype, const void* block, float* out, int block_size) {
    if (dtype == static_cast<uint32_t>(DType::Q8_0)) dequantize_block_q8_0(block, out, block_size);
    else if (dtype == static_cast<uint32_t>(DType::Q4_0)) dequantize_block_q4_0(block, out, block_size);
}

// dispatch_matvec_q (src/nn/backend.cpp:131-199).  block_size <= 0 passes a
// null QuantScheme (the reference then uses 32).
void qref_dispatch_matvec_q(const void* w, uint64_t w_size, uint32_t dtype, int block_size,
                            uint32_t N, uint32_t K, const float* x, float* y) {
    QuantScheme qs = make_scheme(block_size);
    dispatch_matvec_q(w, w_size, static_cast<DType>(dtype), block_size > 0 ? &qs : nullptr,
                      N, K, x, y);
}

// ops::matvec_quantized (src/nn/ops.cpp:72-103).
void qref_ops_matvec_quantized(const void* w, uint64_t w_size, uint32_t dtype, int block_size,
                               uint32_t N, uint32_t K, const float* x, float* y) {
    QuantScheme qs = make_scheme(block_size);
    ops::matvec_quantized(w, w_size, static_cast<DType>(dtype), block_size > 0 ? &qs : nullptr,
                          N, K, x, y);
}

// The same per-row dot fanned out over `threads` host threads, rows split in
// contiguous ranges.  This mirrors the row fan-out the reference uses on its
// threaded build (parallel_for over output rows, src/nn/backend.cpp:145-151);
// each row is still the reference's own scalar dot, so results are identical.
void qref_matvec_q_threaded(const void* w, uint32_t dtype, int block_size, uint32_t N, uint32_t K,
                            const float* x, float* y, int threads) {
    if (threads <= 1) {
        qref_dispatch_matvec_q(w, 0, dtype, block_size, N, K, x, y);
        return;
    }
    const int bs = block_size > 0 ? block_size : 32;
    const size_t nb = (static_cast<size_t>(K) + bs - 1) / bs;
    const size_t rb = nb * (dtype == static_cast<uint32_t>(DType::Q8_0) ? (4u + bs) : (2u + bs / 2));
    const u8* base = static_cast<const u8*>(w);
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; t++) {
        uint32_t r0 = static_cast<uint32_t>(static_cast<uint64_t>(N) * t / threads);
        uint32_t r1 = static_cast<uint32_t>(static_cast<uint64_t>(N) * (t + 1) / threads);
        pool.emplace_back([=]() {
            for (uint32_t r = r0; r < r1; r++)
                y[r] = qref_dot(dtype, base + static_cast<size_t>(r) * rb, x, K, bs);
        });
    }
    for (auto& th : pool) th.join();
}

// mlp_forward (src/nn/attention.cpp:159-186): SwiGLU MLP of the reference with
// quantized gate/up/down weights, each projection through dispatch_matvec_q.
void qref_mlp_forward(float* out, const float* x, const void* w_gate, const void* w_up, const void* w_down,
                      uint64_t gate_bytes, uint64_t down_bytes, uint32_t dtype, int block_size, uint32_t hidden,
                      uint32_t inter) {
    static QuantScheme qs;
    qs = make_scheme(block_size);
    MLPWeights w;
    w.w_gate_data = w_gate;
    w.w_up_data = w_up;
    w.w_down_data = w_down;
    w.w_gate_size = gate_bytes;
    w.w_up_size = gate_bytes;
    w.w_down_size = down_bytes;
    w.dtype = static_cast<DType>(dtype);
    w.quant = &qs;
    ModelConfig cfg;
    cfg.hidden_size = hidden;
    cfg.intermediate_size = inter;
    mlp_forward(out, x, w, cfg);
}

// fp32_to_fp16 / fp16_to_fp32 (src/tensor/dtype.cpp:9-59).
uint16_t qref_fp32_to_fp16(float f) { return fp32_to_fp16(f); }
// ops::rms_norm_inplace (src/nn/ops.cpp:107-118), in place.
void qref_rms_norm(float* x, const float* w, int size, float eps) { ops::rms_norm_inplace(x, w, size, eps); }
float qref_fp16_to_fp32(uint16_t h) { return fp16_to_fp32(h); }

// The reference's own .qraf writer (src/qraf/writer.cpp, QrafWriter) and loader
// (src/qraf/loader.cpp, QrafModel) behind plain C handles, to pin the product's
// writer byte for byte and to read its files back with the reference's code.
void* qref_writer_new() { return new QrafWriter(); }
void qref_writer_free(void* h) { delete static_cast<QrafWriter*>(h); }
void qref_writer_config_u32(void* h, const char* key, uint32_t v) { static_cast<QrafWriter*>(h)->set_config(key, v); }
void qref_writer_config_f32(void* h, const char* key, float v) { static_cast<QrafWriter*>(h)->set_config(key, v); }
void qref_writer_config_string(void* h, const char* key, const char* v) {
    static_cast<QrafWriter*>(h)->set_config_string(key, v);
}
uint32_t qref_writer_quant_scheme(void* h, uint32_t dtype, uint32_t block_size, uint32_t group_size) {
    return static_cast<QrafWriter*>(h)->add_quant_scheme(static_cast<DType>(dtype), block_size, group_size);
}
void qref_writer_tensor(void* h, const char* name, uint32_t ndim, const uint32_t* shape, uint32_t dtype,
                        const void* data, uint64_t size, uint32_t quant_id) {
    std::vector<u32> sh(shape, shape + ndim);
    static_cast<QrafWriter*>(h)->add_tensor(name, sh, static_cast<DType>(dtype), data, size, quant_id);
}
void qref_writer_vocab(void* h, const char* const* tokens, const float* scores, uint32_t n) {
    std::vector<std::string> t(tokens, tokens + n);
    std::vector<f32> sc(scores, scores + n);
    static_cast<QrafWriter*>(h)->set_vocab(t, sc);
}
void qref_writer_merges(void* h, const uint32_t* abr, const float* priority, uint32_t n) {
    std::vector<std::tuple<u32, u32, u32, f32>> m;
    for (uint32_t i = 0; i < n; ++i) m.emplace_back(abr[3 * i], abr[3 * i + 1], abr[3 * i + 2], priority[i]);
    static_cast<QrafWriter*>(h)->set_merges(m);
}
void qref_writer_special(void* h, uint32_t bos, uint32_t eos, uint32_t pad, uint32_t unk) {
    static_cast<QrafWriter*>(h)->set_special_tokens(bos, eos, pad, unk);
}
int qref_writer_write(void* h, const char* path) { return static_cast<QrafWriter*>(h)->write(path) ? 0 : 1; }

void* qref_model_open(const char* path) {
    QrafModel* m = new QrafModel();
    if (!m->load(path)) {
        delete m;
        return nullptr;
    }
    return m;
}
void qref_model_close(void* h) { delete static_cast<QrafModel*>(h); }
// One tensor: its bytes (a view into the reference's mapping), dtype, shape and
// the block size of its quantization scheme (0 if none).  Returns 0 if found.
int qref_model_tensor(void* h, const char* name, const void** data, uint64_t* size, uint32_t* dtype,
                      uint32_t* ndim, uint32_t* shape, uint32_t* block_size) {
    QrafModel* m = static_cast<QrafModel*>(h);
    if (!m->has_tensor(name)) return 1;
    TensorView tv = m->get_tensor(name);
    *data = tv.data;
    *size = tv.data_size;
    *dtype = static_cast<uint32_t>(tv.dtype);
    *ndim = tv.ndim();
    for (uint32_t i = 0; i < tv.ndim() && i < 8; i++) shape[i] = tv.shape[i];
    *block_size = tv.quant ? tv.quant->block_size : 0;
    return 0;
}
uint32_t qref_model_hidden_size(void* h) { return static_cast<QrafModel*>(h)->config().hidden_size; }

// The reference's Transformer over a .qraf file (src/nn/transformer.cpp:
// init at :300-440, forward -> forward_llama at :573-620 for llama / qwen2):
// the decode engine's oracle.  forward() copies the logits out.
struct RefTransformer {
    QrafModel model;
    Transformer tf;
};
void* qref_transformer_open(const char* path) {
    RefTransformer* r = new RefTransformer();
    if (!r->model.load(path) || !r->tf.init(r->model)) {
        delete r;
        return nullptr;
    }
    return r;
}
void qref_transformer_close(void* h) { delete static_cast<RefTransformer*>(h); }
void qref_transformer_reset(void* h) { static_cast<RefTransformer*>(h)->tf.reset(); }
int qref_transformer_forward(void* h, uint32_t token, int pos, float* logits, uint32_t vocab) {
    Tensor t = static_cast<RefTransformer*>(h)->tf.forward(token, pos);
    if (t.numel() != vocab) return 1;
    std::memcpy(logits, t.data_f32(), vocab * sizeof(float));
    return 0;
}

// The reference's int8 KV cache (include/nn/kv_cache_quant.h): one row of K and V
// (kv_heads * head_dim floats each) stored at position 0 of a one-layer cache and
// read back as codes and per-head scales; dot_with_key for a query against it.
void qref_kvq_store(const float* k, const float* v, int kv_heads, int head_dim, int8_t* kq, int8_t* vq, float* ks,
                    float* vs) {
    QuantizedKVCache c;
    c.init(1, kv_heads, head_dim, 1);
    c.store(0, 0, k, v);
    std::memcpy(kq, c.keys_q[0].data(), static_cast<size_t>(kv_heads) * head_dim);
    std::memcpy(vq, c.values_q[0].data(), static_cast<size_t>(kv_heads) * head_dim);
    std::memcpy(ks, c.key_scales[0].data(), kv_heads * sizeof(float));
    std::memcpy(vs, c.value_scales[0].data(), kv_heads * sizeof(float));
}

// Seeded synthetic data with the reference's idiom (std::mt19937 +
// std::normal_distribution<float>, tools/dummy_model.cpp:12-16,
// benchmarks/bench_main.cpp:43-44).
void qref_fill_normal(uint32_t seed, float mean, float stddev, float* out, size_t n) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> dist(mean, stddev);
    for (size_t i = 0; i < n; i++) out[i] = dist(rng);
}

}  // extern "C"
