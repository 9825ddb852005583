/* C ABI of libnutcuda.so (include/nutllm_cuda.h).
 *
 * Owns the device images of quantised matrices and models, the per-sequence
 * KV cache and decode state, and drives the token loop on one CUDA stream
 * per model.  Every failure is reported as a nut_status plus a thread-local
 * "component: reason" message; argument checks raise the same classes, in
 * the same order, as the reference's decode_quantized_token
 * (src/quant_model.cpp:161-172) and prefill_quantized (:212-213).
 */
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/nutllm_cuda.h"
#include "kernels.h"

namespace {

thread_local std::string g_error;

struct Failure {
    nut_status status;
    std::string message;
};

[[noreturn]] void raise(nut_status s, const std::string &m) {
    throw Failure{s, m};
}

void cuda_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess)
        raise(NUT_RUNTIME_ERROR,
              std::string("cuda: ") + what + ": " + cudaGetErrorString(e));
}

template <typename F> nut_status guarded(F &&body) {
    try {
        body();
        return NUT_OK;
    } catch (const Failure &f) {
        g_error = f.message;
        return f.status;
    } catch (const std::bad_alloc &) {
        g_error = "nutllm: host allocation failed";
        return NUT_RUNTIME_ERROR;
    } catch (const std::exception &e) {
        g_error = e.what();
        return NUT_RUNTIME_ERROR;
    }
}

/* RAII device scope: makes `device` current, restores the caller's. */
struct DeviceScope {
    int previous = 0;
    explicit DeviceScope(int device) {
        cuda_check(cudaGetDevice(&previous), "get device");
        cuda_check(cudaSetDevice(device), "set device");
    }
    ~DeviceScope() { cudaSetDevice(previous); }
};

template <typename T> T *dev_alloc(size_t count, const char *what) {
    void *p = nullptr;
    if (count == 0)
        count = 1;
    cuda_check(cudaMalloc(&p, count * sizeof(T)), what);
    return static_cast<T *>(p);
}

void dev_free(void *p) {
    if (p != nullptr)
        cudaFree(p);
}

void validate_config(const nut_config &c) {
    const int64_t kv = c.kv_heads == 0 ? c.heads : c.kv_heads;
    if (c.layers <= 0 || c.heads <= 0 || c.dim <= 0 || c.head_dim <= 0 ||
        c.ffn_dim <= 0 || c.vocab_size <= 0 || c.max_seq <= 0 ||
        c.heads * c.head_dim != c.dim || c.head_dim % 2 != 0 ||
        c.eos_token < 0 || c.eos_token >= c.vocab_size || kv <= 0 ||
        kv > c.heads || c.heads % kv != 0)
        raise(NUT_INVALID_ARGUMENT, "model config: invalid dimensions");
    if (c.dim > (1 << 20) || c.ffn_dim > (1 << 20) ||
        c.vocab_size > (int64_t(1) << 30) || c.max_seq > (1 << 20) ||
        c.layers > 4096)
        raise(NUT_LENGTH_ERROR, "model config: dimensions exceed device limits");
}

nut::DevQMatrix upload(const nut_qmatrix_view &v, int64_t rows, int64_t cols,
                       int type, const char *name) {
    if (v.data == nullptr || v.scales == nullptr)
        raise(NUT_INVALID_ARGUMENT, std::string("model: null storage for ") + name);
    if (v.rows != rows || v.cols != cols)
        raise(NUT_INVALID_ARGUMENT,
              std::string("quantized decode: shape mismatch for ") + name);
    if (v.block_size != 32)
        raise(NUT_INVALID_ARGUMENT, "quantized matrix: block size must be 32");
    if (v.type != type)
        raise(NUT_INVALID_ARGUMENT,
              std::string("quantized decode: quant type mismatch for ") + name);
    nut::DevQMatrix m;
    m.rows = rows;
    m.cols = cols;
    m.type = type;
    m.data = dev_alloc<uint8_t>(m.data_bytes(), "alloc weights");
    m.scales = dev_alloc<uint16_t>(m.scale_count(), "alloc scales");
    cuda_check(cudaMemcpy(m.data, v.data, m.data_bytes(), cudaMemcpyHostToDevice),
               "copy weights");
    cuda_check(cudaMemcpy(m.scales, v.scales, m.scale_count() * 2,
                          cudaMemcpyHostToDevice),
               "copy scales");
    return m;
}

void release(nut::DevQMatrix &m) {
    dev_free(m.data);
    dev_free(m.scales);
    m.data = nullptr;
    m.scales = nullptr;
}

nut::QSeg seg(const nut::DevQMatrix &m, float *out, int accumulate) {
    return nut::QSeg{m.data, m.scales, int(m.rows), out, accumulate};
}

} // namespace

struct nut_qmatrix {
    int device = 0;
    nut::DevQMatrix m;
    float *x = nullptr, *y = nullptr; /* staging for host-buffer calls */
    cudaStream_t stream = nullptr;
    ~nut_qmatrix() {
        if (stream) {
            cudaStreamSynchronize(stream);
            cudaStreamDestroy(stream);
        }
        release(m);
        dev_free(x);
        dev_free(y);
    }
};

struct DevLayer {
    nut::DevQMatrix q, k, v, o, gate, up, down;
    float *attention_norm = nullptr, *ffn_norm = nullptr;
};

struct nut_model {
    int device = 0;
    nut_config cfg{};
    int64_t kv_heads = 0;
    int type = 0;
    bool tied = false;
    float *embeddings = nullptr, *final_norm = nullptr, *lm_head = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr; /* [max_seq][hd/2] */
    std::vector<DevLayer> layers;
    uint64_t storage_bytes = 0;
    cudaStream_t stream = nullptr;
    ~nut_model() {
        if (stream) {
            cudaStreamSynchronize(stream);
            cudaStreamDestroy(stream);
        }
        for (auto &l : layers) {
            release(l.q), release(l.k), release(l.v), release(l.o);
            release(l.gate), release(l.up), release(l.down);
            dev_free(l.attention_norm), dev_free(l.ffn_norm);
        }
        dev_free(embeddings), dev_free(final_norm), dev_free(lm_head);
        dev_free(rope_cos), dev_free(rope_sin);
    }
    const float *output_weights() const { return tied ? embeddings : lm_head; }
};

struct nut_kv {
    nut_model *model = nullptr;
    int64_t length = 0;
    float *keys = nullptr, *values = nullptr; /* [L][kvh][max_seq][hd] */
    float *hidden = nullptr;                 /* [dim] last hidden */
    float *q = nullptr, *k = nullptr, *v = nullptr, *ctx = nullptr;
    float *gate = nullptr, *up = nullptr, *logits = nullptr;
    unsigned long long *argmax_key = nullptr;
    int32_t *ids = nullptr; /* [max_seq] generated ids */
    bool has_hidden = false;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    ~nut_kv() {
        if (model)
            cudaStreamSynchronize(model->stream);
        dev_free(keys), dev_free(values), dev_free(hidden), dev_free(q);
        dev_free(k), dev_free(v), dev_free(ctx), dev_free(gate), dev_free(up);
        dev_free(logits), dev_free(argmax_key), dev_free(ids);
        for (auto e : ev)
            if (e)
                cudaEventDestroy(e);
    }
    size_t cache_elements() const {
        const nut_config &c = model->cfg;
        return size_t(c.layers) * model->kv_heads * c.max_seq * c.head_dim;
    }
};

namespace {

/* One token through every layer at position kv->length; token < 0 reads
 * the previous argmax from the device (the greedy loop) and records it in
 * ids[id_index]. */
void enqueue_decode(nut_model *m, nut_kv *kv, int token, int id_index) {
    const nut_config &c = m->cfg;
    cudaStream_t s = m->stream;
    const int pos = int(kv->length);
    const int dim = int(c.dim), hd = int(c.head_dim), H = int(c.heads);
    const int KVH = int(m->kv_heads), S = int(c.max_seq);
    nut::launch_embed(m->embeddings, dim, int(c.vocab_size), token,
                      kv->argmax_key,
                      token < 0 ? kv->ids + id_index : nullptr, kv->hidden, s);
    for (int l = 0; l < int(c.layers); l++) {
        const DevLayer &w = m->layers[size_t(l)];
        nut::QSegs qkv{};
        qkv.seg[0] = seg(w.q, kv->q, 0);
        qkv.seg[1] = seg(w.k, kv->k, 0);
        qkv.seg[2] = seg(w.v, kv->v, 0);
        qkv.count = 3;
        qkv.cols = dim;
        qkv.type = m->type;
        nut::launch_qmatvec(qkv, kv->hidden, w.attention_norm, s);
        nut::launch_rope_store(kv->q, kv->k, kv->v, kv->keys, kv->values,
                               m->rope_cos, m->rope_sin, pos, l, H, KVH, hd,
                               S, s);
        nut::launch_attention(kv->q, kv->keys, kv->values, kv->ctx, pos, l, H,
                              KVH, hd, S, s);
        nut::QSegs wo{};
        wo.seg[0] = seg(w.o, kv->hidden, 1);
        wo.count = 1;
        wo.cols = dim;
        wo.type = m->type;
        nut::launch_qmatvec(wo, kv->ctx, nullptr, s);
        nut::QSegs gu{};
        gu.seg[0] = seg(w.gate, kv->gate, 0);
        gu.seg[1] = seg(w.up, kv->up, 0);
        gu.count = 2;
        gu.cols = dim;
        gu.type = m->type;
        nut::launch_qmatvec(gu, kv->hidden, w.ffn_norm, s);
        nut::launch_swiglu(kv->gate, kv->up, int(c.ffn_dim), s);
        nut::QSegs dn{};
        dn.seg[0] = seg(w.down, kv->hidden, 1);
        dn.count = 1;
        dn.cols = int(c.ffn_dim);
        dn.type = m->type;
        nut::launch_qmatvec(dn, kv->gate, nullptr, s);
    }
    cuda_check(cudaGetLastError(), "decode launch");
    kv->length++;
    kv->has_hidden = true;
}

void enqueue_logits(nut_model *m, nut_kv *kv) {
    cuda_check(cudaMemsetAsync(kv->argmax_key, 0, sizeof(unsigned long long),
                               m->stream),
               "reset argmax");
    nut::launch_lmhead(kv->hidden, m->final_norm, m->output_weights(),
                       int(m->cfg.vocab_size), int(m->cfg.dim), kv->logits,
                       kv->argmax_key, m->stream);
    cuda_check(cudaGetLastError(), "lm_head launch");
}

void check_decode_args(nut_model *m, nut_kv *kv, int64_t token) {
    if (m == nullptr || kv == nullptr)
        raise(NUT_INVALID_ARGUMENT, "quantized decode: null handle");
    if (kv->model != m)
        raise(NUT_INVALID_ARGUMENT, "quantized decode: cache configuration mismatch");
    if (token < 0 || token >= m->cfg.vocab_size)
        raise(NUT_OUT_OF_RANGE, "quantized decode: token out of range");
    if (kv->length >= m->cfg.max_seq)
        raise(NUT_LENGTH_ERROR, "quantized decode: context is full");
}

void sync(nut_model *m) { cuda_check(cudaStreamSynchronize(m->stream), "synchronize"); }

} // namespace

extern "C" {

const char *nut_last_error(void) { return g_error.c_str(); }

nut_status nut_device_count(int *count) {
    return guarded([&] {
        if (count == nullptr)
            raise(NUT_INVALID_ARGUMENT, "device: null output");
        cuda_check(cudaGetDeviceCount(count), "device count");
    });
}

nut_status nut_qmatrix_create(const nut_qmatrix_view *view, int device,
                              nut_qmatrix **out) {
    return guarded([&] {
        if (view == nullptr || out == nullptr)
            raise(NUT_INVALID_ARGUMENT, "quantized matrix: null argument");
        if (view->rows <= 0 || view->cols <= 0)
            raise(NUT_INVALID_ARGUMENT, "quantize: invalid dimensions");
        if (view->type != NUT_QUANT_INT8 && view->type != NUT_QUANT_INT4)
            raise(NUT_INVALID_ARGUMENT, "quantized matrix: unknown type");
        if (view->rows > (int64_t(1) << 30) || view->cols > (int64_t(1) << 24))
            raise(NUT_LENGTH_ERROR, "quantized matrix: dimensions exceed device limits");
        DeviceScope scope(device);
        auto q = std::make_unique<nut_qmatrix>();
        q->device = device;
        q->m = upload(*view, view->rows, view->cols, view->type, "matrix");
        q->x = dev_alloc<float>(size_t(view->cols), "alloc x");
        q->y = dev_alloc<float>(size_t(view->rows), "alloc y");
        cuda_check(cudaStreamCreateWithFlags(&q->stream, cudaStreamNonBlocking),
                   "create stream");
        *out = q.release();
    });
}

nut_status nut_qmatrix_destroy(nut_qmatrix *matrix) {
    return guarded([&] {
        if (matrix == nullptr)
            return;
        DeviceScope scope(matrix->device);
        delete matrix;
    });
}

nut_status nut_qmatrix_download(const nut_qmatrix *matrix, uint8_t *data,
                                uint16_t *scales) {
    return guarded([&] {
        if (matrix == nullptr || data == nullptr || scales == nullptr)
            raise(NUT_INVALID_ARGUMENT, "quantized matrix: null argument");
        DeviceScope scope(matrix->device);
        cuda_check(cudaMemcpy(data, matrix->m.data, matrix->m.data_bytes(),
                              cudaMemcpyDeviceToHost),
                   "download weights");
        cuda_check(cudaMemcpy(scales, matrix->m.scales, matrix->m.scale_count() * 2,
                              cudaMemcpyDeviceToHost),
                   "download scales");
    });
}

nut_status nut_qmatvec_async(nut_qmatrix *matrix, const float *x_device,
                             float *y_device, void *stream) {
    return guarded([&] {
        if (matrix == nullptr || x_device == nullptr || y_device == nullptr)
            raise(NUT_INVALID_ARGUMENT, "quantized matvec: null pointer");
        DeviceScope scope(matrix->device);
        nut::QSegs s{};
        s.seg[0] = seg(matrix->m, y_device, 0);
        s.count = 1;
        s.cols = int(matrix->m.cols);
        s.type = matrix->m.type;
        nut::launch_qmatvec(s, x_device, nullptr,
                            static_cast<cudaStream_t>(stream));
        cuda_check(cudaGetLastError(), "qmatvec launch");
    });
}

nut_status nut_qmatvec(nut_qmatrix *matrix, const float *x, float *y) {
    return guarded([&] {
        if (matrix == nullptr || x == nullptr || y == nullptr)
            raise(NUT_INVALID_ARGUMENT, "quantized matvec: null pointer");
        DeviceScope scope(matrix->device);
        const size_t cols = size_t(matrix->m.cols), rows = size_t(matrix->m.rows);
        cuda_check(cudaMemcpyAsync(matrix->x, x, cols * 4, cudaMemcpyHostToDevice,
                                   matrix->stream),
                   "copy x");
        nut::QSegs s{};
        s.seg[0] = seg(matrix->m, matrix->y, 0);
        s.count = 1;
        s.cols = int(cols);
        s.type = matrix->m.type;
        nut::launch_qmatvec(s, matrix->x, nullptr, matrix->stream);
        cuda_check(cudaGetLastError(), "qmatvec launch");
        cuda_check(cudaMemcpyAsync(y, matrix->y, rows * 4, cudaMemcpyDeviceToHost,
                                   matrix->stream),
                   "copy y");
        cuda_check(cudaStreamSynchronize(matrix->stream), "synchronize");
    });
}

nut_status nut_model_create(const nut_model_view *view, int device,
                            nut_model **out) {
    return guarded([&] {
        if (view == nullptr || out == nullptr)
            raise(NUT_INVALID_ARGUMENT, "model: null argument");
        const nut_config &c = view->config;
        validate_config(c);
        if (view->quant_type != NUT_QUANT_INT8 && view->quant_type != NUT_QUANT_INT4)
            raise(NUT_INVALID_ARGUMENT, "model: unknown quant type");
        if (view->n_layers != c.layers || view->layers == nullptr)
            raise(NUT_INVALID_ARGUMENT, "quantized decode: layer count mismatch");
        if (view->embeddings == nullptr || view->final_norm == nullptr ||
            (!view->tied_embeddings && view->lm_head == nullptr))
            raise(NUT_INVALID_ARGUMENT, "model: null fp32 tensor");
        DeviceScope scope(device);
        auto m = std::make_unique<nut_model>();
        m->device = device;
        m->cfg = c;
        m->kv_heads = c.kv_heads == 0 ? c.heads : c.kv_heads;
        m->type = view->quant_type;
        m->tied = view->tied_embeddings != 0;
        cuda_check(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking),
                   "create stream");
        const size_t dim = size_t(c.dim), V = size_t(c.vocab_size);
        const int64_t kvd = m->kv_heads * c.head_dim;
        uint64_t bytes = (V * dim + dim + (m->tied ? 0 : V * dim)) * 4;
        m->embeddings = dev_alloc<float>(V * dim, "alloc embeddings");
        cuda_check(cudaMemcpy(m->embeddings, view->embeddings, V * dim * 4,
                              cudaMemcpyHostToDevice),
                   "copy embeddings");
        m->final_norm = dev_alloc<float>(dim, "alloc final norm");
        cuda_check(cudaMemcpy(m->final_norm, view->final_norm, dim * 4,
                              cudaMemcpyHostToDevice),
                   "copy final norm");
        if (!m->tied) {
            m->lm_head = dev_alloc<float>(V * dim, "alloc lm_head");
            cuda_check(cudaMemcpy(m->lm_head, view->lm_head, V * dim * 4,
                                  cudaMemcpyHostToDevice),
                       "copy lm_head");
        }
        for (int64_t l = 0; l < c.layers; l++) {
            const nut_layer_view &lv = view->layers[l];
            if (lv.attention_norm == nullptr || lv.ffn_norm == nullptr)
                raise(NUT_INVALID_ARGUMENT, "model: null norm weights");
            m->layers.emplace_back();
            DevLayer &d = m->layers.back();
            const int t = view->quant_type;
            d.q = upload(lv.query, c.dim, c.dim, t, "query");
            d.k = upload(lv.key, kvd, c.dim, t, "key");
            d.v = upload(lv.value, kvd, c.dim, t, "value");
            d.o = upload(lv.output, c.dim, c.dim, t, "output");
            d.gate = upload(lv.gate, c.ffn_dim, c.dim, t, "gate");
            d.up = upload(lv.up, c.ffn_dim, c.dim, t, "up");
            d.down = upload(lv.down, c.dim, c.ffn_dim, t, "down");
            for (const nut::DevQMatrix *q : {&d.q, &d.k, &d.v, &d.o, &d.gate,
                                             &d.up, &d.down})
                bytes += q->data_bytes() + q->scale_count() * 2;
            d.attention_norm = dev_alloc<float>(dim, "alloc norm");
            d.ffn_norm = dev_alloc<float>(dim, "alloc norm");
            cuda_check(cudaMemcpy(d.attention_norm, lv.attention_norm, dim * 4,
                                  cudaMemcpyHostToDevice),
                       "copy norm");
            cuda_check(cudaMemcpy(d.ffn_norm, lv.ffn_norm, dim * 4,
                                  cudaMemcpyHostToDevice),
                       "copy norm");
            bytes += 2 * dim * 4;
        }
        m->storage_bytes = bytes;
        /* RoPE table with the reference's exact fp32 values: frequency
         * 10000^(-pair/d) and cos/sin in double, rounded to fp32
         * (src/quant_model.cpp:26-37). */
        const size_t half = size_t(c.head_dim / 2), S = size_t(c.max_seq);
        std::vector<float> cs(S * half), sn(S * half);
        for (size_t p = 0; p < S; p++)
            for (size_t j = 0; j < half; j++) {
                const double f =
                    std::pow(10000.0, -double(2 * j) / double(c.head_dim));
                cs[p * half + j] = float(std::cos(double(p) * f));
                sn[p * half + j] = float(std::sin(double(p) * f));
            }
        m->rope_cos = dev_alloc<float>(S * half, "alloc rope");
        m->rope_sin = dev_alloc<float>(S * half, "alloc rope");
        cuda_check(cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4,
                              cudaMemcpyHostToDevice),
                   "copy rope");
        cuda_check(cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4,
                              cudaMemcpyHostToDevice),
                   "copy rope");
        *out = m.release();
    });
}

nut_status nut_model_destroy(nut_model *model) {
    return guarded([&] {
        if (model == nullptr)
            return;
        DeviceScope scope(model->device);
        delete model;
    });
}

nut_status nut_model_storage_bytes(const nut_model *model, uint64_t *bytes) {
    return guarded([&] {
        if (model == nullptr || bytes == nullptr)
            raise(NUT_INVALID_ARGUMENT, "model: null argument");
        *bytes = model->storage_bytes;
    });
}

nut_status nut_kv_create(nut_model *model, nut_kv **out) {
    return guarded([&] {
        if (model == nullptr || out == nullptr)
            raise(NUT_INVALID_ARGUMENT, "kv cache: null argument");
        DeviceScope scope(model->device);
        auto kv = std::make_unique<nut_kv>();
        kv->model = model;
        const nut_config &c = model->cfg;
        const size_t n = kv->cache_elements();
        kv->keys = dev_alloc<float>(n, "alloc keys");
        kv->values = dev_alloc<float>(n, "alloc values");
        cuda_check(cudaMemset(kv->keys, 0, n * 4), "clear keys");
        cuda_check(cudaMemset(kv->values, 0, n * 4), "clear values");
        const size_t kvd = size_t(model->kv_heads * c.head_dim);
        kv->hidden = dev_alloc<float>(size_t(c.dim), "alloc hidden");
        kv->q = dev_alloc<float>(size_t(c.dim), "alloc q");
        kv->k = dev_alloc<float>(kvd, "alloc k");
        kv->v = dev_alloc<float>(kvd, "alloc v");
        kv->ctx = dev_alloc<float>(size_t(c.dim), "alloc ctx");
        kv->gate = dev_alloc<float>(size_t(c.ffn_dim), "alloc gate");
        kv->up = dev_alloc<float>(size_t(c.ffn_dim), "alloc up");
        kv->logits = dev_alloc<float>(size_t(c.vocab_size), "alloc logits");
        kv->argmax_key = dev_alloc<unsigned long long>(1, "alloc argmax");
        kv->ids = dev_alloc<int32_t>(size_t(c.max_seq), "alloc ids");
        for (auto &e : kv->ev)
            cuda_check(cudaEventCreate(&e), "create event");
        *out = kv.release();
    });
}

nut_status nut_kv_destroy(nut_kv *kv) {
    return guarded([&] {
        if (kv == nullptr)
            return;
        DeviceScope scope(kv->model->device);
        delete kv;
    });
}

nut_status nut_kv_reset(nut_kv *kv) {
    return guarded([&] {
        if (kv == nullptr)
            raise(NUT_INVALID_ARGUMENT, "kv cache: null argument");
        kv->length = 0;
        kv->has_hidden = false;
    });
}

nut_status nut_kv_length(const nut_kv *kv, int64_t *length) {
    return guarded([&] {
        if (kv == nullptr || length == nullptr)
            raise(NUT_INVALID_ARGUMENT, "kv cache: null argument");
        *length = kv->length;
    });
}

nut_status nut_kv_set_length(nut_kv *kv, int64_t length) {
    return guarded([&] {
        if (kv == nullptr)
            raise(NUT_INVALID_ARGUMENT, "kv cache: null argument");
        if (length < 0 || length > kv->model->cfg.max_seq)
            raise(NUT_LENGTH_ERROR, "kv cache: context exceeds capacity");
        kv->length = length;
    });
}

nut_status nut_kv_memory_bytes(const nut_kv *kv, uint64_t *bytes) {
    return guarded([&] {
        if (kv == nullptr || bytes == nullptr)
            raise(NUT_INVALID_ARGUMENT, "kv cache: null argument");
        *bytes = uint64_t(kv->cache_elements()) * 2 * sizeof(float);
    });
}

nut_status nut_kv_read(const nut_kv *kv, int64_t layer, int64_t head,
                       int64_t position, float *key, float *value) {
    return guarded([&] {
        if (kv == nullptr)
            raise(NUT_INVALID_ARGUMENT, "kv cache: null argument");
        const nut_config &c = kv->model->cfg;
        if (layer < 0 || layer >= c.layers || head < 0 ||
            head >= kv->model->kv_heads || position < 0 || position >= c.max_seq)
            raise(NUT_OUT_OF_RANGE, "kv cache: index out of range");
        DeviceScope scope(kv->model->device);
        sync(kv->model);
        const size_t off =
            ((size_t(layer) * kv->model->kv_heads + size_t(head)) * c.max_seq +
             size_t(position)) * c.head_dim;
        if (key)
            cuda_check(cudaMemcpy(key, kv->keys + off, c.head_dim * 4,
                                  cudaMemcpyDeviceToHost),
                       "read key");
        if (value)
            cuda_check(cudaMemcpy(value, kv->values + off, c.head_dim * 4,
                                  cudaMemcpyDeviceToHost),
                       "read value");
    });
}

nut_status nut_decode_token(nut_model *model, nut_kv *kv, int32_t token,
                            float *hidden) {
    return guarded([&] {
        check_decode_args(model, kv, token);
        DeviceScope scope(model->device);
        enqueue_decode(model, kv, token, 0);
        if (hidden != nullptr) {
            cuda_check(cudaMemcpyAsync(hidden, kv->hidden, model->cfg.dim * 4,
                                       cudaMemcpyDeviceToHost, model->stream),
                       "copy hidden");
        }
        sync(model);
    });
}

nut_status nut_prefill(nut_model *model, nut_kv *kv, const int32_t *tokens,
                       int64_t n, float *hidden) {
    return guarded([&] {
        if (model == nullptr || kv == nullptr)
            raise(NUT_INVALID_ARGUMENT, "quantized prefill: null handle");
        if (tokens == nullptr || n <= 0 || n > model->cfg.max_seq)
            raise(NUT_INVALID_ARGUMENT, "quantized prefill: invalid prompt");
        kv->length = 0;
        kv->has_hidden = false;
        DeviceScope scope(model->device);
        for (int64_t i = 0; i < n; i++) {
            check_decode_args(model, kv, tokens[i]);
            enqueue_decode(model, kv, tokens[i], 0);
        }
        if (hidden != nullptr)
            cuda_check(cudaMemcpyAsync(hidden, kv->hidden, model->cfg.dim * 4,
                                       cudaMemcpyDeviceToHost, model->stream),
                       "copy hidden");
        sync(model);
    });
}

nut_status nut_logits(nut_model *model, nut_kv *kv, float *logits,
                      int32_t *argmax) {
    return guarded([&] {
        if (model == nullptr || kv == nullptr || kv->model != model)
            raise(NUT_INVALID_ARGUMENT, "logits: invalid handle");
        if (!kv->has_hidden)
            raise(NUT_INVALID_ARGUMENT, "logits: no decoded token");
        DeviceScope scope(model->device);
        enqueue_logits(model, kv);
        if (logits != nullptr)
            cuda_check(cudaMemcpyAsync(logits, kv->logits,
                                       model->cfg.vocab_size * 4,
                                       cudaMemcpyDeviceToHost, model->stream),
                       "copy logits");
        unsigned long long key = 0;
        cuda_check(cudaMemcpyAsync(&key, kv->argmax_key, sizeof key,
                                   cudaMemcpyDeviceToHost, model->stream),
                   "copy argmax");
        sync(model);
        if (argmax != nullptr)
            *argmax = int32_t(~uint32_t(key & 0xffffffffull));
    });
}

nut_status nut_generate_greedy(nut_model *model, nut_kv *kv,
                               const int32_t *prompt, int64_t n,
                               int64_t max_tokens, int32_t stop_at_eos,
                               int32_t *ids, int64_t *n_generated,
                               float *logits, nut_generation_stats *stats) {
    return guarded([&] {
        if (model == nullptr || kv == nullptr || kv->model != model)
            raise(NUT_INVALID_ARGUMENT, "generation: invalid handle");
        const nut_config &c = model->cfg;
        if (prompt == nullptr || n <= 0 || n > c.max_seq)
            raise(NUT_INVALID_ARGUMENT, "generation: invalid prompt length");
        if (max_tokens < 0 || (max_tokens > 0 && ids == nullptr))
            raise(NUT_INVALID_ARGUMENT, "generation: invalid output");
        for (int64_t i = 0; i < n; i++)
            if (prompt[i] < 0 || prompt[i] >= c.vocab_size)
                raise(NUT_OUT_OF_RANGE, "quantized decode: token out of range");
        DeviceScope scope(model->device);
        cudaStream_t s = model->stream;
        kv->length = 0;
        kv->has_hidden = false;
        cuda_check(cudaEventRecord(kv->ev[0], s), "event");
        for (int64_t i = 0; i < n; i++)
            enqueue_decode(model, kv, prompt[i], 0);
        cuda_check(cudaEventRecord(kv->ev[1], s), "event");
        /* steps while generated < max_tokens and length < capacity */
        const int64_t steps = std::min<int64_t>(max_tokens, c.max_seq - n);
        int64_t produced = 0;
        for (int64_t step = 0; step < steps; step++) {
            enqueue_logits(model, kv);
            if (logits != nullptr)
                cuda_check(cudaMemcpyAsync(logits + step * c.vocab_size,
                                           kv->logits, c.vocab_size * 4,
                                           cudaMemcpyDeviceToHost, s),
                           "copy logits");
            if (stop_at_eos) {
                unsigned long long key = 0;
                cuda_check(cudaMemcpyAsync(&key, kv->argmax_key, sizeof key,
                                           cudaMemcpyDeviceToHost, s),
                           "copy argmax");
                sync(model);
                const int32_t token = int32_t(~uint32_t(key & 0xffffffffull));
                if (token == c.eos_token)
                    break;
                ids[produced] = token;
            }
            enqueue_decode(model, kv, -1, int(step));
            produced++;
        }
        cuda_check(cudaEventRecord(kv->ev[2], s), "event");
        if (!stop_at_eos && produced > 0)
            cuda_check(cudaMemcpyAsync(ids, kv->ids, size_t(produced) * 4,
                                       cudaMemcpyDeviceToHost, s),
                       "copy ids");
        sync(model);
        if (n_generated != nullptr)
            *n_generated = produced;
        if (stats != nullptr) {
            float a = 0.0f, b = 0.0f;
            cuda_check(cudaEventElapsedTime(&a, kv->ev[0], kv->ev[1]), "elapsed");
            cuda_check(cudaEventElapsedTime(&b, kv->ev[1], kv->ev[2]), "elapsed");
            stats->prefill_tokens = n;
            stats->generated_tokens = produced;
            stats->prefill_seconds = double(a) * 1e-3;
            stats->decode_seconds = double(b) * 1e-3;
        }
    });
}

} // extern "C"
